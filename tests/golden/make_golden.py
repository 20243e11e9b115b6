"""Generate the golden fixtures in this directory from the reference project itself.

Run in a container where the reference checkout is readable (it is not needed,
and not read, anywhere else)::

    REF=/path/to/Triton-MuonAdamW python tests/golden/make_golden.py

It imports the reference package ``triton_muon_adamw`` from
``$REF/MuonAdamW package`` and records, on CPU:

* ``wrapper_*.pt`` -- ``PyTorchMuonAdamW`` (optimizer.py:178-260: fused
  ``torch.optim.AdamW`` + ``torch.optim.Muon``) over seeded parameter sets,
  several steps, with the per-step gradients and the parameters after each step.
* ``triton_adamw.pt`` -- the reference ``TritonAdamW`` (triton_adam.py:106-161)
  executed by the Triton interpreter (``TRITON_INTERPRET=1``), including a
  parameter whose gradient is ``None`` (the branch-global step count).
* ``triton_muon_glue.pt`` -- the reference ``TritonMuon.step`` (triton_muon.py:414-448)
  and its ``muon_step`` eager code (momentum EMA, Nesterov, bf16 cast,
  transpose, Frobenius normalisation, decay and update: :346-372), float32
  and bf16 parameters, with the Newton-Schulz call (:313-325) replaced by a
  recorder that returns its input: the X each step hands to Newton-Schulz,
  the momentum and the parameters after each step.

The reference's Newton-Schulz kernels (triton_muon.py:35-310) cannot run in the
Triton 3.6 interpreter (no bf16 there), so no Triton Muon golden exists; the
Muon rounding points are pinned through the wrapper goldens, whose
``torch.optim.Muon`` rounds at the same places.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle.muon_adamw_oracle import gpt_c1_shapes  # noqa: E402

MUON_TORCH = dict(lr=1e-3, beta=0.95, eps=1e-7, weight_decay=0.1, coeffs=(3.4445, -4.7750, 2.0315),
                  nesterov=True, ns_steps=5, adjust_lr_fn="original")
ADAM_C1 = dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-7, weight_decay=0.01)


def _ref_pkg():
    ref = os.environ.get("REF")
    if not ref:
        raise SystemExit("set REF to the reference checkout")
    sys.path.insert(0, str(Path(ref) / "MuonAdamW package"))
    import triton_muon_adamw as R  # noqa: PLC0415
    return R


def _params(shapes, gen, std, dtype=torch.float32):
    return [torch.nn.Parameter((torch.randn(s, generator=gen) * std).to(dtype)) for s in shapes]


def wrapper_case(R, name, adam_shapes, muon_shapes, *, steps, muon, adam, seed, grad_std=1e-3,
                 param_std=0.02, zero_params=False, dtype=torch.float32):
    gen = torch.Generator().manual_seed(seed)
    adam_p = _params(adam_shapes, gen, param_std, dtype)
    muon_p = _params(muon_shapes, gen, param_std, dtype)
    if zero_params:
        for p in muon_p:
            p.data.zero_()
    init = [p.detach().clone() for p in adam_p + muon_p]
    opt = R.PyTorchMuonAdamW({"adam": adam_p, "muon": muon_p},
                             muon_config=R.MuonConfig(**muon), adam_config=R.AdamConfig(**adam),
                             parameter_split="explicit")
    grads, after = [], []
    ggen = torch.Generator().manual_seed(seed + 1000)
    for _ in range(steps):
        gs = [(torch.randn(p.shape, generator=ggen) * grad_std).to(dtype) for p in adam_p + muon_p]
        for p, g in zip(adam_p + muon_p, gs):
            p.grad = g.clone()
        opt.step()
        grads.append(gs)
        after.append([p.detach().clone() for p in adam_p + muon_p])
    out = dict(name=name, adam_shapes=adam_shapes, muon_shapes=muon_shapes, muon=muon, adam=adam,
               init=init, grads=grads, after=after, steps=steps)
    torch.save(out, HERE / f"wrapper_{name}.pt")
    return out


def triton_adamw_case(R):
    from triton_muon_adamw.adamw import TritonAdamW  # noqa: PLC0415
    gen = torch.Generator().manual_seed(7)
    shapes = [(1,), (7,), (513,), (3, 700), (4096,), (1, 33)]
    params = _params(shapes, gen, 0.02)
    init = [p.detach().clone() for p in params]
    cfg = dict(lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    opt = TritonAdamW(params, lr=cfg["lr"], betas=cfg["betas"], weight_decay=cfg["weight_decay"], eps=cfg["eps"])
    grads, after = [], []
    for step in range(5):
        gs = []
        for i, p in enumerate(params):
            if i == 2 and step == 1:          # a missing gradient: parameter skipped, step count still advances
                p.grad = None
                gs.append(None)
                continue
            g = torch.randn(p.shape, generator=gen) * 1e-2
            p.grad = g.clone()
            gs.append(g)
        opt.step()
        grads.append(gs)
        after.append([p.detach().clone() for p in params])
    torch.save(dict(shapes=shapes, cfg=cfg, init=init, grads=grads, after=after), HERE / "triton_adamw.pt")


def triton_muon_glue_case(R):
    import triton_muon_adamw.muon.triton_muon as TM  # noqa: PLC0415
    seen = []

    def recorder(X, a, b, c, out):   # stands in for the Triton Newton-Schulz step
        seen.append(X.detach().clone())
        out.copy_(X)

    real = TM.newton_shultz_step
    TM.newton_shultz_step = recorder
    cases = []
    try:
        shapes = [(33, 70), (70, 33), (64, 64), (5, 3)]
        for dtype in (torch.float32, torch.bfloat16):
            for nesterov in (True, False):
                gen = torch.Generator().manual_seed(len(cases) + 40)
                params = _params(shapes, gen, 0.02, dtype)
                init = [p.detach().clone() for p in params]
                opt = TM.TritonMuon(params, lr=2e-2, weight_decay=0.1, coeffs=MUON_TORCH["coeffs"],
                                    nesterov=nesterov, beta=0.95, ns_steps=2, eps=1e-7)
                grads, xs, moms, after = [], [], [], []
                for _ in range(2):
                    gs = [(torch.randn(p.shape, generator=gen) * 1e-2).to(dtype) for p in params]
                    for p, g in zip(params, gs):
                        p.grad = g.clone()
                    seen.clear()
                    opt.step()
                    xs.append(seen[0::2])        # the first Newton-Schulz input of each matrix
                    grads.append(gs)
                    moms.append([opt.momentum[p].clone() for p in params])
                    after.append([p.detach().clone() for p in params])
                cases.append(dict(dtype=str(dtype), nesterov=nesterov, shapes=shapes, lr=2e-2, weight_decay=0.1,
                                  beta=0.95, eps=1e-7, init=init, grads=grads, x=xs, momentum=moms, after=after))
    finally:
        TM.newton_shultz_step = real
    torch.save(cases, HERE / "triton_muon_glue.pt")


def main():
    R = _ref_pkg()
    triton_adamw_case(R)
    triton_muon_glue_case(R)
    # A tiny GPT with the C1 layout (tied embedding), two steps.
    a, m = gpt_c1_shapes(d=32, layers=2, ffn=128, vocab=256)
    wrapper_case(R, "gpt_tiny", a, m, steps=2, muon=MUON_TORCH, adam=ADAM_C1, seed=0)
    # Ragged / tall / degenerate Muon shapes, Nesterov off, ns_steps 6.
    ragged = [(1, 7), (7, 1), (5, 3), (33, 70), (130, 66), (64, 64), (200, 129)]
    wrapper_case(R, "ragged", [(5,), (130,)], ragged, steps=2,
                 muon=dict(MUON_TORCH, nesterov=False, ns_steps=6), adam=ADAM_C1, seed=3, grad_std=1.0)
    # lr=1, wd=0, zero parameters: the parameters after one step are exactly
    # -scaled_lr * (orthogonalised update), pinning Newton-Schulz output directly.
    wrapper_case(R, "ns_direct", [(4,)], [(96, 160), (256, 128), (128, 128)], steps=1,
                 muon=dict(MUON_TORCH, lr=1.0, weight_decay=0.0), adam=ADAM_C1, seed=5, zero_params=True)
    wrapper_case(R, "match_rms", [(16,)], [(48, 80), (80, 48)], steps=2,
                 muon=dict(MUON_TORCH, adjust_lr_fn="match_rms_adamw"), adam=ADAM_C1, seed=9)
    # bf16 parameters: the wrapper keeps its AdamW moments in bf16, the Triton path in fp32.
    a, m = gpt_c1_shapes(d=32, layers=1, ffn=128, vocab=128)
    wrapper_case(R, "bf16", a, m + [(96, 40)], steps=2, muon=MUON_TORCH, adam=ADAM_C1, seed=11, dtype=torch.bfloat16)
    print("wrote", sorted(p.name for p in HERE.glob("*.pt")))


if __name__ == "__main__":
    main()
