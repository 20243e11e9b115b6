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


def _params(shapes, gen, std):
    return [torch.nn.Parameter(torch.randn(s, generator=gen) * std) for s in shapes]


def wrapper_case(R, name, adam_shapes, muon_shapes, *, steps, muon, adam, seed, grad_std=1e-3,
                 param_std=0.02, zero_params=False):
    gen = torch.Generator().manual_seed(seed)
    adam_p = _params(adam_shapes, gen, param_std)
    muon_p = _params(muon_shapes, gen, param_std)
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
        gs = [torch.randn(p.shape, generator=ggen) * grad_std for p in adam_p + muon_p]
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


def main():
    R = _ref_pkg()
    triton_adamw_case(R)
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
    print("wrote", sorted(p.name for p in HERE.glob("*.pt")))


if __name__ == "__main__":
    main()
