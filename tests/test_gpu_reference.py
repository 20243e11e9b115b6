"""Parity against the reference itself, run on the B200 next to ours, on the BASELINE configs.

The reference package is imported unmodified from ``baseline/_ref``
(``tests/reference_pkg.py``); a missing install fails these tests rather than
skipping them.  Reference paths are relative to its ``MuonAdamW package/``.

* C1 (17M GPT, d=512, 4 layers, vocab 8192 tied): ``MuonAdamW`` against the
  reference's ``PyTorchMuonAdamW`` (``torch.optim`` AdamW(fused) + Muon,
  ``triton_muon_adamw/optimizer.py:178-260``) and the reference's own Triton
  ``MuonAdamW`` (``optimizer.py:70-175``) over 300 steps on fixed gradients,
  the form of the reference's own check (``benchmarks/muon_adamw_benchmark.py:117-134``:
  hundreds of steps, then atol/rtol 1e-2 on every parameter; AdamW parameters
  at ``benchmarks/adam_benchmark.py:111-115``'s 1e-4 / 1e-3).  The drift of
  each pair is recorded at checkpoints (``MAD_PARITY_LOG``, when set, names a
  JSON file to write it to) and bounded: the Muon parameters' displacement
  from their start differs from the wrapper's by < 3e-2 relative Frobenius at
  every checkpoint, the per-step bar of the folded normalisation.
* The reference's Triton Newton-Schulz path (``TritonMuon.step``,
  ``muon/triton_muon.py:327-448``, kernels ``:35-310``) against ours on the
  four 8B matrix shapes: one step each on identical inputs.
* C3 batches: 8 and 32 matrices of 4096x14336 (and 14336x4096) in one plan,
  ns_steps 5 and 6, against the oracle's folded-normalisation restatement
  (``oracle.muon_adamw_oracle.orthogonalize(normalize="fold")``) evaluated in
  float64 on the GPU, and each matrix bit-identical to its single-matrix run.
"""

from __future__ import annotations

import json
import math
import os

import pytest
import torch

from oracle.muon_adamw_oracle import bf16_round, gpt_c1_shapes, orthogonalize, scaled_lr
from reference_pkg import load_reference

pytestmark = pytest.mark.gpu

COEFFS = (3.4445, -4.7750, 2.0315)     # torch.optim.Muon's coefficients (the wrapper forwards none)
C1_MUON = dict(lr=1e-3, beta=0.95, eps=1e-7, weight_decay=0.1, coeffs=COEFFS, nesterov=True, ns_steps=5,
               adjust_lr_fn="original")
C1_ADAM = dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-7, weight_decay=0.01)


def _params(init, dev):
    return [torch.nn.Parameter(t.clone().to(dev)) for t in init]


def _max_abs(a, b):
    return max(float((x.detach() - y.detach()).abs().max()) for x, y in zip(a, b))


def _disp_err(p, q, init):
    """Relative Frobenius difference of two runs' displacements from the common start."""
    num = math.sqrt(sum(float(((x.detach() - y.detach()).double() ** 2).sum()) for x, y in zip(p, q)))
    den = math.sqrt(sum(float(((y.detach() - i).double() ** 2).sum()) for y, i in zip(q, init)))
    return num / den


def test_c1_gpt_many_steps_vs_reference_wrapper_and_reference_triton(cuda_device):
    from triton_muon_adamw import AdamConfig, MuonAdamW, MuonConfig
    R = load_reference()
    adam_shapes, muon_shapes = gpt_c1_shapes()
    gen = torch.Generator(device=cuda_device).manual_seed(0)
    init = [torch.empty(s, device=cuda_device).normal_(0.0, 0.02, generator=gen) for s in adam_shapes + muon_shapes]
    ggen = torch.Generator(device=cuda_device).manual_seed(1)
    grads = [torch.empty(s, device=cuda_device).normal_(0.0, 1e-3, generator=ggen) for s in adam_shapes + muon_shapes]
    na = len(adam_shapes)
    assert sum(t.numel() for t in init) > 16_000_000

    ours, wrap, rtri = _params(init, cuda_device), _params(init, cuda_device), _params(init, cuda_device)
    o = MuonAdamW({"adam": ours[:na], "muon": ours[na:]}, muon_config=MuonConfig(**C1_MUON),
                  adam_config=AdamConfig(**C1_ADAM), parameter_split="explicit")
    w = R.PyTorchMuonAdamW({"adam": wrap[:na], "muon": wrap[na:]}, muon_config=R.MuonConfig(**C1_MUON),
                           adam_config=R.AdamConfig(**C1_ADAM), parameter_split="explicit")
    t = R.MuonAdamW({"adam": rtri[:na], "muon": rtri[na:]}, muon_config=R.MuonConfig(**C1_MUON),
                    adam_config=R.AdamConfig(**C1_ADAM), parameter_split="explicit")
    for ps in (ours, wrap, rtri):
        for p, g in zip(ps, grads):
            p.grad = g.clone()

    checkpoints, drift = {1, 2, 10, 50, 100, 200, 300}, []
    for step in range(1, 301):
        o.step()
        w.step()
        t.step()
        if step not in checkpoints:
            continue
        torch.cuda.synchronize()
        rec = {"step": step,
               "adam_max_abs_vs_wrapper": _max_abs(ours[:na], wrap[:na]),
               "muon_max_abs_vs_wrapper": _max_abs(ours[na:], wrap[na:]),
               "muon_max_abs_vs_ref_triton": _max_abs(ours[na:], rtri[na:]),
               "ref_triton_muon_max_abs_vs_wrapper": _max_abs(rtri[na:], wrap[na:]),
               "muon_disp_rel_vs_wrapper": _disp_err(ours[na:], wrap[na:], init[na:]),
               "muon_disp_rel_vs_ref_triton": _disp_err(ours[na:], rtri[na:], init[na:]),
               "ref_triton_disp_rel_vs_wrapper": _disp_err(rtri[na:], wrap[na:], init[na:])}
        drift.append(rec)
        for p, q in zip(ours[:na], wrap[:na]):
            torch.testing.assert_close(p.detach(), q.detach(), atol=1e-4, rtol=1e-3)
        for p, q, r in zip(ours[na:], wrap[na:], rtri[na:]):
            torch.testing.assert_close(p.detach(), q.detach(), atol=1e-2, rtol=1e-2)
            torch.testing.assert_close(p.detach(), r.detach(), atol=1e-2, rtol=1e-2)
        assert rec["muon_disp_rel_vs_wrapper"] < 3e-2, rec
        assert rec["muon_disp_rel_vs_ref_triton"] < 3e-2, rec
    if os.environ.get("MAD_PARITY_LOG"):
        with open(os.environ["MAD_PARITY_LOG"], "w") as f:
            json.dump({"config": "C1 17M GPT, fixed gradients", "drift": drift}, f, indent=1)
    print(json.dumps(drift))
    assert o.device_status() == 0


@pytest.mark.parametrize("shape", [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)])
def test_reference_triton_newton_schulz_on_8b_shapes(cuda_device, shape):
    """One TritonMuon.step of the reference's Triton kernels against one of ours, identical inputs."""
    from triton_muon_adamw.muon import TritonMuon
    R = load_reference()
    RefMuon = R.muon.triton_muon.TritonMuon
    gen = torch.Generator(device=cuda_device).manual_seed(sum(shape))
    g = torch.empty(shape, device=cuda_device).normal_(0.0, 1e-3, generator=gen)
    p0 = torch.empty(shape, device=cuda_device).normal_(0.0, 0.02, generator=gen)
    results = {}
    for name, cls in (("ours", TritonMuon), ("ref", RefMuon)):
        # the orthogonalised update itself (lr=1, wd=0, zero parameter) ...
        pz = torch.nn.Parameter(torch.zeros(shape, device=cuda_device))
        pz.grad = g.clone()
        cls([pz], lr=1.0, weight_decay=0.0, coeffs=COEFFS, nesterov=True, ns_steps=5).step()
        # ... and a realistic step on a seeded parameter
        pr = torch.nn.Parameter(p0.clone())
        pr.grad = g.clone()
        cls([pr], lr=1e-3, weight_decay=0.1, coeffs=COEFFS, nesterov=True, ns_steps=5).step()
        results[name] = (-pz.detach() / scaled_lr(1.0, shape, "original"), pr.detach())
    (o_ours, p_ours), (o_ref, p_ref) = results["ours"], results["ref"]
    err = float((o_ours - o_ref).norm() / o_ref.norm())
    assert err < 2e-2, f"{shape}: orthogonalised update vs reference Triton, rel Frobenius {err:.3e}"
    torch.testing.assert_close(p_ours, p_ref, atol=1e-2, rtol=1e-2)
    print(json.dumps({"shape": list(shape), "update_rel_frobenius_vs_ref_triton": err}))


def _fold_orthogonalize_gpu(u, coeffs, ns_steps, eps):
    """``oracle.muon_adamw_oracle.orthogonalize(normalize="fold")`` restated on the GPU in float64.

    Same rounding points: bf16 cast and transpose-to-wide, the bf16 norm of X
    clamped at bf16(eps), s = float32(1/norm) folded into the first Gram (s²)
    and the first update (s), every product accumulated in float64 and
    rounded to bf16 once.
    """
    a, b, c = coeffs
    x = u.to(torch.bfloat16).float()
    tall = x.shape[0] > x.shape[1]
    if tall:
        x = x.t().contiguous()
    xd = x.double()
    norm = float(torch.tensor(math.sqrt(float((xd * xd).sum()))).to(torch.bfloat16).float())
    norm = max(norm, float(torch.tensor(eps).to(torch.bfloat16).float()))
    s = float(torch.tensor(1.0, dtype=torch.float32) / torch.tensor(norm, dtype=torch.float32))

    def r(t):
        return t.float().to(torch.bfloat16).double()

    for it in range(ns_steps):
        s1 = s if it == 0 else 1.0
        A = r((s1 * s1) * (xd @ xd.t()))
        B = r(b * A + c * (A @ A))
        xd = r(s1 * (a * xd + B @ xd))
    out = xd.float()
    return out.t() if tall else out


def test_gpu_fold_restatement_matches_the_cpu_oracle(cuda_device):
    gen = torch.Generator().manual_seed(9)
    for shape in [(96, 160), (200, 64)]:
        u = torch.randn(shape, generator=gen) * 1e-3
        want = orthogonalize(u, COEFFS, 5, 1e-7, normalize="fold")
        got = _fold_orthogonalize_gpu(u.to(cuda_device), COEFFS, 5, 1e-7).cpu()
        assert float((got - want).norm() / want.norm()) < 1e-3, shape


def _one_step_updates(shapes_grads, ns_steps, dev):
    """Orthogonalised updates of one TritonMuon step over all matrices in one plan (u = gradient)."""
    from triton_muon_adamw.muon import TritonMuon
    ps = []
    for g in shapes_grads:
        p = torch.nn.Parameter(torch.zeros(g.shape, device=dev))
        p.grad = g
        ps.append(p)
    opt = TritonMuon(ps, lr=1.0, weight_decay=0.0, coeffs=COEFFS, nesterov=False, beta=0.0, ns_steps=ns_steps,
                     eps=1e-7)
    opt.step()
    torch.cuda.synchronize()
    assert opt.device_status() == 0
    return [-p.detach() / scaled_lr(1.0, p.shape, "original") for p in ps]


@pytest.mark.parametrize("shape,batch,ns_steps", [((4096, 14336), 8, 5), ((4096, 14336), 8, 6),
                                                  ((4096, 14336), 32, 5), ((14336, 4096), 8, 6)])
def test_c3_newton_schulz_batches_vs_oracle_fold(cuda_device, shape, batch, ns_steps):
    gen = torch.Generator(device=cuda_device).manual_seed(batch * 10 + ns_steps)
    # C3 inputs: bf16 N(0,1) matrices; with beta=0 and no Nesterov the momentum is the gradient itself.
    grads = [bf16_round(torch.empty(shape, device=cuda_device).normal_(0.0, 1.0, generator=gen))
             for _ in range(batch)]
    outs = _one_step_updates(grads, ns_steps, cuda_device)
    oracle_idx = list(range(batch)) if batch <= 8 else [0, 11, 22, batch - 1]
    for i in oracle_idx:
        want = _fold_orthogonalize_gpu(grads[i], COEFFS, ns_steps, 1e-7)
        err = float((outs[i] - want).norm() / want.norm())
        assert err < 1.2e-2, f"matrix {i} of {batch} {shape} ns={ns_steps}: vs oracle fold {err:.3e}"
    for i in (0, batch // 2, batch - 1):
        alone = _one_step_updates([grads[i]], ns_steps, cuda_device)[0]
        assert torch.equal(alone, outs[i]), f"matrix {i}: batched result differs from its single-matrix run"
