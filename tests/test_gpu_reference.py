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
        # The reference's Triton kernels round a, b and their products to bf16 (see the NS tests
        # below), which moves them further from torch.optim.Muon than ours: ours must stay at least
        # as close to the wrapper as the reference's own Triton path is.
        assert rec["muon_disp_rel_vs_wrapper"] <= rec["ref_triton_disp_rel_vs_wrapper"], rec
    if os.environ.get("MAD_PARITY_LOG"):
        with open(os.environ["MAD_PARITY_LOG"], "w") as f:
            json.dump({"config": "C1 17M GPT, fixed gradients", "drift": drift}, f, indent=1)
    print(json.dumps(drift))
    assert o.device_status() == 0


def _orthogonalize_gpu(u, coeffs, ns_steps, eps, normalize="fold", triton_scalars=False):
    """``oracle.muon_adamw_oracle.orthogonalize`` restated on the GPU in float64.

    Same rounding points: bf16 cast and transpose-to-wide, the bf16 norm of X
    clamped at bf16(eps), every product accumulated in float64 and rounded to
    bf16 once.  ``normalize="fold"``: s = float32(1/norm) folded into the first
    Gram (s²) and the first update (s) -- the CUDA path's ordering.
    ``"reference"``: X/norm rounded to bf16 first.  ``triton_scalars``: the
    reference Triton kernels' bf16 rounding of a, b and of a·X, b·A
    (``oracle.muon_adamw_oracle.ns_iteration``).
    """
    a, b, c = coeffs
    x = u.to(torch.bfloat16).float()
    tall = x.shape[0] > x.shape[1]
    if tall:
        x = x.t().contiguous()
    xd = x.double()
    norm = float(torch.tensor(math.sqrt(float((xd * xd).sum()))).to(torch.bfloat16).float())
    norm = max(norm, float(torch.tensor(eps).to(torch.bfloat16).float()))

    def r(t):
        return t.float().to(torch.bfloat16).double()

    if normalize == "fold":
        s = float(torch.tensor(1.0, dtype=torch.float32) / torch.tensor(norm, dtype=torch.float32))
    else:
        xd = r(xd.float() / torch.tensor(norm, dtype=torch.float32))
        s = 1.0
    if triton_scalars:
        a_h, b_h = float(bf16_round(torch.tensor(a))), float(bf16_round(torch.tensor(b)))
        c_32 = float(torch.tensor(c, dtype=torch.float32))
    for it in range(ns_steps):
        s1 = s if it == 0 else 1.0
        A = r((s1 * s1) * (xd @ xd.t()))
        if triton_scalars:
            B = r(r(b_h * A) + c_32 * (A @ A))
            xd = r(r(a_h * xd) + B @ xd)
        else:
            B = r(b * A + c * (A @ A))
            xd = r(s1 * (a * xd + B @ xd))
    out = xd.float()
    return out.t() if tall else out


def _fold_orthogonalize_gpu(u, coeffs, ns_steps, eps):
    return _orthogonalize_gpu(u, coeffs, ns_steps, eps, normalize="fold")


def _frac_equal(model, got):
    """Fraction of elements where the float64 model, rounded to bf16, equals the kernel's bf16 output."""
    return float((model.float().to(torch.bfloat16) == got).float().mean())


def test_reference_triton_kernels_round_their_scalar_coefficients_to_bf16(cuda_device):
    """The reference's three NS kernels (triton_muon.py:35-310), run on the GPU, against float64 models.

    ``ns_kernel_2`` forms ``b_coeff * A`` and ``ns_kernel_3`` ``a_coeff * X``
    from a float ``tl.constexpr`` and a bf16 block: Triton keeps such products
    in bf16, so the coefficient and the product are rounded to bf16 before the
    float32 accumulator is added.  The model with that rounding
    (``oracle.ns_iteration(triton_scalars=True)``) reproduces the kernels'
    outputs bit for bit on nearly every element; the exact-coefficient model
    does not.  This pins the oracle to the reference's Triton kernels directly.
    """
    R = load_reference()
    T = R.muon.triton_muon
    a, b, c = COEFFS
    gen = torch.Generator(device=cuda_device).manual_seed(5)
    m, n = 320, 704
    x = (torch.randn(m, n, device=cuda_device, generator=gen) / math.sqrt(m * n) * 1.3).to(torch.bfloat16)
    A = torch.empty(m, m, device=cuda_device, dtype=torch.bfloat16)
    B = torch.empty_like(A)
    X2 = torch.empty_like(x)
    T.solve_ns_kernel_1(x, A)
    T.solve_ns_kernel_2(A, b, c, B)
    T.solve_ns_kernel_3(x, B, a, X2)
    torch.cuda.synchronize()
    xd, Ad, Bd = x.double(), A.double(), B.double()
    a_h, b_h = float(bf16_round(torch.tensor(a))), float(bf16_round(torch.tensor(b)))
    c_32 = float(torch.tensor(c, dtype=torch.float32))

    def r(t):
        return t.float().to(torch.bfloat16).double()

    fr = {"gram": _frac_equal(xd @ xd.t(), A),
          "poly_triton_scalars": _frac_equal(r(b_h * Ad) + c_32 * (Ad @ Ad), B),
          "poly_exact": _frac_equal(b * Ad + c * (Ad @ Ad), B),
          "update_triton_scalars": _frac_equal(r(a_h * xd) + Bd @ xd, X2),
          "update_exact": _frac_equal(a * xd + Bd @ xd, X2)}
    print(json.dumps({"bit_equal_fraction": fr}))
    assert fr["gram"] > 0.99, fr
    assert fr["poly_triton_scalars"] > 0.99 and fr["update_triton_scalars"] > 0.99, fr
    assert fr["poly_exact"] < fr["poly_triton_scalars"] - 0.05, fr
    assert fr["update_exact"] < fr["update_triton_scalars"] - 0.05, fr


@pytest.mark.parametrize("shape", [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)])
def test_reference_triton_newton_schulz_on_8b_shapes(cuda_device, shape):
    """One TritonMuon.step of the reference's Triton kernels against one of ours, identical inputs.

    * the reference's update vs the oracle's model of its Triton path
      (reference normalisation order, bf16-rounded scalars): < 1.2e-2 -- the
      oracle is pinned to the reference kernels at full 8B size;
    * ours vs the oracle with the stated coefficients (folded normalisation):
      < 1.2e-2;
    * a realistic step (lr 1e-3, wd 0.1, seeded parameter): ours equals the
      reference's within its Muon tolerance, atol/rtol 1e-2 (README.md:52).
    The remaining ours-vs-reference difference on the bare update is the
    reference's bf16 coefficient rounding; it is recorded, not bounded.
    """
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
    # First step from zero momentum: mom = 0.05 g; Nesterov u = g + 0.95 (mom - g), float32 as both compute it.
    mom = g * torch.tensor(1.0 - 0.95, dtype=torch.float32).item()
    u = g + (mom - g) * 0.95
    m_tri = _orthogonalize_gpu(u, COEFFS, 5, 1e-7, normalize="reference", triton_scalars=True)
    m_fold = _orthogonalize_gpu(u, COEFFS, 5, 1e-7, normalize="fold")

    def rel(x, y):
        return float((x - y).norm() / y.norm())

    rec = {"shape": list(shape), "ref_triton_vs_oracle_triton_model": rel(o_ref, m_tri),
           "ours_vs_oracle_fold": rel(o_ours, m_fold), "ours_vs_ref_triton": rel(o_ours, o_ref),
           "oracle_fold_vs_oracle_triton_model": rel(m_fold, m_tri)}
    print(json.dumps(rec))
    assert rec["ref_triton_vs_oracle_triton_model"] < 1.2e-2, rec
    assert rec["ours_vs_oracle_fold"] < 1.2e-2, rec
    torch.testing.assert_close(p_ours, p_ref, atol=1e-2, rtol=1e-2)


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
