"""bf16 parameters on the CUDA path, against the oracle and the reference's bf16 golden (needs a B200).

With bf16 parameters the reference's Triton path keeps the AdamW moments in
float32 (triton_adam.py:128-130) and stores the updated parameter in bf16;
its Muon branch keeps the momentum in the parameter dtype, so every eager op
of the momentum/Nesterov glue and of the parameter update rounds to bf16
(triton_muon.py:346-349, 368-372).  The oracle restates exactly those
rounding points; the kernels compute each float32 intermediate with the same
operations, so results agree to the bf16 rounding of float32 values that
match to a few ulps (at most one bf16 ulp apart, almost always identical).
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import load_golden
from oracle.muon_adamw_oracle import (OracleMuonAdamW, adamw_bias_corrections, adamw_update_, muon_momentum_,
                                      orthogonalize, scaled_lr, to_wide_bf16)

pytestmark = pytest.mark.gpu

COEFFS = (3.4445, -4.7750, 2.0315)
BF16_ULP = 2.0 ** -7    # relative spacing of bf16 values (8 significant bits)


def _within_one_ulp(got: torch.Tensor, want: torch.Tensor, what: str) -> None:
    """Bit-equal except for values one bf16 ulp apart (a float32 tie broken the other way); few of those."""
    got, want = got.float().cpu(), want.float().cpu()
    diff = (got - want).abs()
    assert bool((diff <= want.abs() * BF16_ULP + 1e-30).all()), f"{what}: max diff {float(diff.max()):.3e}"
    n_diff = int((diff > 0).sum())
    assert n_diff <= max(2, diff.numel() // 1000), f"{what}: {n_diff} of {diff.numel()} values differ"


# ----------------------------------------------------------------- AdamW
@pytest.mark.parametrize("sizes", [[1, 7, 4096, 4097, 100003], [65536, 3, 9000]])
def test_adamw_bf16_params_vs_oracle(cuda_device, sizes):
    from triton_muon_adamw.adamw import TritonAdamW
    gen = torch.Generator().manual_seed(sum(sizes))
    cpu = [(torch.randn(s, generator=gen) * 0.02).to(torch.bfloat16) for s in sizes]
    params = [torch.nn.Parameter(t.clone().to(cuda_device)) for t in cpu]
    opt = TritonAdamW(params, lr=3e-4, betas=(0.9, 0.999), weight_decay=0.01, eps=1e-8)
    ms = [torch.zeros(s) for s in sizes]
    vs = [torch.zeros(s) for s in sizes]
    for step in range(1, 4):
        grads = [(torch.randn(s, generator=gen) * 1e-2).to(torch.bfloat16) for s in sizes]
        for p, g in zip(params, grads):
            p.grad = g.to(cuda_device)
        opt.step()
        b1, b2 = adamw_bias_corrections(0.9, 0.999, step)
        for t, g, m, v in zip(cpu, grads, ms, vs):
            adamw_update_(t, g, m, v, lr=3e-4, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, bias1=b1,
                          bias2=b2)
    for p, t, m, v in zip(params, cpu, ms, vs):
        assert p.dtype == torch.bfloat16
        _within_one_ulp(p.detach(), t, f"param {t.numel()}")
        torch.testing.assert_close(opt.m[p].cpu(), m, atol=1e-9, rtol=2e-6)
        torch.testing.assert_close(opt.v[p].cpu(), v, atol=1e-12, rtol=2e-6)


def test_adamw_mixed_dtypes_one_launch(cuda_device):
    """float32 and bf16 tensors in the same table: each keeps its own dtype and arithmetic."""
    from triton_muon_adamw.adamw import TritonAdamW
    gen = torch.Generator().manual_seed(5)
    cpu = [torch.randn(5000, generator=gen) * 0.02, (torch.randn(777, generator=gen) * 0.02).to(torch.bfloat16)]
    params = [torch.nn.Parameter(t.clone().to(cuda_device)) for t in cpu]
    opt = TritonAdamW(params, lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1, eps=1e-8)
    ms = [torch.zeros(t.numel()) for t in cpu]
    vs = [torch.zeros(t.numel()) for t in cpu]
    for step in range(1, 3):
        grads = [(torch.randn(t.numel(), generator=gen) * 1e-2).to(t.dtype) for t in cpu]
        for p, g in zip(params, grads):
            p.grad = g.to(cuda_device)
        opt.step()
        b1, b2 = adamw_bias_corrections(0.9, 0.95, step)
        for t, g, m, v in zip(cpu, grads, ms, vs):
            adamw_update_(t, g, m, v, lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, bias1=b1,
                          bias2=b2)
    torch.testing.assert_close(params[0].detach().cpu(), cpu[0], atol=1e-7, rtol=2e-6)
    _within_one_ulp(params[1].detach(), cpu[1], "bf16 tensor")


# ----------------------------------------------------------------- Muon
SHAPES = [(64, 64), (200, 300), (300, 200), (5, 3), (256, 1000), (1000, 256), (96, 40)]


def test_muon_bf16_prep_matches_oracle(cuda_device):
    """bf16 momentum EMA + Nesterov glue and the bf16 X the Newton-Schulz GEMMs read."""
    from triton_muon_adamw import _lib as L
    from triton_muon_adamw.muon import TritonMuon
    lib = L.load()
    gen = torch.Generator().manual_seed(21)
    params = [torch.nn.Parameter((torch.randn(s, generator=gen) * 0.02).to(torch.bfloat16).to(cuda_device))
              for s in SHAPES]
    grads = [torch.randn(s, generator=gen).to(torch.bfloat16) for s in SHAPES]
    moms = [(torch.randn(s, generator=gen) * 0.1).to(torch.bfloat16) for s in SHAPES]
    opt = TritonMuon(params, lr=1e-3, weight_decay=0.1, coeffs=COEFFS, ns_steps=5)
    for p, g, mm in zip(params, grads, moms):
        p.grad = g.to(cuda_device)
        opt.momentum[p].copy_(mm)
    plan = opt._plan
    plan.ensure(opt._active(), opt.adjust_lr_fn, cuda_device)
    L.check(lib.mad_muon_prep(ctypes.byref(plan.info), plan.table.data_ptr(), 0.95, 1, 1e-7, L.stream_handle()))
    torch.cuda.synchronize()
    for i, (p, g, mm) in enumerate(zip(params, grads, moms)):
        mom = mm.clone()
        u = muon_momentum_(g, mom, 0.95, True)
        assert opt.momentum[p].dtype == torch.bfloat16
        _within_one_ulp(opt.momentum[p], mom, f"momentum {SHAPES[i]}")
        b = plan.buffers[i]
        off = b.x[0] - plan.work.data_ptr()
        x_gpu = plan.work[off:off + b.m * b.ld_x * 2].view(torch.bfloat16).view(b.m, b.ld_x)[:, :b.n]
        x, _ = to_wide_bf16(u.float())
        _within_one_ulp(x_gpu, x, f"X {SHAPES[i]}")


@pytest.mark.parametrize("nesterov", [True, False])
def test_muon_bf16_update_matches_oracle(cuda_device, nesterov):
    """Orthogonalised update with bf16 parameters (lr=1, wd=0, zero params) vs the oracle."""
    from triton_muon_adamw.muon import TritonMuon
    gen = torch.Generator().manual_seed(8)
    params = [torch.nn.Parameter(torch.zeros(s, device=cuda_device, dtype=torch.bfloat16)) for s in SHAPES]
    opt = TritonMuon(params, lr=1.0, weight_decay=0.0, coeffs=COEFFS, nesterov=nesterov, ns_steps=5)
    moms = [torch.zeros(s, dtype=torch.bfloat16) for s in SHAPES]
    for step in range(2):
        grads = [(torch.randn(s, generator=gen) * 1e-3).to(torch.bfloat16) for s in SHAPES]
        for p, g in zip(params, grads):
            p.data.zero_()
            p.grad = g.to(cuda_device)
        opt.step()
        for p, g, mom in zip(params, grads, moms):
            u = muon_momentum_(g, mom, 0.95, nesterov)
            # p = bf16(0 - bf16(slr * o)): -p / slr recovers o to bf16 resolution.
            o_gpu = -p.detach().float().cpu() / scaled_lr(1.0, p.shape, "original")
            tiny = min(p.shape) < 16
            o_fold = orthogonalize(u.float(), COEFFS, 5, 1e-7, normalize="fold")
            err = float((o_gpu - o_fold).norm() / o_fold.norm())
            assert err < (2e-2 if tiny else 1.5e-2), f"{tuple(p.shape)} step {step}: vs fold {err:.3e}"
        for p, mom in zip(params, moms):
            _within_one_ulp(opt.momentum[p], mom, f"momentum {tuple(p.shape)} step {step}")
    assert opt.device_status() == 0


# ----------------------------------------------------------------- end to end
def test_muonadamw_bf16_vs_reference_wrapper_golden(cuda_device):
    """Full MuonAdamW.step() on bf16 parameters vs PyTorchMuonAdamW outputs recorded from the reference.

    The wrapper keeps torch's AdamW moments in bf16 where the reference's
    Triton path (and this one) keeps float32, so the bar is bf16 resolution
    (1e-2), the tolerance the reference's own comparison script uses.  The
    AdamW parameters are also held to the Triton-path oracle at one bf16 ulp.
    """
    from triton_muon_adamw import AdamConfig, MuonAdamW, MuonConfig
    d = load_golden("wrapper_bf16.pt")
    na = len(d["adam_shapes"])
    params = [torch.nn.Parameter(t.clone().to(cuda_device)) for t in d["init"]]
    assert all(p.dtype == torch.bfloat16 for p in params)
    mc = dict(d["muon"])
    mc["coeffs"] = COEFFS
    opt = MuonAdamW({"adam": params[:na], "muon": params[na:]}, muon_config=MuonConfig(**mc),
                    adam_config=AdamConfig(**d["adam"]), parameter_split="explicit")
    o = OracleMuonAdamW([t.clone() for t in d["init"][:na]], [t.clone() for t in d["init"][na:]],
                        adam=d["adam"], muon=dict(d["muon"], coeffs=COEFFS, normalize="fold"))
    for gs, after in zip(d["grads"], d["after"]):
        for p, g in zip(params, gs):
            p.grad = g.to(cuda_device)
        opt.step()
        o.step(gs[:na], gs[na:])
        for p, a in zip(params, after):
            assert p.dtype == torch.bfloat16
            torch.testing.assert_close(p.detach().float().cpu(), a.float(), atol=1e-2, rtol=1e-2)
        for p, q in zip(params[:na], o.params_adam):
            _within_one_ulp(p.detach(), q, f"AdamW {tuple(p.shape)}")
    assert opt.device_status() == 0


# ----------------------------------------------------------------- float32 masters
def test_master_weights_match_float32_run_on_the_masters(cuda_device):
    """master_weights=True: bf16 parameters and gradients, float32 masters and Muon momentum.

    The masters must equal, bit for bit, a float32 MuonAdamW run whose
    parameters start as the masters and whose gradients are the bf16 ones
    widened; every bf16 parameter must be its master rounded to bf16.
    """
    from triton_muon_adamw import AdamConfig, MuonAdamW, MuonConfig
    gen = torch.Generator().manual_seed(17)
    adam_shapes = [(300,), (64, 8), (1000,)]
    muon_shapes = [(64, 96), (200, 72), (5, 3), (256, 256)]
    init = [(torch.randn(s, generator=gen) * 0.02).to(torch.bfloat16) for s in adam_shapes + muon_shapes]
    na = len(adam_shapes)
    mc, ac = MuonConfig(coeffs=COEFFS), AdamConfig(lr=3e-4, betas=(0.9, 0.95))
    bf = [torch.nn.Parameter(t.clone().to(cuda_device)) for t in init]
    f32 = [torch.nn.Parameter(t.float().to(cuda_device)) for t in init]
    opt = MuonAdamW({"adam": bf[:na], "muon": bf[na:]}, muon_config=mc, adam_config=ac, parameter_split="explicit",
                    master_weights=True)
    ref = MuonAdamW({"adam": f32[:na], "muon": f32[na:]}, muon_config=mc, adam_config=ac, parameter_split="explicit")
    for _ in range(3):
        grads = [(torch.randn(t.shape, generator=gen) * 1e-3).to(torch.bfloat16).to(cuda_device) for t in init]
        for p, q, g in zip(bf, f32, grads):
            p.grad, q.grad = g, g.float()
        opt.step()
        ref.step()
    masters = {**opt.adamw.masters, **opt.muon.masters}
    for p, q in zip(bf, f32):
        assert torch.equal(masters[p], q.detach()), f"master {tuple(p.shape)}"
        assert p.dtype == torch.bfloat16 and torch.equal(p.detach(), q.detach().to(torch.bfloat16)), tuple(p.shape)
    sd = opt.state_dict()
    assert torch.equal(sd["muon"]["state"][0]["master_param"], f32[na].detach())
    assert opt.device_status() == 0


def test_master_weights_need_bf16_parameters(cuda_device):
    from triton_muon_adamw import MuonAdamW
    p = torch.nn.Parameter(torch.zeros(8, 8, device=cuda_device))
    with pytest.raises(TypeError):
        MuonAdamW({"adam": [], "muon": [p]}, parameter_split="explicit", master_weights=True)
