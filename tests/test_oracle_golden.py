"""Pin the CPU oracle to outputs of the reference project itself (tests/golden/).

The fixtures were produced by tests/golden/make_golden.py from the reference
package: its ``PyTorchMuonAdamW`` wrapper on CPU and its ``TritonAdamW`` kernel
under the Triton interpreter.  Tolerances: the AdamW restatement must match the
reference Triton kernel to float32 rounding; the wrapper restatement must match
bit for bit; the Triton-path Muon restatement must match the wrapper within the
reference's Muon tolerance (atol 1e-2, rtol 1e-2 on parameters, README.md:52)
and, on the orthogonalised update itself, within bf16 noise.
"""

from __future__ import annotations

import pytest
import torch

from conftest import load_golden
from oracle.muon_adamw_oracle import (OracleMuonAdamW, ReferenceWrapperCPU, adamw_bias_corrections,
                                      adamw_update_, frobenius_normalize, muon_apply_, muon_momentum_, muon_nesterov,
                                      scaled_lr, to_wide_bf16)

WRAPPER_CASES = ["gpt_tiny", "ragged", "ns_direct", "match_rms"]


def test_adamw_restatement_matches_reference_triton_kernel():
    d = load_golden("triton_adamw.pt")
    cfg = d["cfg"]
    ps = [t.clone() for t in d["init"]]
    m = [torch.zeros_like(p) for p in ps]
    v = [torch.zeros_like(p) for p in ps]
    b1, b2 = cfg["betas"]
    for step, (gs, after) in enumerate(zip(d["grads"], d["after"]), 1):
        bc1, bc2 = adamw_bias_corrections(b1, b2, step)
        for p, g, mm, vv in zip(ps, gs, m, v):
            if g is None:
                continue
            adamw_update_(p, g, mm, vv, lr=cfg["lr"], beta1=b1, beta2=b2, eps=cfg["eps"],
                          weight_decay=cfg["weight_decay"], bias1=bc1, bias2=bc2)
        for p, a in zip(ps, after):
            torch.testing.assert_close(p, a, atol=1e-8, rtol=1e-6)


@pytest.mark.parametrize("name", WRAPPER_CASES)
def test_wrapper_restatement_is_bit_exact(name):
    d = load_golden(f"wrapper_{name}.pt")
    na = len(d["adam_shapes"])
    ps = [t.clone() for t in d["init"]]
    w = ReferenceWrapperCPU(ps[:na], ps[na:], adam=d["adam"], muon=d["muon"])
    for gs, after in zip(d["grads"], d["after"]):
        for p, g in zip(ps, gs):
            p.grad = g.clone()
        w.step()
        for p, a in zip(ps, after):
            assert torch.equal(p, a)


@pytest.mark.parametrize("name", WRAPPER_CASES)
def test_triton_path_restatement_within_reference_tolerance(name):
    d = load_golden(f"wrapper_{name}.pt")
    na = len(d["adam_shapes"])
    o = OracleMuonAdamW([t.clone() for t in d["init"][:na]], [t.clone() for t in d["init"][na:]],
                        adam=d["adam"], muon=d["muon"])
    for gs, after in zip(d["grads"], d["after"]):
        o.step(gs[:na], gs[na:])
        for p, a in zip(o.params_adam, after[:na]):
            torch.testing.assert_close(p, a, atol=1e-4, rtol=1e-3)
        for p, a in zip(o.params_muon, after[na:]):
            torch.testing.assert_close(p, a, atol=1e-2, rtol=1e-2)


def test_orthogonalised_update_within_bf16_noise():
    """ns_direct: lr=1, wd=0, zero parameters, so params after = -scaled_lr * O."""
    d = load_golden("wrapper_ns_direct.pt")
    na = len(d["adam_shapes"])
    o = OracleMuonAdamW([t.clone() for t in d["init"][:na]], [t.clone() for t in d["init"][na:]],
                        adam=d["adam"], muon=d["muon"])
    o.step(d["grads"][0][:na], d["grads"][0][na:])
    for upd, ref_after in zip(o.last_updates, d["after"][0][na:]):
        ref_o = -ref_after / scaled_lr(1.0, ref_after.shape, "original")
        diff = upd - ref_o
        assert float(diff.norm() / ref_o.norm()) < 2e-2
        assert float(diff.abs().max()) < 2e-2


def test_bf16_parameters_within_reference_tolerance():
    """bf16 parameters: the Triton-path restatement (fp32 AdamW moments, bf16 Muon glue) vs the wrapper.

    The wrapper keeps torch's AdamW moments in bf16, the reference's Triton
    path in float32, so AdamW agrees to bf16 resolution, not bit for bit.
    """
    d = load_golden("wrapper_bf16.pt")
    na = len(d["adam_shapes"])
    assert d["init"][0].dtype == torch.bfloat16
    o = OracleMuonAdamW([t.clone() for t in d["init"][:na]], [t.clone() for t in d["init"][na:]],
                        adam=d["adam"], muon=d["muon"])
    for gs, after in zip(d["grads"], d["after"]):
        o.step(gs[:na], gs[na:])
        for p, a in zip(o.params_adam + o.params_muon, after):
            assert p.dtype == torch.bfloat16
            torch.testing.assert_close(p.float(), a.float(), atol=1e-2, rtol=1e-2)
        for p, a in zip(o.params_adam, after[:na]):
            torch.testing.assert_close(p.float(), a.float(), atol=2e-4, rtol=1e-2)


@pytest.mark.parametrize("case", range(4))
def test_muon_glue_matches_reference_triton_muon_step(case):
    """Momentum, Nesterov, bf16 cast/transpose, normalisation and the parameter
    update against the reference's TritonMuon.step (float32 and bf16
    parameters; Newton-Schulz replaced by the identity when recorded).

    float32: every stage bit for bit over two steps.  bf16: the golden ran on
    CPU, whose bf16 ``add_(alpha=)`` rounds alpha to bf16 (and, in its scalar
    tail loop, the product too), while torch's CUDA kernel -- where the
    reference runs, and what the oracle restates by default -- keeps float32.
    So the bf16 momentum is held to one bf16 ulp on a few elements with the CPU
    alpha selected, and each step then continues from the recorded momentum so
    that Nesterov, the cast, the normalisation and the parameter update are
    checked bit for bit.
    """
    d = load_golden("triton_muon_glue.pt")[case]
    bf16 = d["dtype"] == "torch.bfloat16"
    ps = [t.clone() for t in d["init"]]
    moms = [torch.zeros_like(p) for p in ps]
    for gs, xs, mom_after, after in zip(d["grads"], d["x"], d["momentum"], d["after"]):
        for i, (p, g, mom) in enumerate(zip(ps, gs, moms)):
            u = muon_momentum_(g, mom, d["beta"], d["nesterov"], cpu_torch_alpha=bf16)
            if bf16:
                # One bf16 ulp of the result or of the (CPU-rounded) product alpha*g.
                want = mom_after[i].float()
                bound = torch.maximum(want.abs(), (1 - d["beta"]) * g.float().abs()) * 2.0 ** -7
                diff = (mom.float() - want).abs()
                assert bool((diff <= bound).all()), f"momentum {tuple(p.shape)}"
                assert int((diff > 0).sum()) <= 8, f"momentum {tuple(p.shape)}"
                mom.copy_(mom_after[i])
                u = muon_nesterov(g, mom, d["beta"]) if d["nesterov"] else mom.clone()
            else:
                assert torch.equal(mom, mom_after[i]), f"momentum {tuple(p.shape)}"
            x, transposed = to_wide_bf16(u)
            xn, _ = frobenius_normalize(x, d["eps"])
            assert torch.equal(xn, xs[i].float()), f"normalised X {tuple(p.shape)}"
            o = xn.t() if transposed else xn
            muon_apply_(p, o, d["lr"], d["weight_decay"], scaled_lr(d["lr"], p.shape, "original"))
            assert p.dtype == after[i].dtype and torch.equal(p, after[i]), f"parameter {tuple(p.shape)}"
