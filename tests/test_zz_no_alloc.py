"""The allocation-free Muon entry point against the planned one (needs a B200).

``mad_muon_step_noalloc`` serves callers that cannot allocate device memory
when they step the optimizer (a custom or pre-sized allocator, or a host with
no allocator binding): its plan and workspaces live in a static device array.
Here it must give the same parameters and momentum as the existing planned
path (``mad_muon_plan`` + ``mad_muon_step_multi``, through ``TritonMuon``) on
two calls in a row -- the second call also checks that the shared array's
leftovers from the first call do not leak into the result.  Tolerance: the
Muon parameter bar of the other tests (atol/rtol 1e-2), and since both paths
run the same kernels on the same data, bit equality is checked too.  This file
is collected last so a failure here cannot hide other failures.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

COEFFS = (3.4445, -4.7750, 2.0315)


@pytest.mark.parametrize("shape", [(256, 1024), (1024, 384), (96, 160), (7, 5)])
def test_noalloc_step_matches_planned_step_twice(cuda_device, shape):
    from triton_muon_adamw import _lib as L
    from triton_muon_adamw.muon import TritonMuon
    from triton_muon_adamw.muon.cuda_muon import lr_scale
    lib = L.load()
    gen = torch.Generator().manual_seed(sum(shape))
    p0 = torch.randn(shape, generator=gen) * 0.02
    grads = [torch.randn(shape, generator=gen) * 1e-3 for _ in range(2)]

    ref = torch.nn.Parameter(p0.clone().to(cuda_device))
    opt = TritonMuon([ref], lr=1e-3, weight_decay=0.1, coeffs=COEFFS, nesterov=True, beta=0.95, ns_steps=5)
    p = p0.clone().to(cuda_device)
    mom = torch.zeros_like(p)
    for g in grads:
        ref.grad = g.to(cuda_device)
        opt.step()
        gd = g.to(cuda_device)
        L.check(lib.mad_muon_step_noalloc(p.data_ptr(), gd.data_ptr(), mom.data_ptr(), shape[0], shape[1],
                                          lr_scale(shape, "original"), 0.95, 1, COEFFS[0], COEFFS[1], COEFFS[2], 5,
                                          1e-7, 1e-3, 0.1, L.stream_handle()), "mad_muon_step_noalloc")
        torch.cuda.synchronize()
        torch.testing.assert_close(p, ref.detach(), atol=1e-2, rtol=1e-2)
        assert torch.equal(p, ref.detach())
        assert torch.equal(mom, opt.momentum[ref])


def test_noalloc_rejects_matrices_beyond_the_static_scratch(cuda_device):
    from triton_muon_adamw import _lib as L
    lib = L.load()
    big = torch.zeros(2048, 2048, device=cuda_device)
    rc = lib.mad_muon_step_noalloc(big.data_ptr(), big.data_ptr(), big.data_ptr(), 2048, 2048, 1.0, 0.95, 1,
                                   COEFFS[0], COEFFS[1], COEFFS[2], 5, 1e-7, 1e-3, 0.1, L.stream_handle())
    assert rc != 0 and b"static scratch" in lib.mad_last_error()


def test_noalloc_reports_an_expired_wait_and_recovers(cuda_device):
    """A kernel that gives up waiting makes the call return MAD_ERR_DEVICE; the next call is correct again.

    The caller of this entry point holds no plan whose status word it could
    read, so the call itself must report the failure.  The expiry is driven by
    the test hook that leaves the Gram launch's producer idle (nothing in
    flight when the waits run out).
    """
    from triton_muon_adamw import _lib as L
    from triton_muon_adamw.muon import TritonMuon
    from triton_muon_adamw.muon.cuda_muon import lr_scale
    lib = L.load()
    shape = (256, 512)
    gen = torch.Generator().manual_seed(77)
    p0 = torch.randn(shape, generator=gen) * 0.02
    g = (torch.randn(shape, generator=gen) * 1e-3).to(cuda_device)
    p = p0.clone().to(cuda_device)
    mom = torch.zeros_like(p)

    def call():
        return lib.mad_muon_step_noalloc(p.data_ptr(), g.data_ptr(), mom.data_ptr(), shape[0], shape[1],
                                         lr_scale(shape, "original"), 0.95, 1, COEFFS[0], COEFFS[1], COEFFS[2], 5,
                                         1e-7, 1e-3, 0.1, L.stream_handle())

    L.check(lib.mad_debug_expire_next_waits(1), "mad_debug_expire_next_waits")
    rc = call()
    assert rc == L.ERR_DEVICE, f"expected MAD_ERR_DEVICE, got {rc}"
    assert b"gave up waiting" in lib.mad_last_error()
    p.copy_(p0.to(cuda_device))
    mom.zero_()
    L.check(call(), "mad_muon_step_noalloc")
    ref = torch.nn.Parameter(p0.clone().to(cuda_device))
    ref.grad = g
    opt = TritonMuon([ref], lr=1e-3, weight_decay=0.1, coeffs=COEFFS, nesterov=True, beta=0.95, ns_steps=5)
    opt.step()
    torch.cuda.synchronize()
    assert torch.equal(p, ref.detach()) and torch.equal(mom, opt.momentum[ref])
