"""The Newton-Schulz kernels' error path: barrier waits that expire (needs a B200).

``mad_debug_expire_next_waits(n)`` arms the next n Gram launches: their TMA
producer issues no load and their barrier waits give up after ~10 ms.  The
Gram epilogue reads no input, so when the waits expire no copy and no MMA is
in flight -- the kernel records its status bits, releases its tensor memory
and returns, and the context stays usable.  Nothing here faults or hangs the
GPU: the wait that runs out is one nothing was ever going to satisfy.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

COEFFS = (3.4445, -4.7750, 2.0315)
SHAPES = [(256, 512), (768, 256), (300, 300)]


def _opt(params):
    from triton_muon_adamw.muon import TritonMuon
    return TritonMuon(params, lr=1e-2, weight_decay=0.1, coeffs=COEFFS, nesterov=True, ns_steps=5)


def test_expired_wait_is_reported_and_the_next_step_is_correct(cuda_device):
    from triton_muon_adamw import _lib as L
    lib = L.load()
    gen = torch.Generator().manual_seed(31)
    init = [torch.randn(s, generator=gen) * 0.02 for s in SHAPES]
    grads = [[torch.randn(s, generator=gen) * 1e-3 for s in SHAPES] for _ in range(2)]
    armed = [torch.nn.Parameter(t.clone().to(cuda_device)) for t in init]
    clean = [torch.nn.Parameter(t.clone().to(cuda_device)) for t in init]
    oa, ob = _opt(armed), _opt(clean)

    for p, g in zip(armed, grads[0]):
        p.grad = g.to(cuda_device)
    L.check(lib.mad_debug_expire_next_waits(1), "mad_debug_expire_next_waits")
    oa.step()
    st = oa.device_status(clear=True)
    assert st & L.DEV_ERR_TIMEOUT_MMA, f"status {st:#x}: the MMA issuer's wait did not report"
    assert st & L.DEV_ERR_TIMEOUT_EPILOGUE, f"status {st:#x}: the epilogue's wait did not report"
    assert oa.device_status() == 0, "status must be clear after a clearing read"

    # The aborted step left its matrices invalid; restore the state and step both optimizers normally.
    with torch.no_grad():
        for p, t in zip(armed, init):
            p.copy_(t.to(cuda_device))
        for p in armed:
            oa.momentum[p].zero_()
    for step in range(2):
        for ps in (armed, clean):
            for p, g in zip(ps, grads[step]):
                p.grad = g.to(cuda_device)
        oa.step()
        ob.step()
        torch.cuda.synchronize()
        for p, q in zip(armed, clean):
            assert torch.equal(p.detach(), q.detach()), f"{tuple(p.shape)} step {step} after the expired launch"
    assert oa.device_status() == 0 and ob.device_status() == 0


def test_disarmed_hook_changes_nothing(cuda_device):
    from triton_muon_adamw import _lib as L
    lib = L.load()
    L.check(lib.mad_debug_expire_next_waits(1), "mad_debug_expire_next_waits")
    L.check(lib.mad_debug_expire_next_waits(0), "mad_debug_expire_next_waits")
    p = torch.nn.Parameter(torch.randn(256, 256, device=cuda_device) * 0.02)
    p.grad = torch.randn(256, 256, device=cuda_device) * 1e-3
    o = _opt([p])
    o.step()
    assert o.device_status() == 0
    assert lib.mad_debug_expire_next_waits(-1) == 1
