"""Checkpoints on the GPU: save, load, keep stepping (needs a B200).

The reference's own ``MuonAdamW.state_dict`` returns only the parameter lists
(``triton_muon_adamw/optimizer.py:166-168``), so its training state cannot be
resumed.  Ours returns the state in ``PyTorchMuonAdamW``'s layout
(``optimizer.py:248-260``: the ``torch.optim`` AdamW and Muon state dicts):

* save after k steps, load into a fresh optimizer over the saved parameters,
  continue: bit-identical to never stopping;
* the same dict loads into the reference's ``PyTorchMuonAdamW`` (imported
  unmodified from ``baseline/_ref``), and the wrapper's own dict loads into
  ours; both continue within the reference's tolerances (AdamW atol 1e-4 /
  rtol 1e-3, Muon atol/rtol 1e-2) of the optimizer that saved it.
"""

from __future__ import annotations

import copy
import io

import pytest
import torch

from reference_pkg import load_reference

pytestmark = pytest.mark.gpu

COEFFS = (3.4445, -4.7750, 2.0315)
ADAM_SHAPES = [(512, 64), (64,), (64,), (300,)]
MUON_SHAPES = [(64, 64), (256, 64), (64, 256), (96, 160), (384, 128)]
MUON = dict(lr=1e-3, beta=0.95, eps=1e-7, weight_decay=0.1, coeffs=COEFFS, nesterov=True, ns_steps=5)
ADAM = dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01)
NA = len(ADAM_SHAPES)


def _init():
    gen = torch.Generator().manual_seed(3)
    return [torch.randn(s, generator=gen) * 0.02 for s in ADAM_SHAPES + MUON_SHAPES]


def _grads(step):
    gen = torch.Generator().manual_seed(100 + step)
    return [torch.randn(s, generator=gen) * 1e-3 for s in ADAM_SHAPES + MUON_SHAPES]


def _params(tensors, dev):
    return [torch.nn.Parameter(t.detach().clone().to(dev)) for t in tensors]


def _ours(params):
    from triton_muon_adamw import AdamConfig, MuonAdamW, MuonConfig
    return MuonAdamW({"adam": params[:NA], "muon": params[NA:]}, muon_config=MuonConfig(**MUON),
                     adam_config=AdamConfig(**ADAM), parameter_split="explicit")


def _wrapper(params):
    R = load_reference()
    return R.PyTorchMuonAdamW({"adam": params[:NA], "muon": params[NA:]}, muon_config=R.MuonConfig(**MUON),
                              adam_config=R.AdamConfig(**ADAM), parameter_split="explicit")


def _step(opt, params, step, dev):
    for p, g in zip(params, _grads(step)):
        p.grad = g.to(dev)
    opt.step()


def _saved(sd):
    """The dict as a checkpoint file would give it back (torch.save / torch.load round trip)."""
    buf = io.BytesIO()
    torch.save(sd, buf)
    buf.seek(0)
    return torch.load(buf, weights_only=False)


def _close(got, want):
    for i, (p, q) in enumerate(zip(got, want)):
        tol = dict(atol=1e-4, rtol=1e-3) if i < NA else dict(atol=1e-2, rtol=1e-2)
        torch.testing.assert_close(p.detach(), q.detach(), **tol)


def test_save_load_continue_is_bit_identical_to_never_stopping(cuda_device):
    straight = _params(_init(), cuda_device)
    o = _ours(straight)
    for step in range(5):
        _step(o, straight, step, cuda_device)

    first = _params(_init(), cuda_device)
    a = _ours(first)
    for step in range(3):
        _step(a, first, step, cuda_device)
    sd = _saved(a.state_dict())
    resumed = _params(first, cuda_device)           # the model checkpoint: parameters at step 3
    b = _ours(resumed)
    b.load_state_dict(sd)
    assert b.adamw.step_num == 3
    for step in range(3, 5):
        _step(b, resumed, step, cuda_device)
    torch.cuda.synchronize()
    for p, q in zip(resumed, straight):
        assert torch.equal(p.detach(), q.detach()), tuple(p.shape)
    assert b.device_status() == 0


def test_our_checkpoint_resumes_in_the_reference_wrapper(cuda_device):
    mine = _params(_init(), cuda_device)
    o = _ours(mine)
    for step in range(3):
        _step(o, mine, step, cuda_device)
    sd = _saved(o.state_dict())
    theirs = _params(mine, cuda_device)
    w = _wrapper(theirs)
    w.load_state_dict(sd)
    for step in range(3, 5):
        _step(o, mine, step, cuda_device)
        _step(w, theirs, step, cuda_device)
    torch.cuda.synchronize()
    _close(mine, theirs)


def test_reference_wrapper_checkpoint_resumes_in_ours(cuda_device):
    theirs = _params(_init(), cuda_device)
    w = _wrapper(theirs)
    for step in range(3):
        _step(w, theirs, step, cuda_device)
    sd = _saved(copy.deepcopy(w.state_dict()))
    mine = _params(theirs, cuda_device)
    o = _ours(mine)
    o.load_state_dict(sd)
    assert o.adamw.step_num == 3
    for step in range(3, 5):
        _step(w, theirs, step, cuda_device)
        _step(o, mine, step, cuda_device)
    torch.cuda.synchronize()
    _close(mine, theirs)
    assert o.device_status() == 0
