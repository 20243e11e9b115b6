"""Checkpoint layout (triton_muon_adamw/checkpoint.py) on CPU, with stand-in branch objects.

The branches of MuonAdamW need CUDA tensors, but the state-dict code only
reads and writes their attributes, so plain objects carrying the same
attributes exercise it here: the torch.optim layout, the float32 masters of
mixed precision, and the reference's list form of load_state_dict
(optimizer.py:170-175).
"""

from __future__ import annotations

from types import SimpleNamespace

import torch

from triton_muon_adamw.checkpoint import branch_state_dicts, load_branch_state_dicts


def _opt(seed: int, masters: bool):
    gen = torch.Generator().manual_seed(seed)
    dt = torch.bfloat16 if masters else torch.float32
    ap = [torch.nn.Parameter((torch.randn(s, generator=gen) * 0.02).to(dt)) for s in [(7,), (3, 5)]]
    mp = [torch.nn.Parameter((torch.randn(s, generator=gen) * 0.02).to(dt)) for s in [(4, 6), (6, 4)]]
    ad = SimpleNamespace(model_params=ap, lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.01, step_num=3,
                         m={p: torch.randn(p.shape, generator=gen) for p in ap},
                         v={p: torch.rand(p.shape, generator=gen) for p in ap},
                         masters={p: torch.randn(p.shape, generator=gen) for p in ap} if masters else None)
    mu = SimpleNamespace(model_params=mp, lr=1e-3, weight_decay=0.1, beta=0.95, is_nesterov=True, a=3.4445,
                         b=-4.775, c=2.0315, eps=1e-7, steps=5, adjust_lr_fn="original",
                         momentum={p: torch.randn(p.shape, generator=gen) for p in mp},
                         masters={p: torch.randn(p.shape, generator=gen) for p in mp} if masters else None)
    return SimpleNamespace(distributed=None, adamw=ad, muon=mu, param_group={})


def test_state_dict_round_trip_with_masters():
    src, dst = _opt(0, masters=True), _opt(1, masters=True)
    sd = branch_state_dicts(src)
    assert set(sd) == {"adam", "muon"}
    assert sd["adam"]["param_groups"][0]["betas"] == (0.9, 0.95) and sd["muon"]["param_groups"][0]["nesterov"]
    load_branch_state_dicts(dst, sd)
    assert dst.adamw.step_num == 3
    for a, b in ((src.adamw, dst.adamw), (src.muon, dst.muon)):
        for p, q in zip(a.model_params, b.model_params):
            assert torch.equal(a.masters[p], b.masters[q])
    for p, q in zip(src.adamw.model_params, dst.adamw.model_params):
        assert torch.equal(src.adamw.m[p], dst.adamw.m[q]) and torch.equal(src.adamw.v[p], dst.adamw.v[q])
    for p, q in zip(src.muon.model_params, dst.muon.model_params):
        assert torch.equal(src.muon.momentum[p], dst.muon.momentum[q])


def test_state_dict_without_masters_has_the_torch_layout():
    sd = branch_state_dicts(_opt(2, masters=False))
    assert all("master_param" not in st for st in sd["adam"]["state"].values())
    assert all(set(st) == {"momentum_buffer"} for st in sd["muon"]["state"].values())
    assert all(set(st) == {"step", "exp_avg", "exp_avg_sq"} for st in sd["adam"]["state"].values())


def test_loading_a_dict_without_masters_takes_them_from_the_parameters():
    src, dst = _opt(3, masters=False), _opt(4, masters=True)
    load_branch_state_dicts(dst, branch_state_dicts(src))
    for p in dst.adamw.model_params + dst.muon.model_params:
        br = dst.adamw if p in dst.adamw.masters else dst.muon
        assert torch.equal(br.masters[p], p.detach().float())


def test_list_form_gives_new_parameters_zero_state_and_float32_masters():
    """The reference's load_state_dict form: a branch given as a parameter list replaces that list."""
    opt = _opt(5, masters=True)
    extra = torch.nn.Parameter(torch.randn(2, 3).to(torch.bfloat16))
    load_branch_state_dicts(opt, {"muon": opt.muon.model_params + [extra]})
    assert opt.muon.model_params[-1] is extra
    assert opt.muon.momentum[extra].dtype == torch.float32 and not opt.muon.momentum[extra].any()
    assert torch.equal(opt.muon.masters[extra], extra.detach().float())
    assert opt.param_group["muon"][-1] is extra
