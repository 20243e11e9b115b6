"""Checkpoint layout of MuonAdamW: the two ``torch.optim`` state dicts of PyTorchMuonAdamW.

``{"adam": AdamW state dict, "muon": Muon state dict}`` with per-parameter
entries indexed by position in each branch's parameter list:

* AdamW: ``{"step": float32 tensor, "exp_avg": ..., "exp_avg_sq": ...}``
* Muon:  ``{"momentum_buffer": ...}``

plus one ``param_groups`` entry per branch carrying the hyperparameters under
torch's names.  With ``master_weights=True`` each entry also holds the float32
master of its (bf16) parameter under ``"master_param"``.  A dict saved by ``PyTorchMuonAdamW`` loads here and vice
versa.  For compatibility with the reference's ``load_state_dict``
(optimizer.py:170-175), a branch given as a plain parameter list replaces that
branch's parameter list (new parameters get zero state).

In sharded (multi-GPU) mode the state lives in per-rank shards; saving
gathers them one flat buffer at a time (to every rank, or to one rank and
optionally into host memory) and loading cuts them back into shards (from a
dict every rank holds, or scattered from one rank).
"""

from __future__ import annotations

import torch


def _adam_group(ad, n):
    return {"lr": ad.lr, "betas": (ad.beta1, ad.beta2), "eps": ad.eps, "weight_decay": ad.weight_decay,
            "amsgrad": False, "maximize": False, "foreach": None, "capturable": False, "differentiable": False,
            "fused": True, "decoupled_weight_decay": True, "params": list(range(n))}


def _muon_group(mu, n):
    return {"lr": mu.lr, "weight_decay": mu.weight_decay, "momentum": mu.beta, "nesterov": mu.is_nesterov,
            "ns_coefficients": (mu.a, mu.b, mu.c), "eps": mu.eps, "ns_steps": mu.steps,
            "adjust_lr_fn": mu.adjust_lr_fn, "params": list(range(n))}


def branch_state_dicts(opt) -> dict:
    ad, mu = opt.adamw, opt.muon
    adam_state = {}
    if ad.step_num > 0:
        for i, p in enumerate(ad.model_params):
            adam_state[i] = {"step": torch.tensor(float(ad.step_num), dtype=torch.float32, device=p.device),
                             "exp_avg": ad.m[p], "exp_avg_sq": ad.v[p]}
            if ad.masters is not None:
                adam_state[i]["master_param"] = ad.masters[p]
    muon_state = {i: {"momentum_buffer": mu.momentum[p]} for i, p in enumerate(mu.model_params)}
    if mu.masters is not None:
        for i, p in enumerate(mu.model_params):
            muon_state[i]["master_param"] = mu.masters[p]
    return {"adam": {"state": adam_state, "param_groups": [_adam_group(ad, len(ad.model_params))]},
            "muon": {"state": muon_state, "param_groups": [_muon_group(mu, len(mu.model_params))]}}


def _replace_params(branch, params, states):
    branch.model_params = list(params)
    masters = getattr(branch, "masters", None)
    for name in states:
        store = getattr(branch, name)
        for p in branch.model_params:
            if p not in store:
                fp32 = name in ("m", "v") or masters is not None   # master mode: float32 momentum
                store[p] = torch.zeros_like(p, dtype=torch.float32 if fp32 else p.dtype)
    if masters is not None:
        for p in branch.model_params:
            if p not in masters:
                masters[p] = p.detach().float()


@torch.no_grad()
def load_branch_state_dicts(opt, sd: dict) -> None:
    ad, mu = opt.adamw, opt.muon
    if "adam" in sd:
        a = sd["adam"]
        if isinstance(a, (list, tuple)):
            _replace_params(ad, a, ("m", "v"))
        else:
            g = a["param_groups"][0]
            ad.lr, (ad.beta1, ad.beta2), ad.eps, ad.weight_decay = g["lr"], tuple(g["betas"]), g["eps"], g["weight_decay"]
            steps = []
            for i, p in enumerate(ad.model_params):
                st = a["state"].get(i)
                if st is None:
                    continue
                ad.m[p].copy_(st["exp_avg"])
                ad.v[p].copy_(st["exp_avg_sq"])
                if ad.masters is not None:
                    ad.masters[p].copy_(st["master_param"] if "master_param" in st else p.detach().float())
                steps.append(int(float(st["step"])))
            ad.step_num = max(steps) if steps else 0
    if "muon" in sd:
        m = sd["muon"]
        if isinstance(m, (list, tuple)):
            _replace_params(mu, m, ("momentum",))
        else:
            g = m["param_groups"][0]
            mu.lr, mu.weight_decay, mu.beta, mu.is_nesterov = g["lr"], g["weight_decay"], g["momentum"], g["nesterov"]
            if "ns_coefficients" in g:
                mu.a, mu.b, mu.c = g["ns_coefficients"]
            mu.eps, mu.steps = g.get("eps", mu.eps), g.get("ns_steps", mu.steps)
            mu.adjust_lr_fn = g.get("adjust_lr_fn") or "original"
            for i, p in enumerate(mu.model_params):
                st = m["state"].get(i)
                if st is not None and "momentum_buffer" in st:
                    mu.momentum[p].copy_(st["momentum_buffer"])
                if mu.masters is not None:
                    mu.masters[p].copy_(st["master_param"] if st is not None and "master_param" in st
                                        else p.detach().float())
    opt.param_group = {"adam": ad.model_params, "muon": mu.model_params}
