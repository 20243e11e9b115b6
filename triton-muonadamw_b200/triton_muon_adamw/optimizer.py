"""Hybrid MuonAdamW optimizer: drop-in replacement of the reference's API.

Same public surface as the reference's ``triton_muon_adamw/optimizer.py``:
``AdamConfig`` and ``MuonConfig`` (field names, types and defaults,
optimizer.py:14-67), ``MuonAdamW`` (constructor, auto/explicit parameter
routing, ``step``/``zero_grad``/``state_dict``/``load_state_dict``,
attributes ``adamw``/``muon``/``param_group``; optimizer.py:70-175) and
``PyTorchMuonAdamW``, the ``torch.optim`` comparison wrapper
(optimizer.py:178-260).

``MuonAdamW.step()`` runs the AdamW branch (one CUDA launch) and then the
Muon branch (2 + 3*ns_steps CUDA launches) on the current CUDA stream.  Given
a ``torch.distributed`` process group of size > 1 it shards the work: whole
Muon matrices per rank (size-balanced) and ZeRO-1 AdamW element ranges,
followed by an NCCL all-gather of the updated parameters.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal, TypeAlias

import torch
import torch.nn as nn

from .adamw.cuda_adam import TritonAdamW
from .muon.cuda_muon import TritonMuon

ParameterGroups: TypeAlias = dict[str, list[nn.Parameter]]


@dataclass
class AdamConfig:
    """Hyperparameters for the AdamW branch of :class:`MuonAdamW`.

    Parameters
    ----------
    lr:
        Learning rate used by AdamW.
    betas:
        Coefficients of the first- and second-moment running averages.
    eps:
        Term added to the denominator for numerical stability.
    weight_decay:
        Decoupled AdamW weight decay coefficient.
    """

    lr: float = 1e-3
    betas: tuple[float, float] = (0.9, 0.999)
    eps: float = 1e-7
    weight_decay: float = 0.01


@dataclass
class MuonConfig:
    """Hyperparameters for the Muon branch of :class:`MuonAdamW`.

    Parameters
    ----------
    lr:
        Learning rate used by Muon.
    beta:
        Momentum coefficient.
    eps:
        Lower bound of the Frobenius norm used to normalise the update.
    weight_decay:
        Decoupled weight decay coefficient.
    coeffs:
        Coefficients (a, b, c) of the Newton-Schulz polynomial.
    nesterov:
        Whether to use Nesterov momentum.
    ns_steps:
        Number of Newton-Schulz iterations.
    adjust_lr_fn:
        Shape-dependent learning-rate adjustment of the Muon update.
    """

    lr: float = 1e-3
    beta: float = 0.95
    eps: float = 1e-7
    weight_decay: float = 0.1
    coeffs: tuple[float, float, float] = (3.445, -4.775, 2.0315)
    nesterov: bool = True
    ns_steps: int = 5
    adjust_lr_fn: Literal["original", "match_rms_adamw", "spectral_unclamped"] = "original"


def split_parameters(model_params, parameter_split):
    """Route parameters to AdamW or Muon exactly as the reference does (optimizer.py:107-130).

    ``explicit``: the ``"adam"``/``"muon"`` lists of a dict.  ``auto``: every
    trainable 2-D parameter except the input embedding and the output head
    goes to Muon, everything else to AdamW; parameters sharing storage (a
    tied head) are taken once.
    """
    adam_params, muon_params = [], []
    if parameter_split == "explicit" and not isinstance(model_params, dict):
        raise ValueError("When parameter_split is 'explicit', params must be a dictionary with keys 'adam' and "
                         "'muon' and their corresponding parameters.")
    if parameter_split == "auto" and isinstance(model_params, dict):
        raise ValueError("When parameter_split is 'auto', params must be an nn.Module (ie the model itself), not a "
                         "dictionary.")
    if parameter_split == "explicit":
        adam_params = list(model_params.get("adam", []))
        muon_params = list(model_params.get("muon", []))
    elif parameter_split == "auto":
        embed = model_params.get_input_embeddings().weight
        out = model_params.get_output_embeddings()
        head = out.weight if out is not None else None
        seen_ptrs = set()
        for p in model_params.parameters():
            if not p.requires_grad or p.data_ptr() in seen_ptrs:
                continue
            seen_ptrs.add(p.data_ptr())
            if p.ndim == 2 and p is not embed and p is not head:
                muon_params.append(p)
            else:
                adam_params.append(p)
    return adam_params, muon_params


class MuonAdamW(TritonMuon, TritonAdamW):
    """Optimizer that routes parameters to Muon or AdamW and updates them on the GPU.

    Two-dimensional parameters are updated with Muon, except the input
    embedding and the output head; all other trainable parameters (biases,
    norms, embeddings, heads) use AdamW.  Parameters must be float32 or
    bfloat16, contiguous CUDA tensors (gradients and Muon momentum in the
    parameter's dtype, AdamW moments float32); there is no CPU implementation.

    Parameters
    ----------
    model_params:
        The model (``parameter_split="auto"``) or a dict with ``"adam"`` and
        ``"muon"`` parameter lists (``"explicit"``).  In auto mode the model
        must provide ``get_input_embeddings()`` and ``get_output_embeddings()``.
    muon_config, adam_config:
        Hyperparameters of the two branches.
    parameter_split:
        ``"auto"`` or ``"explicit"``.
    process_group:
        Optional ``torch.distributed`` process group (NCCL).  With more than
        one rank, Muon matrices are owned whole by one rank each, AdamW state
        is sharded ZeRO-1 style, and the updated parameters are all-gathered.
        Gradients are expected to be identical on every rank already, unless
        ``reduce_grads`` is given.
    reduce_grads:
        ``None`` (default), ``"mean"`` or ``"sum"``: with a process group of
        more than one rank, each rank's gradients are its own (data-parallel,
        not yet reduced).  ``param.grad`` tensors are re-homed into a buffer
        the other ranks map over CUDA IPC, and the step's first kernels read
        every rank's copy of the elements they update over NVLink and use the
        mean (or sum) -- the gradient reduce-scatter fused into the step, in
        place of a data-parallel all-reduce.  Zero gradients in place
        (:meth:`zero_grad`) to keep them in that buffer; gradients found
        elsewhere at ``step()`` are copied in.  Call :meth:`close` on every
        rank before the process group is destroyed.
    peer_push:
        With more than one rank, how each rank's updated parameters reach the
        others: ``"auto"`` (default; the copy engines up to 4 ranks, NCCL
        above), ``"nccl"`` (all-gather), ``"copy_engine"`` (each rank writes its
        segment into the others' replicas with ``cudaMemcpyAsync``, no SM),
        ``"kernel"`` (a small broadcast kernel beside the GEMMs),
        ``"hybrid"`` (copy engines and kernel, half each) or ``"mixed"`` (the
        step's first three exchanges by the copy engines, the later ones by
        NCCL).
    master_weights:
        Mixed precision: the parameters (and their gradients) are bfloat16 and
        the optimizer keeps a float32 master copy of each, with float32 Muon
        momentum.  Every update runs on the master in float32, as for float32
        parameters, and writes the bf16 parameter with the same store; the
        master and the update are what a float32 run on the masters with the
        bf16 gradients would give, bit for bit.  Sharded, each rank keeps the
        masters of what it owns and the all-gather moves bf16 (half the bytes).
        Checkpoints carry the masters (``"master_param"`` per parameter).
    reserve_sms:
        With more than one rank and the NCCL exchange, SMs handed to it
        (0..64): the Newton-Schulz GEMMs leave that many SMs free (rounded up
        to CTA pairs) and the all-gathers run on a communicator capped to as
        many CTAs, so NCCL's kernels run beside the GEMMs instead of taking
        SMs from them.  0 (default): every SM for the GEMMs and NCCL's own CTA
        count -- the faster choice measured (the GEMMs hand out tiles
        dynamically, so a pair whose SMs NCCL holds for a while takes fewer
        tiles, while a capped all-gather falls behind the compute).
    """

    def __init__(
        self,
        model_params: nn.Module | ParameterGroups,
        muon_config: MuonConfig = MuonConfig(),  # noqa: B008
        adam_config: AdamConfig = AdamConfig(),  # noqa: B008
        parameter_split: Literal["auto", "explicit"] = "auto",
        process_group=None,
        reduce_grads: Literal["mean", "sum"] | None = None,
        peer_push: Literal["auto", "nccl", "copy_engine", "kernel", "hybrid", "mixed"] = "auto",
        master_weights: bool = False,
        reserve_sms: int = 0,
    ) -> None:
        if reduce_grads not in (None, "mean", "sum"):
            raise ValueError(f"reduce_grads must be None, 'mean' or 'sum', got {reduce_grads!r}")
        from .distributed import CudaBackend  # noqa: PLC0415
        if peer_push not in CudaBackend.PUSH_MODES:
            raise ValueError(f"peer_push must be one of {CudaBackend.PUSH_MODES}, got {peer_push!r}")
        adam_params, muon_params = split_parameters(model_params, parameter_split)
        self.master_weights = bool(master_weights)
        if self.master_weights and any(p.dtype != torch.bfloat16 for p in adam_params + muon_params):
            raise TypeError("master_weights=True needs bfloat16 parameters (the masters are float32)")
        self.process_group = process_group
        self.distributed = None
        if process_group is not None and torch.distributed.get_world_size(process_group) > 1:
            from .distributed import ShardedMuonAdamW  # noqa: PLC0415
            self.distributed = ShardedMuonAdamW(adam_params, muon_params, muon_config, adam_config, process_group,
                                                reduce_grads=reduce_grads,
                                                backend=CudaBackend(push=peer_push, reserve_sms=reserve_sms),
                                                master_weights=self.master_weights)
            self.adamw = self.distributed.adamw
            self.muon = self.distributed.muon
        else:
            self.adamw = TritonAdamW(params=adam_params, lr=adam_config.lr, betas=adam_config.betas,
                                     weight_decay=adam_config.weight_decay, eps=adam_config.eps)
            self.muon = TritonMuon(params=muon_params, lr=muon_config.lr, beta=muon_config.beta,
                                   eps=muon_config.eps, weight_decay=muon_config.weight_decay,
                                   coeffs=muon_config.coeffs, nesterov=muon_config.nesterov,
                                   ns_steps=muon_config.ns_steps, adjust_lr_fn=muon_config.adjust_lr_fn)
            if self.master_weights:
                with torch.no_grad():
                    self.adamw.masters = {p: p.detach().float() for p in self.adamw.model_params}
                    self.muon.masters = {p: p.detach().float() for p in self.muon.model_params}
                    self.muon.momentum = {p: torch.zeros_like(p, dtype=torch.float32) for p in self.muon.model_params}
        self.param_group = {
            "adam": self.adamw.model_params,
            "muon": self.muon.model_params,
        }

    def close(self) -> None:
        """Release the resources shared with other ranks (collective with ``reduce_grads``; else a no-op)."""
        if self.distributed is not None:
            self.distributed.close()

    def step(self) -> None:
        """Apply one update with both branches: AdamW, then Muon (optimizer.py:156-159)."""
        if self.distributed is not None:
            self.distributed.step()
            return
        self.adamw.step()
        self.muon.step()

    @torch.no_grad()
    def step_from_host(self, host_grads, n_buckets: int = 8) -> None:
        """One step whose gradients live in (pinned) host memory.

        ``host_grads`` maps each parameter to its host gradient (a dict keyed by
        Parameter, or a sequence in the order ``param_group["adam"] +
        param_group["muon"]``).  The result equals copying every gradient into
        ``param.grad`` and calling :meth:`step`, but the host-to-device copies
        run on a side stream while the GPU computes: a two-stage pipeline
        (copy, then compute) ordered by Johnson's rule -- the Muon matrices,
        whose compute outweighs their copy, first, in buckets of increasing
        size so the compute starts after a short copy; the AdamW tensors,
        whose copy outweighs their compute, last, their copy hidden under the
        Muon work.  The two branches update disjoint parameters, so the order
        does not change any result.
        """
        params = list(self.param_group["adam"]) + list(self.param_group["muon"])
        if not isinstance(host_grads, dict):
            host_grads = dict(zip(params, host_grads))
        if self.distributed is not None:
            self.distributed.step_from_host(host_grads)
            return
        from .distributed import ns_cost, split_buckets  # noqa: PLC0415
        from .muon.cuda_muon import MuonPlan, run_muon_plan  # noqa: PLC0415
        main = torch.cuda.current_stream()
        if not hasattr(self, "_copy_stream"):
            self._copy_stream = torch.cuda.Stream(device=main.device)
            self._bucket_plans = {}
        copy = self._copy_stream
        copy.wait_stream(main)  # the previous step may still read the gradient buffers

        for p in params:  # allocated on the main stream, which owns them afterwards
            if p.grad is None and host_grads.get(p) is not None:
                p.grad = torch.empty_like(p)

        def upload(ps):
            with torch.cuda.stream(copy):
                for p in ps:
                    h = host_grads.get(p)
                    if h is not None:
                        p.grad.copy_(h, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(copy)
            return ev

        mu = self.muon
        mats = [p for p in mu.model_params if p in host_grads or p.grad is not None]
        buckets = split_buckets([ns_cost(p.shape) for p in mats], n_buckets, increasing=True) if mats else []
        groups = [[p for p, b in zip(mats, buckets) if b == k] for k in range(max(buckets) + 1 if buckets else 0)]
        events = [upload(g) for g in groups]
        adam_ready = upload(self.adamw.model_params)
        for k, (g, ev) in enumerate(zip(groups, events)):
            main.wait_event(ev)
            triples = mu._active(only=g)
            if not triples:
                continue
            plan = self._bucket_plans.setdefault(k, MuonPlan())
            plan.ensure(triples, mu.adjust_lr_fn, triples[0][0].device)
            run_muon_plan(plan, beta=mu.beta, nesterov=mu.is_nesterov, a=mu.a, b=mu.b, c=mu.c, ns_steps=mu.steps,
                          eps=mu.eps, lr=mu.lr, weight_decay=mu.weight_decay)
        main.wait_event(adam_ready)
        self.adamw.step()
        for p in params:
            if p.grad is not None:
                p.grad.record_stream(copy)

    def zero_grad(self) -> None:
        """Reset the gradients of both branches to zero in place."""
        self.adamw.zero_grad()
        self.muon.zero_grad()

    def device_status(self, clear: bool = True) -> int:
        """Error bits recorded by the Muon kernels since the last read (0 = healthy)."""
        if self.distributed is not None:
            return self.distributed.status()
        st = self.muon.device_status(clear)
        for plan in getattr(self, "_bucket_plans", {}).values():
            st |= plan.read_status(clear)
        return st

    # -- checkpointing -----------------------------------------------------
    def state_dict(self, to_rank: int | None = None, cpu: bool = False) -> dict[str, object]:
        """Optimizer state in the layout of ``PyTorchMuonAdamW.state_dict()``.

        ``{"adam": <torch.optim.AdamW state dict>, "muon": <torch.optim.Muon
        state dict>}``: per-parameter ``step``/``exp_avg``/``exp_avg_sq`` and
        ``momentum_buffer``, indexed by position in each branch's parameter
        list, so checkpoints move between the two classes.  (The reference's
        own ``state_dict`` returns only the parameter lists, optimizer.py:166-168.)

        Sharded (collective): the shards are gathered one flat buffer at a
        time; ``to_rank=k`` delivers the dict to rank k only (``{}``
        elsewhere) and ``cpu=True`` moves each gathered buffer to host memory
        before the next, so device memory never holds more than one.  On one
        GPU ``cpu=True`` returns host copies and ``to_rank`` has no effect.
        """
        from .checkpoint import branch_state_dicts  # noqa: PLC0415
        if self.distributed is not None:
            return self.distributed.state_dict(to_rank=to_rank, cpu=cpu)
        sd = branch_state_dicts(self)
        if cpu:
            sd = {k: {"state": {i: {n: t.detach().cpu() for n, t in st.items()} for i, st in br["state"].items()},
                      "param_groups": br["param_groups"]} for k, br in sd.items()}
        return sd

    def load_state_dict(self, state_dict: dict[str, object], from_rank: int | None = None) -> None:
        """Load a dict produced by :meth:`state_dict` or by ``PyTorchMuonAdamW.state_dict()``.

        Sharded (collective): with ``from_rank=k`` only rank k needs the dict
        (the others may pass ``None``); it is scattered one buffer at a time.
        """
        from .checkpoint import load_branch_state_dicts  # noqa: PLC0415
        if self.distributed is not None:
            self.distributed.load_state_dict(state_dict, from_rank=from_rank)
            return
        load_branch_state_dicts(self, state_dict)


class PyTorchMuonAdamW:
    """``torch.optim`` comparison optimizer with the same routing and configs.

    Delegates to ``torch.optim.AdamW(fused=True)`` and ``torch.optim.Muon``
    exactly as the reference's wrapper does (optimizer.py:178-260), including
    passing neither ``coeffs`` nor ``eps`` to ``torch.optim.Muon`` (which then
    uses its own defaults).  It is for comparisons; :class:`MuonAdamW` never
    uses it.
    """

    def __init__(
        self,
        model_params: nn.Module | ParameterGroups,
        muon_config: MuonConfig = MuonConfig(),  # noqa: B008
        adam_config: AdamConfig = AdamConfig(),  # noqa: B008
        parameter_split: Literal["auto", "explicit"] = "auto",
    ) -> None:
        adam_params, muon_params = split_parameters(model_params, parameter_split)
        self.adamw = torch.optim.AdamW(params=adam_params, lr=adam_config.lr, betas=adam_config.betas,
                                       weight_decay=adam_config.weight_decay, eps=adam_config.eps, fused=True)
        self.muon = torch.optim.Muon(params=muon_params, lr=muon_config.lr, momentum=muon_config.beta,
                                     weight_decay=muon_config.weight_decay, nesterov=muon_config.nesterov,
                                     ns_steps=muon_config.ns_steps, adjust_lr_fn=muon_config.adjust_lr_fn)

    def step(self) -> None:
        """One ``torch.optim`` AdamW update, then one Muon update."""
        self.adamw.step()
        self.muon.step()

    def zero_grad(self) -> None:
        self.adamw.zero_grad()
        self.muon.zero_grad()

    def state_dict(self) -> dict[str, object]:
        return {"adam": self.adamw.state_dict(), "muon": self.muon.state_dict()}

    def load_state_dict(self, state_dict: dict[str, object]) -> None:
        if "adam" in state_dict:
            self.adamw.load_state_dict(state_dict["adam"])
        if "muon" in state_dict:
            self.muon.load_state_dict(state_dict["muon"])
