"""Sharded MuonAdamW step across the ranks of one node (one process per GPU).

The reference is single-GPU; this module adds the partitioning a multi-GPU
optimizer step needs, with one real exchange step:

* **Muon, whole matrices.**  Every Muon matrix is updated by exactly one rank
  (its owner).  Matrices are split into ``n_buckets`` groups in parameter
  order, and within a bucket assigned to ranks longest-processing-time first
  by their Newton-Schulz cost (``3m²n + m³`` per iteration), each to the least
  loaded rank.  Only the owner keeps the momentum buffer.
* **AdamW, ZeRO-1.**  The AdamW parameters are laid end to end in one flat
  buffer (each tensor 64-element aligned) cut into ``world`` equal element
  ranges; rank r updates range r and holds exp_avg/exp_avg_sq for it only.
  A tensor may straddle two ranges; each rank updates its piece.
* **Exchange.**  Parameters are re-homed as views into flat buffers laid out
  so that every rank's updated elements form one contiguous segment at
  offset ``rank * segment``.  On GPUs the flats live in a peer arena (CUDA
  IPC) and each rank pushes its segment into every other rank's replica
  right after the AdamW launch and after each Muon bucket's launches, on a
  side stream, with a small broadcast kernel (``mad_peer_push``) whose CTAs
  fit beside the persistent Newton-Schulz GEMM's -- so the transfer runs
  during the GEMMs, where NCCL's kernels would wait for free SMs -- or with
  the copy engines (``CudaBackend(push="copy_engine")``).  Stream-ordered
  barriers (a one-element all-reduce) open and close a step, so no rank
  writes a replica its owner may still be reading.
  Without a peer arena (the CPU test backend) one in-place
  ``all_gather_into_tensor`` per buffer does the same.

Gradients are expected to be identical on every rank already (data-parallel
all-reduce upstream) -- unless ``reduce_grads`` is set: then each rank's
gradients are its own, un-reduced, and live in a gradient arena shared over
CUDA IPC (``peer.PeerArena``) laid out like the parameter flat buffers; the
AdamW and Muon-prep kernels read every rank's copy of the elements they own
over NVLink and use the mean (or sum).  That replaces the data-parallel
all-reduce (2x the gradient bytes per rank) by the reduce-scatter volume
(1x), fused into the optimizer's first kernels.  All ranks must call
``step()`` together.

The arithmetic is delegated to a backend: :class:`CudaBackend` (the CUDA
kernels) by default.  Tests of the partitioning logic on CPU ranks (gloo)
inject a CPU checker backend instead; the optimizer itself never selects one.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _lib
from .adamw.cuda_adam import AdamWTable
from .muon.cuda_muon import ADJUST_LR_FNS, MuonPlan, lr_scale, run_muon_plan

ALIGN = 64  # elements: 256-byte alignment of every tensor inside a flat buffer


def _round_up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


def ns_cost(shape) -> float:
    """Newton-Schulz flops of one iteration with symmetric products: 3m²n + m³."""
    m, n = min(shape[0], shape[1]), max(shape[0], shape[1])
    return 3.0 * m * m * n + float(m) ** 3


def lpt_assign(costs, n_ranks: int) -> list[int]:
    """Longest-processing-time-first owners: largest cost to the least-loaded rank (ties: lowest rank)."""
    load = [0.0] * n_ranks
    owner = [0] * len(costs)
    for i in sorted(range(len(costs)), key=lambda k: (-costs[k], k)):
        r = min(range(n_ranks), key=lambda q: (load[q], q))
        owner[i] = r
        load[r] += costs[i]
    return owner


def split_buckets(costs, n_buckets: int, increasing: bool = False) -> list[int]:
    """Contiguous groups in parameter order with decreasing total cost (weights n, n-1, ..., 1).

    Each bucket's all-gather overlaps the compute of the buckets after it; only
    the last one's is exposed, so the last bucket is made the smallest while
    every earlier gather still fits under the (larger) compute that follows it.
    ``increasing=True`` gives weights 1, 2, ..., n instead: for a pipeline whose
    first stage is a copy (gradients from the host), a small first bucket
    starts the compute early.
    """
    n_buckets = max(1, min(n_buckets, len(costs)))
    total = sum(costs) or 1.0
    weights = [k + 1 if increasing else n_buckets - k for k in range(n_buckets)]
    bounds, acc = [], 0.0
    for w in weights:
        acc += w
        bounds.append(total * acc / sum(weights))
    bucket, run, out = 0, 0.0, []
    for c in costs:
        if run >= bounds[bucket] and bucket < n_buckets - 1:
            bucket += 1
        out.append(bucket)
        run += c
    return out


@dataclass
class MuonSlot:
    index: int    # position in the Muon parameter list
    owner: int
    bucket: int
    offset: int   # element offset inside the bucket's flat buffer
    numel: int


def muon_layout(shapes, n_ranks: int, n_buckets: int):
    """Owner, bucket and flat-buffer offset of every Muon matrix, and each bucket's segment size."""
    costs = [ns_cost(s) for s in shapes]
    buckets = split_buckets(costs, n_buckets)
    nb = (max(buckets) + 1) if buckets else 0
    slots = [None] * len(shapes)
    seg_sizes = []
    for b in range(nb):
        idx = [i for i in range(len(shapes)) if buckets[i] == b]
        owners = lpt_assign([costs[i] for i in idx], n_ranks)
        fill = [0] * n_ranks
        per_rank = [[] for _ in range(n_ranks)]
        for i, r in zip(idx, owners):
            per_rank[r].append(i)
        for r in range(n_ranks):
            for i in per_rank[r]:
                numel = int(math.prod(shapes[i]))
                slots[i] = MuonSlot(i, r, b, fill[r], numel)
                fill[r] += _round_up(numel, ALIGN)
        seg = _round_up(max(fill) if fill else 0, ALIGN)
        seg_sizes.append(seg)
        for i in idx:
            slots[i].offset += slots[i].owner * seg
    return slots, seg_sizes


def zero1_layout(numels, n_ranks: int):
    """Offsets of the AdamW tensors in one flat buffer and the per-rank shard size."""
    offsets, off = [], 0
    for n in numels:
        offsets.append(off)
        off += _round_up(n, ALIGN)
    shard = _round_up(-(-off // n_ranks) if n_ranks else 0, ALIGN)
    return offsets, shard, shard * n_ranks


def shard_pieces(offsets, numels, lo: int, hi: int):
    """Pieces (tensor, start in tensor, length, start in shard) of tensors intersecting [lo, hi)."""
    out = []
    for i, (o, n) in enumerate(zip(offsets, numels)):
        a, b = max(o, lo), min(o + n, hi)
        if a < b:
            out.append((i, a - o, b - a, a - lo))
    return out


def _rehome(params, flat: torch.Tensor, offsets) -> None:
    """Move each parameter's storage into ``flat`` (values copied); the Parameter objects stay the same."""
    with torch.no_grad():
        for p, o in zip(params, offsets):
            view = flat[o:o + p.numel()].view_as(p)
            view.copy_(p.data)
            p.data = view


# --------------------------------------------------------------------------- backends
# NCCL communicators for the parameter exchange with a CTA cap, one per
# (default group, ranks, cap) in this process: every optimizer over the same
# ranks shares it instead of creating another communicator (and another set of
# NVLS buffers).
_EXCHANGE_GROUPS: dict = {}


def nccl_exchange_group(process_group, ctas: int):
    """A process group over ``process_group``'s ranks whose NCCL communicator uses at most
    ``ctas`` CTAs per collective (NCCL config ``maxCTAs`` and ``nvlsCTAs``).

    Created by every member (``use_local_synchronization``), the first time a
    given (ranks, cap) is asked for, so the ranks must ask in the same order --
    which constructing the optimizer collectively gives.
    """
    ranks = tuple(dist.get_process_group_ranks(process_group))
    key = (id(dist.distributed_c10d._get_default_group()), ranks, int(ctas))
    g = _EXCHANGE_GROUPS.get(key)
    if g is None:
        opts = dist.ProcessGroupNCCL.Options()
        opts.config.max_ctas = int(ctas)
        opts.config.nvls_ctas = int(ctas)
        g = dist.new_group(list(ranks), backend="nccl", pg_options=opts, use_local_synchronization=True)
        _EXCHANGE_GROUPS[key] = g
    return g


class CudaBackend:
    """The product's arithmetic: the CUDA AdamW and Muon kernels, and the peer transfers."""

    PUSH_MODES = ("auto", "nccl", "copy_engine", "kernel", "hybrid", "mixed")

    def __init__(self, push: str = "auto", ce_splits: int = 1, ce_fraction: float = 0.5, reserve_sms: int = 0,
                 ce_exchanges: int = 3):
        if push not in self.PUSH_MODES:
            raise ValueError(f"push must be one of {self.PUSH_MODES}, got {push!r}")
        if not 0 <= int(reserve_sms) <= 64:
            raise ValueError(f"reserve_sms must be in 0..64, got {reserve_sms!r}")
        if int(ce_exchanges) < 0:
            raise ValueError(f"ce_exchanges must be >= 0, got {ce_exchanges!r}")
        self.push = push
        # push="mixed": the first ce_exchanges exchanges issued in a step go by the
        # copy engines, the later ones by NCCL all-gathers (see exchange_kind).
        self.ce_exchanges = int(ce_exchanges)
        # SMs handed to the NCCL exchange: the GEMMs leave them free and the
        # exchange communicator is capped to as many CTAs.  0 (default): every
        # SM for the GEMMs, NCCL's own CTA count.  Measured on the 8B step at
        # 4 ranks, a cap of 8 CTAs kept the GEMMs at their single-rank rate
        # per clock but left the all-gather too slow to hide (197 ms/step
        # against 125 without a cap; 16: 136 ms).
        self.reserve_sms = int(reserve_sms)
        self.ce_splits = max(1, int(ce_splits))
        self.ce_fraction = float(ce_fraction)
        self.adam_table = AdamWTable()
        self.plans = {}

    def grad_arena(self, nbytes: int, device, process_group):
        """The gradient arena shared with the other ranks (CUDA IPC)."""
        from .peer import PeerArena  # noqa: PLC0415
        return PeerArena(nbytes, device, process_group)

    def param_arena(self, nbytes: int, device, process_group):
        """The parameter flats' arena: every rank writes its updated segments into the others' copies.

        None for ``push="nccl"`` (plain device memory, NCCL all-gathers).  ``"auto"``
        picks by group size, from 8B-step measurements: the copy engines up to
        4 ranks (they carry the (N-1)/N x parameter bytes each rank sends under
        the GEMMs, using no SM), NCCL beyond (its NVLS all-gather sends each
        segment once and the switch replicates it, where the copy engines'
        ~310 GB/s of peer writes no longer hide under the compute).
        """
        if self.push == "auto":
            self.push = "copy_engine" if dist.get_world_size(process_group) <= 4 else "nccl"
        if self.push == "nccl":
            return None
        from .peer import PeerArena  # noqa: PLC0415
        return PeerArena(nbytes, device, process_group)

    def exchange_kind(self, index: int) -> str:
        """How the ``index``-th exchange issued in a step moves: ``"push"`` (written into
        the peers' replicas, :meth:`push_segment`) or ``"nccl"`` (all-gather).

        ``push="mixed"`` splits a step's exchanges: the early ones -- issued
        while most of the step's compute is still ahead, and carrying most of
        the bytes (the AdamW flat and the largest Muon buckets) -- go by the
        copy engines, which use no SM; only the late ones go by NCCL, whose
        kernels take SMs from the Newton-Schulz GEMMs while they run.
        """
        if self.push == "nccl":
            return "nccl"
        if self.push == "mixed":
            return "push" if index < self.ce_exchanges else "nccl"
        return "push"

    def exchange_group(self, process_group):
        """The group the NCCL all-gathers of the exchange run on: with SMs
        reserved for it, a communicator capped to that many CTAs, so NCCL's
        kernels fit on the SMs the GEMMs leave free; else ``process_group``."""
        if self.push != "nccl" or not self.reserve_sms:
            return process_group
        return nccl_exchange_group(process_group, self.reserve_sms)

    def push_segment(self, arena, flat: torch.Tensor, seg: int, rank: int):
        """Write this rank's segment of ``flat`` into every other rank's replica, after the work queued so
        far on the current stream; returns a work whose ``wait()`` orders the current stream after it.

        ``push="kernel"``: one ``mad_peer_push`` launch on a side stream -- a
        small kernel whose CTAs fit beside the persistent GEMM's, reading each
        vector once and storing it to every peer over NVLink.
        ``push="copy_engine"``: ``cudaMemcpyAsync`` per peer, each peer's copy cut
        into ``ce_splits`` pieces on their own streams (no SM at all).
        ``push="hybrid"``: the first ``ce_fraction`` of the segment by the copy
        engines, the rest by the kernel, concurrently.
        """
        if self.push not in ("kernel", "copy_engine", "hybrid", "mixed"):
            raise ValueError(f"push mode {self.push!r} does not write into peer replicas")
        lib = _lib.load()
        cur = torch.cuda.current_stream()
        n_peers = arena.world - 1
        ce_streams = 0 if self.push == "kernel" else n_peers * self.ce_splits
        while len(getattr(self, "_push_streams", ())) < ce_streams + 1:
            self._push_streams = getattr(self, "_push_streams", []) + [torch.cuda.Stream(device=cur.device)]
        ready = torch.cuda.Event()
        ready.record(cur)
        src = flat[rank * seg:(rank + 1) * seg]
        off = src.data_ptr() - arena.ptr
        nbytes = src.numel() * src.element_size()
        peers = [(rank + k) % arena.world for k in range(1, arena.world)]
        ce_bytes = {"kernel": 0, "copy_engine": nbytes, "mixed": nbytes}.get(
            self.push, int(nbytes * self.ce_fraction) // 256 * 256)
        done = []

        def finish(st):
            e = torch.cuda.Event()
            e.record(st)
            done.append(e)

        if ce_bytes:
            piece = (-(-ce_bytes // self.ce_splits) + 255) // 256 * 256   # ceil(ce_bytes / splits), 256-aligned
            streams = iter(self._push_streams[1:])
            for q in peers:
                for a in range(0, ce_bytes, piece):
                    st = next(streams)
                    st.wait_event(ready)
                    _lib.check(lib.mad_copy_async(arena.peer_ptrs[q] + off + a, src.data_ptr() + a,
                                                  min(piece, ce_bytes - a), st.cuda_stream), "mad_copy_async")
                    finish(st)
        if ce_bytes < nbytes:
            st = self._push_streams[0]
            st.wait_event(ready)
            ps = _lib.PeerSet()
            ps.n_peers = len(peers)
            for j, q in enumerate(peers):
                ps.delta[j] = arena.peer_ptrs[q] - arena.ptr
            _lib.check(lib.mad_peer_push(src.data_ptr() + ce_bytes, nbytes - ce_bytes, ctypes.byref(ps),
                                         st.cuda_stream), "mad_peer_push")
            finish(st)
        return _StreamWork(done)

    def adamw(self, quads, *, lr, beta1, beta2, eps, weight_decay, bias1, bias2, timer=None, reduce=None):
        if not quads:
            return
        self.adam_table.ensure(quads, quads[0][0].device)
        if timer is not None:
            timer.mark("adamw")
        self.adam_table.launch(lr=lr, beta1=beta1, beta2=beta2, eps=eps, weight_decay=weight_decay, bias1=bias1,
                               bias2=bias2, reduce=reduce)

    def muon(self, bucket: int, triples, *, adjust_lr_fn, beta, nesterov, a, b, c, ns_steps, eps, lr,
             weight_decay, timer=None, reduce=None):
        if not triples:
            return
        plan = self.plans.setdefault(bucket, MuonPlan())
        plan.ensure(triples, adjust_lr_fn, triples[0][0].device)
        run_muon_plan(plan, beta=beta, nesterov=nesterov, a=a, b=b, c=c, ns_steps=ns_steps, eps=eps, lr=lr,
                      weight_decay=weight_decay, timer=timer, reduce=reduce, reserve_sms=self.reserve_sms)

    def status(self) -> int:
        st = 0
        for plan in self.plans.values():
            st |= plan.read_status()
        return st


class _StreamWork:
    """Completion of copies queued on side streams: ``wait()`` orders the current stream after them."""

    def __init__(self, events):
        self.events = events

    def wait(self):
        cur = torch.cuda.current_stream()
        for e in self.events:
            cur.wait_event(e)


class _Branch:
    """Hyperparameter holder exposing the attributes of the reference's branch optimizers."""

    def __init__(self, params):
        self.model_params = list(params)
        self._timer = None

    def zero_grad(self):
        for p in self.model_params:
            if p.grad is not None:
                p.grad.zero_()


class ShardedMuonAdamW:
    """The MuonAdamW step partitioned over a process group (see the module docstring)."""

    def __init__(self, adam_params, muon_params, muon_config, adam_config, process_group, *, n_buckets=5,
                 backend=None, reduce_grads=None, master_weights=False):
        if reduce_grads not in (None, "mean", "sum"):
            raise ValueError(f"reduce_grads must be None, 'mean' or 'sum', got {reduce_grads!r}")
        if muon_config.adjust_lr_fn not in ADJUST_LR_FNS:
            raise AssertionError(f"Invalid adjust_lr_fn: {muon_config.adjust_lr_fn}")
        for p in muon_params:
            if p.ndim != 2:
                raise AssertionError("Muon only supports 2D tensors")
        dtypes = {p.dtype for p in list(adam_params) + list(muon_params)}
        if len(dtypes) > 1 or not dtypes <= {torch.float32, torch.bfloat16}:
            raise TypeError(f"sharded parameters must all be float32 or all bfloat16, got {sorted(map(str, dtypes))}")
        # Parameters and Muon momentum live in flat buffers of the parameters' dtype;
        # the AdamW moments are float32.  With master_weights the parameters are bf16
        # and each rank keeps float32 masters (and float32 momentum) of what it owns.
        self.dtype = dtypes.pop() if dtypes else torch.float32
        self.master_weights = bool(master_weights)
        if self.master_weights and self.dtype != torch.bfloat16:
            raise TypeError("master_weights=True needs bfloat16 parameters")
        mom_dtype = torch.float32 if self.master_weights else self.dtype
        self.pg = process_group
        self.rank = dist.get_rank(process_group)
        self.world = dist.get_world_size(process_group)
        self.backend = backend if backend is not None else CudaBackend()
        params = list(adam_params) + list(muon_params)
        self.device = params[0].device if params else torch.device("cpu")

        ad = self.adamw = _Branch(adam_params)
        ad.lr, (ad.beta1, ad.beta2) = adam_config.lr, tuple(adam_config.betas)
        ad.eps, ad.weight_decay, ad.step_num = adam_config.eps, adam_config.weight_decay, 0
        mu = self.muon = _Branch(muon_params)
        mu.lr, mu.beta, mu.eps, mu.weight_decay = muon_config.lr, muon_config.beta, muon_config.eps, muon_config.weight_decay
        mu.a, mu.b, mu.c = muon_config.coeffs
        mu.is_nesterov, mu.steps, mu.adjust_lr_fn = muon_config.nesterov, muon_config.ns_steps, muon_config.adjust_lr_fn

        # AdamW: ZeRO-1 ranges over one flat buffer.  Muon: owner segments per bucket.
        self.adam_numels = [p.numel() for p in ad.model_params]
        self.adam_offsets, self.adam_shard, total = zero1_layout(self.adam_numels, self.world)
        lo = self.rank * self.adam_shard
        self.adam_pieces = shard_pieces(self.adam_offsets, self.adam_numels, lo, lo + self.adam_shard)
        self.exp_avg = torch.zeros(self.adam_shard, dtype=torch.float32, device=self.device)
        self.exp_avg_sq = torch.zeros(self.adam_shard, dtype=torch.float32, device=self.device)
        shapes = [tuple(p.shape) for p in mu.model_params]
        self.slots, self.seg_sizes = muon_layout(shapes, self.world, n_buckets)

        # The flat buffers, in a peer arena when the backend has one (the updated
        # segments are then pushed into the other ranks' replicas by the copy
        # engines), else ordinary device memory gathered with NCCL.
        self.param_arena = None
        nbytes, adam_bytes, bucket_base = self._flat_layout(total)
        if hasattr(self.backend, "param_arena"):
            self.param_arena = self.backend.param_arena(nbytes, self.device, self.pg)
        self.exchange_pg = self.pg
        self._exchanges_issued = 0
        if self.param_arena is None and hasattr(self.backend, "exchange_group"):
            self.exchange_pg = self.backend.exchange_group(self.pg)
        if self.param_arena is not None:
            raw = self.param_arena.tensor
            es = self._elem_size()
            self.adam_flat = raw[0:total * es].view(self.dtype)
            self.muon_flats = [raw[base:base + self.world * seg * es].view(self.dtype)
                               for base, seg in zip(bucket_base, self.seg_sizes)]
        else:
            self.adam_flat = torch.zeros(total, dtype=self.dtype, device=self.device)
            self.muon_flats = [torch.zeros(self.world * seg, dtype=self.dtype, device=self.device)
                               for seg in self.seg_sizes]
        _rehome(ad.model_params, self.adam_flat, self.adam_offsets)
        with torch.no_grad():
            for p, s in zip(mu.model_params, self.slots):
                view = self.muon_flats[s.bucket][s.offset:s.offset + s.numel].view_as(p)
                view.copy_(p.data)
                p.data = view
        # Momentum for owned matrices, laid out like the owner's parameter segment.
        self.mom_segs = [torch.zeros(seg, dtype=mom_dtype, device=self.device) for seg in self.seg_sizes]
        # float32 masters of what this rank owns: its AdamW range and its Muon segments.
        self.adam_master, self.master_segs = None, []
        if self.master_weights:
            self.adam_master = self.adam_flat[lo:lo + self.adam_shard].float()
            self.master_segs = [f[self.rank * seg:(self.rank + 1) * seg].float()
                                for f, seg in zip(self.muon_flats, self.seg_sizes)]
        mu.momentum = {}
        for p, s in zip(mu.model_params, self.slots):
            if s.owner == self.rank:
                o = s.offset - self.rank * self.seg_sizes[s.bucket]
                mu.momentum[p] = self.mom_segs[s.bucket][o:o + s.numel].view_as(p)

        self.reduce_grads = reduce_grads
        self.arena = None
        self._grad_views = []
        if reduce_grads is not None:
            self._make_grad_arena()

    # ------------------------------------------------------------------ arenas
    def _elem_size(self) -> int:
        return torch.empty((), dtype=self.dtype).element_size()

    def _flat_layout(self, adam_total: int):
        """Byte layout shared by the parameter and gradient arenas: the AdamW flat, then each bucket's flat."""
        es = self._elem_size()
        off = adam_bytes = _round_up(adam_total * es, 256)
        bucket_base = []
        for seg in self.seg_sizes:
            bucket_base.append(off)
            off += _round_up(self.world * seg * es, 256)
        return off, adam_bytes, bucket_base

    def _make_grad_arena(self):
        """Gradient views laid out like the parameter flats, in one arena every rank maps."""
        es = self._elem_size()
        ad, mu = self.adamw, self.muon
        nbytes, _, bucket_base = self._flat_layout(len(self.adam_flat))
        self.arena = self.backend.grad_arena(nbytes, self.device, self.pg)
        raw = self.arena.tensor

        def view(byte_off, p):
            return raw[byte_off:byte_off + p.numel() * es].view(self.dtype).view(p.shape)

        self._grad_views = [(p, view(o * es, p)) for p, o in zip(ad.model_params, self.adam_offsets)]
        self._grad_views += [(p, view(bucket_base[s.bucket] + s.offset * es, p))
                             for p, s in zip(mu.model_params, self.slots)]
        for p, v in self._grad_views:
            if p.grad is not None:
                v.copy_(p.grad)
            p.grad = v

    def _bind_grads(self):
        """Gradients produced outside the arena (e.g. after ``zero_grad(set_to_none=True)``) are copied in."""
        with torch.no_grad():
            for p, v in self._grad_views:
                g = p.grad
                if g is not None and g.data_ptr() != v.data_ptr():
                    v.copy_(g)
                    p.grad = v

    def _rank_sync(self):
        """Stream-ordered barrier: work after it starts once every rank's stream has reached it."""
        if not hasattr(self, "_sync_flag"):
            self._sync_flag = torch.zeros(1, device=self.device)
        dist.all_reduce(self._sync_flag, group=self.pg)

    def close(self):
        """Release the memory shared with the other ranks (collective).  The parameters move to private
        copies; gradients in the shared gradient buffer are dropped (set to None).  No step afterwards."""
        if self.arena is not None:
            for p, _ in self._grad_views:
                p.grad = None
            self._grad_views = []
            self.arena.close()
            self.arena = None
        if self.param_arena is not None:
            with torch.no_grad():
                for p in list(self.adamw.model_params) + list(self.muon.model_params):
                    p.data = p.data.clone()
            self.adam_flat, self.muon_flats = None, []
            self.param_arena.close()
            self.param_arena = None
            self.closed = True

    # ------------------------------------------------------------------ step
    def _adam_quads(self):
        quads = []
        ad = self.adamw
        for i, start, length, sh in self.adam_pieces:
            p = ad.model_params[i]
            if p.grad is None:
                continue
            o = self.adam_offsets[i] + start
            piece = self.adam_flat[o:o + length]
            g, m, v = p.grad.reshape(-1)[start:start + length], self.exp_avg[sh:sh + length], self.exp_avg_sq[sh:sh + length]
            if self.master_weights:
                quads.append((self.adam_master[sh:sh + length], g, m, v, piece))
            else:
                quads.append((piece, g, m, v))
        return quads

    def _bucket_triples(self, b):
        mu = self.muon
        out = []
        for p, s in zip(mu.model_params, self.slots):
            if s.bucket == b and s.owner == self.rank and p.grad is not None and p.numel() > 0:
                if self.master_weights:
                    o = s.offset - self.rank * self.seg_sizes[b]
                    master = self.master_segs[b][o:o + s.numel].view_as(p)
                    out.append((master, p.grad, mu.momentum[p], p.data))
                else:
                    out.append((p.data, p.grad, mu.momentum[p]))
        return out

    def _gather(self, flat: torch.Tensor, seg: int):
        """Refresh every replica of ``flat`` with this rank's segment (returns a work with ``wait()``)."""
        index = self._exchanges_issued
        self._exchanges_issued += 1
        kind = self.backend.exchange_kind(index) if hasattr(self.backend, "exchange_kind") else "push"
        if self.param_arena is not None and kind == "push":
            return self.backend.push_segment(self.param_arena, flat, seg, self.rank)
        mine = flat[self.rank * seg:(self.rank + 1) * seg]
        return dist.all_gather_into_tensor(flat, mine, group=self.exchange_pg, async_op=True)

    @torch.no_grad()
    def step(self, wait_for=None, adam_last=False):
        """One sharded step.  ``wait_for`` (internal): callables run before the
        AdamW launch (index 0) and before each Muon bucket (index 1 + bucket).
        ``adam_last``: the AdamW shard after the Muon buckets instead of before
        (the branches update disjoint parameters; results are the same)."""
        ad, mu = self.adamw, self.muon
        ad.step_num += 1
        works = []
        self._exchanges_issued = 0
        bias1, bias2 = 1 - ad.beta1 ** ad.step_num, 1 - ad.beta2 ** ad.step_num
        red = None
        if getattr(self, "closed", False):
            raise RuntimeError("this optimizer was closed (close()); it cannot step")
        if self.reduce_grads is not None:
            if self.arena is None:
                raise RuntimeError("the gradient arena was released (close()); this optimizer cannot step")
            self._bind_grads()
            red = self.arena.spec(1.0 / self.world if self.reduce_grads == "mean" else 1.0)
        if red is not None or self.param_arena is not None:
            # Every rank's gradients are complete before any rank reads them, and no rank writes
            # into another's parameter replica while that rank's forward/backward may still read it.
            self._rank_sync()

        def adamw():
            if wait_for:
                wait_for[0]()
            if self.adam_shard:
                self.backend.adamw(self._adam_quads(), lr=ad.lr, beta1=ad.beta1, beta2=ad.beta2, eps=ad.eps,
                                   weight_decay=ad.weight_decay, bias1=bias1, bias2=bias2, timer=ad._timer,
                                   reduce=red)
                works.append(self._gather(self.adam_flat, self.adam_shard))

        if not adam_last:
            adamw()
        for b, seg in enumerate(self.seg_sizes):
            if wait_for:
                wait_for[1 + b]()
            self.backend.muon(b, self._bucket_triples(b), adjust_lr_fn=mu.adjust_lr_fn, beta=mu.beta,
                              nesterov=mu.is_nesterov, a=mu.a, b=mu.b, c=mu.c, ns_steps=mu.steps, eps=mu.eps,
                              lr=mu.lr, weight_decay=mu.weight_decay, timer=mu._timer, reduce=red)
            if seg:
                works.append(self._gather(self.muon_flats[b], seg))
        if adam_last:
            adamw()
        for w in works:
            w.wait()
        if red is not None or self.param_arena is not None:
            # No rank overwrites its gradients while another may still read them, and every
            # rank's pushes into this rank's replicas have landed before step() returns.
            self._rank_sync()

    @torch.no_grad()
    def step_from_host(self, host_grads):
        """:meth:`step` with gradients in host memory: each rank copies only the
        gradient pieces it reads, on a side stream, in the order the work
        consumes them.  Per rank every piece takes longer to copy than to
        update, so by Johnson's rule the Muon buckets go first, largest first,
        and the AdamW shard (the least compute per byte) last."""
        if self.reduce_grads is not None:
            raise NotImplementedError("step_from_host takes reduced gradients; it does not combine with reduce_grads")
        main = torch.cuda.current_stream()
        if not hasattr(self, "_copy_stream"):
            self._copy_stream = torch.cuda.Stream(device=main.device)
        copy = self._copy_stream
        copy.wait_stream(main)
        ad, mu = self.adamw, self.muon
        for p in list(ad.model_params) + list(mu.model_params):
            if p.grad is None and host_grads.get(p) is not None:
                p.grad = torch.empty_like(p)
        events = [None] * (1 + len(self.seg_sizes))

        def mark(k):
            events[k] = torch.cuda.Event()
            events[k].record(copy)

        with torch.cuda.stream(copy):
            for b in range(len(self.seg_sizes)):
                for p, s in zip(mu.model_params, self.slots):
                    h = host_grads.get(p)
                    if s.bucket == b and s.owner == self.rank and h is not None:
                        p.grad.copy_(h, non_blocking=True)
                mark(1 + b)
            for i, start, length, _ in self.adam_pieces:
                p = ad.model_params[i]
                h = host_grads.get(p)
                if h is not None:
                    p.grad.reshape(-1)[start:start + length].copy_(h.reshape(-1)[start:start + length],
                                                                   non_blocking=True)
            mark(0)
        self.step(wait_for=[lambda k=k: main.wait_event(events[k]) for k in range(len(events))], adam_last=True)
        for p in list(ad.model_params) + list(mu.model_params):
            if p.grad is not None:
                p.grad.record_stream(copy)

    # ------------------------------------------------------------------ introspection
    def owned_muon_shapes(self):
        return [tuple(p.shape) for p, s in zip(self.muon.model_params, self.slots)
                if s.owner == self.rank and p.grad is not None]

    def adam_shard_numel(self):
        return sum(length for _, _, length, _ in self.adam_pieces)

    def local_grad_tensors(self):
        """Gradient pieces this rank reads in a step (what a host-resident pipeline must copy in)."""
        out = [p.grad.reshape(-1)[start:start + length]
               for i, start, length, _ in self.adam_pieces
               for p in [self.adamw.model_params[i]] if p.grad is not None]
        out += [g for _, g, _ in (t for b in range(len(self.seg_sizes)) for t in self._bucket_triples(b))]
        return out

    def status(self) -> int:
        return self.backend.status() if hasattr(self.backend, "status") else 0

    # ------------------------------------------------------------------ checkpoint
    def _global(self, group_rank: int) -> int:
        return dist.get_global_rank(self.pg, group_rank) if self.pg is not None else group_rank

    def _gather_flat(self, shard: torch.Tensor, to_rank, cpu: bool):
        """Every rank's ``shard`` end to end in rank order: on every rank (``to_rank`` None) or on
        ``to_rank`` alone (None elsewhere); in host memory when ``cpu``.  One such flat at a time is
        ever held in device memory."""
        full = None
        if to_rank is None:
            full = torch.empty(shard.numel() * self.world, dtype=shard.dtype, device=shard.device)
            dist.all_gather_into_tensor(full, shard, group=self.pg)
        elif self.rank == to_rank:
            full = torch.empty(shard.numel() * self.world, dtype=shard.dtype, device=shard.device)
            dist.gather(shard, gather_list=list(full.chunk(self.world)), dst=self._global(to_rank), group=self.pg)
        else:
            dist.gather(shard, gather_list=None, dst=self._global(to_rank), group=self.pg)
        if full is not None and cpu:
            full = full.cpu()
        return full

    def _scatter_flat(self, full, shard: torch.Tensor, from_rank: int) -> None:
        """``full`` (on ``from_rank``: every rank's shard end to end) cut into the ranks' shards."""
        src = self._global(from_rank)
        if self.rank == from_rank:
            full = full.to(device=shard.device, dtype=shard.dtype)
            dist.scatter(shard, scatter_list=list(full.chunk(self.world)), src=src, group=self.pg)
        else:
            dist.scatter(shard, scatter_list=None, src=src, group=self.pg)

    @torch.no_grad()
    def state_dict(self, to_rank=None, cpu: bool = False):
        """Full state in the layout of ``PyTorchMuonAdamW.state_dict()``; collective.

        The shards are gathered one flat buffer at a time (the AdamW moments, then each bucket's Muon
        momentum and masters).  ``to_rank``: only that rank receives the dict (the others get ``{}``),
        by NCCL gathers rather than all-gathers.  ``cpu``: every gathered flat goes to host memory
        before the next one is gathered, so device memory holds one flat at most -- for large models
        (the 8B set's state is ~36 GB) use ``state_dict(to_rank=0, cpu=True)``.  The per-parameter
        tensors are views into those flats.
        """
        from .checkpoint import _adam_group, _muon_group  # noqa: PLC0415
        ad, mu = self.adamw, self.muon
        mine = to_rank is None or self.rank == to_rank
        full_m = self._gather_flat(self.exp_avg, to_rank, cpu)
        full_v = self._gather_flat(self.exp_avg_sq, to_rank, cpu)
        full_master = self._gather_flat(self.adam_master, to_rank, cpu) if self.master_weights else None
        adam_state = {}
        if mine and ad.step_num > 0:
            for i, p in enumerate(ad.model_params):
                o, n = self.adam_offsets[i], self.adam_numels[i]
                adam_state[i] = {"step": torch.tensor(float(ad.step_num), dtype=torch.float32,
                                                      device="cpu" if cpu else p.device),
                                 "exp_avg": full_m[o:o + n].view(p.shape),
                                 "exp_avg_sq": full_v[o:o + n].view(p.shape)}
                if full_master is not None:
                    adam_state[i]["master_param"] = full_master[o:o + n].view(p.shape)
        del full_m, full_v, full_master
        muon_state = {}
        for b, seg in enumerate(self.seg_sizes):
            mom = self._gather_flat(self.mom_segs[b], to_rank, cpu)
            master = self._gather_flat(self.master_segs[b], to_rank, cpu) if self.master_weights else None
            if not mine:
                continue
            for i, (p, s) in enumerate(zip(mu.model_params, self.slots)):
                if s.bucket != b:
                    continue
                muon_state[i] = {"momentum_buffer": mom[s.offset:s.offset + s.numel].view(p.shape)}
                if master is not None:
                    muon_state[i]["master_param"] = master[s.offset:s.offset + s.numel].view(p.shape)
        if not mine:
            return {}
        return {"adam": {"state": adam_state, "param_groups": [_adam_group(ad, len(ad.model_params))]},
                "muon": {"state": dict(sorted(muon_state.items())),
                         "param_groups": [_muon_group(mu, len(mu.model_params))]}}

    @torch.no_grad()
    def load_state_dict(self, sd, from_rank=None):
        """Load a full state dict; each rank keeps its shard.

        ``from_rank`` None: every rank passes the same dict.  ``from_rank=k``: only rank k holds it (the
        others pass anything, e.g. None); the hyperparameters are broadcast and every flat is assembled on
        rank k and scattered, one at a time.  In that form a parameter missing from the dict starts from
        zero state (as ``torch.optim`` does), and a missing ``master_param`` from the current parameter.
        """
        if from_rank is not None:
            self._load_scattered(sd, from_rank)
            return
        ad, mu = self.adamw, self.muon
        if "adam" in sd:
            a = sd["adam"]
            g = a["param_groups"][0]
            ad.lr, (ad.beta1, ad.beta2), ad.eps, ad.weight_decay = g["lr"], tuple(g["betas"]), g["eps"], g["weight_decay"]
            steps = []
            for i, start, length, sh in self.adam_pieces:
                st = a["state"].get(i)
                if st is None:
                    continue
                self.exp_avg[sh:sh + length].copy_(st["exp_avg"].reshape(-1)[start:start + length])
                self.exp_avg_sq[sh:sh + length].copy_(st["exp_avg_sq"].reshape(-1)[start:start + length])
                if self.master_weights:
                    # A dict without masters (PyTorchMuonAdamW's, or a checkpoint saved without them): the
                    # masters restart from the current bf16 parameters, as the single-GPU path does.
                    src = st["master_param"] if "master_param" in st else ad.model_params[i].detach()
                    self.adam_master[sh:sh + length].copy_(src.reshape(-1)[start:start + length])
            for st in a["state"].values():
                steps.append(int(float(st["step"])))
            ad.step_num = max(steps) if steps else 0
        if "muon" in sd:
            m = sd["muon"]
            self._muon_hyper(m["param_groups"][0])
            for i, (p, s) in enumerate(zip(mu.model_params, self.slots)):
                if p not in mu.momentum:        # owned by another rank
                    continue
                st = m["state"].get(i)
                if st is not None and "momentum_buffer" in st:
                    mu.momentum[p].copy_(st["momentum_buffer"])
                if self.master_weights:
                    src = st["master_param"] if st is not None and "master_param" in st else p.detach()
                    o = s.offset - self.rank * self.seg_sizes[s.bucket]
                    self.master_segs[s.bucket][o:o + s.numel].copy_(src.reshape(-1))

    def _muon_hyper(self, g):
        mu = self.muon
        mu.lr, mu.weight_decay, mu.beta, mu.is_nesterov = g["lr"], g["weight_decay"], g["momentum"], g["nesterov"]
        if "ns_coefficients" in g:
            mu.a, mu.b, mu.c = g["ns_coefficients"]
        mu.eps, mu.steps = g.get("eps", mu.eps), g.get("ns_steps", mu.steps)
        mu.adjust_lr_fn = g.get("adjust_lr_fn") or "original"

    def _load_scattered(self, sd, from_rank: int) -> None:
        ad, mu = self.adamw, self.muon
        root = self.rank == from_rank
        head = [None]
        if root:
            a, m = sd.get("adam"), sd.get("muon")
            steps = [int(float(st["step"])) for st in a["state"].values()] if a else []
            head = [{"adam_group": a["param_groups"][0] if a else None,
                     "muon_group": m["param_groups"][0] if m else None,
                     "step": max(steps) if steps else 0}]
        dist.broadcast_object_list(head, src=self._global(from_rank), group=self.pg)
        head = head[0]
        if head["adam_group"] is not None:
            g = head["adam_group"]
            ad.lr, (ad.beta1, ad.beta2), ad.eps, ad.weight_decay = g["lr"], tuple(g["betas"]), g["eps"], g["weight_decay"]
            ad.step_num = head["step"]

            def adam_flat(key, fallback_param=False):
                if not root:
                    return None
                full = torch.zeros(self.adam_shard * self.world, dtype=torch.float32, device=self.device)
                for i, p in enumerate(ad.model_params):
                    st = sd["adam"]["state"].get(i)
                    o, n = self.adam_offsets[i], self.adam_numels[i]
                    if st is not None and key in st:
                        full[o:o + n].copy_(st[key].reshape(-1))
                    elif fallback_param:
                        full[o:o + n].copy_(p.detach().reshape(-1))
                return full

            self._scatter_flat(adam_flat("exp_avg"), self.exp_avg, from_rank)
            self._scatter_flat(adam_flat("exp_avg_sq"), self.exp_avg_sq, from_rank)
            if self.master_weights:
                self._scatter_flat(adam_flat("master_param", True), self.adam_master, from_rank)
        if head["muon_group"] is not None:
            self._muon_hyper(head["muon_group"])
            for b, seg in enumerate(self.seg_sizes):
                def muon_flat(key, dtype, fallback_param=False):
                    if not root:
                        return None
                    full = torch.zeros(seg * self.world, dtype=dtype, device=self.device)
                    for i, (p, s) in enumerate(zip(mu.model_params, self.slots)):
                        if s.bucket != b:
                            continue
                        st = sd["muon"]["state"].get(i)
                        if st is not None and key in st:
                            full[s.offset:s.offset + s.numel].copy_(st[key].reshape(-1))
                        elif fallback_param:
                            full[s.offset:s.offset + s.numel].copy_(p.detach().reshape(-1))
                    return full

                self._scatter_flat(muon_flat("momentum_buffer", self.mom_segs[b].dtype), self.mom_segs[b], from_rank)
                if self.master_weights:
                    self._scatter_flat(muon_flat("master_param", torch.float32, True), self.master_segs[b], from_rank)


__all__ = ["ShardedMuonAdamW", "CudaBackend", "lpt_assign", "split_buckets", "muon_layout", "zero1_layout",
           "shard_pieces", "ns_cost", "lr_scale"]
