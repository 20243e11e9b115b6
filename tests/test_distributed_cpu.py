"""Multi-rank logic of the sharded MuonAdamW step, on CPU ranks (gloo).

The partitioning (LPT owners, buckets, ZeRO-1 pieces, flat re-homing) and the
exchange (in-place all_gather_into_tensor per flat buffer) run exactly as on
GPUs; only the arithmetic backend is the CPU oracle, injected here.  With the
same arithmetic, every rank must end with parameters bit-identical to a
single-process oracle run.
"""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.muon_adamw_oracle import OracleMuonAdamW, adamw_update_, muon_matrix_step_

ADAM_SHAPES = [(100,), (37,), (64, 3), (5,), (129,)]
MUON_SHAPES = [(16, 24), (24, 16), (8, 8), (32, 16), (5, 7), (40, 8), (12, 12)]
MUON = dict(lr=1e-2, beta=0.95, eps=1e-7, weight_decay=0.1, coeffs=(3.4445, -4.775, 2.0315), nesterov=True,
            ns_steps=5, adjust_lr_fn="original")
ADAM = dict(lr=3e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01)


class CpuArena:
    """The gradient arena of CPU ranks: a plain tensor; a reduction all-gathers every rank's arena."""

    def __init__(self, nbytes, device, process_group):
        self.tensor = torch.zeros(nbytes, dtype=torch.uint8)
        self.pg = process_group

    def spec(self, scale):
        return (self, scale)

    def close(self):
        pass


def reduced(g, copies, arena, scale):
    """Every rank's copy of ``g`` (same arena offset), summed in rank order in float32, scaled, rounded."""
    off = g.data_ptr() - arena.tensor.data_ptr()
    nbytes = g.numel() * g.element_size()
    acc = None
    for c in copies:
        t = c[off:off + nbytes].view(g.dtype).view(g.shape).float()
        acc = t if acc is None else acc + t
    return (acc * torch.tensor(scale, dtype=torch.float32)).to(g.dtype)


class OracleBackend:
    """CPU arithmetic for the sharded step (test only)."""

    def grad_arena(self, nbytes, device, process_group):
        return CpuArena(nbytes, device, process_group)

    @staticmethod
    def _gather(reduce):
        arena, _ = reduce
        copies = [torch.empty_like(arena.tensor) for _ in range(dist.get_world_size(arena.pg))]
        dist.all_gather(copies, arena.tensor, group=arena.pg)
        return copies

    def adamw(self, quads, *, lr, beta1, beta2, eps, weight_decay, bias1, bias2, timer=None, reduce=None):
        copies = self._gather(reduce) if reduce is not None else None
        for q in quads:
            (p, g, m, v), shadow = q[:4], (q[4] if len(q) > 4 else None)
            if reduce is not None:
                g = reduced(g, copies, *reduce)
            if shadow is not None:      # float32 master, bf16 gradient widened, bf16 copy written
                g = g.float()
            adamw_update_(p, g, m, v, lr=lr, beta1=beta1, beta2=beta2, eps=eps, weight_decay=weight_decay,
                          bias1=bias1, bias2=bias2)
            if shadow is not None:
                shadow.copy_(p.to(shadow.dtype))

    def muon(self, bucket, triples, *, adjust_lr_fn, beta, nesterov, a, b, c, ns_steps, eps, lr, weight_decay,
             timer=None, reduce=None):
        copies = self._gather(reduce) if reduce is not None else None
        for t in triples:
            (p, g, mom), shadow = t[:3], (t[3] if len(t) > 3 else None)
            if reduce is not None:
                g = reduced(g, copies, *reduce)
            if shadow is not None:
                g = g.float()
            muon_matrix_step_(p, g, mom, lr=lr, beta=beta, nesterov=nesterov, coeffs=(a, b, c), ns_steps=ns_steps,
                              eps=eps, weight_decay=weight_decay, adjust_lr_fn=adjust_lr_fn)
            if shadow is not None:
                shadow.copy_(p.to(shadow.dtype))


def _make(seed=0, dtype=torch.float32):
    gen = torch.Generator().manual_seed(seed)
    adam = [torch.nn.Parameter((torch.randn(s, generator=gen) * 0.02).to(dtype)) for s in ADAM_SHAPES]
    muon = [torch.nn.Parameter((torch.randn(s, generator=gen) * 0.02).to(dtype)) for s in MUON_SHAPES]
    return adam, muon


def _grads(step, dtype=torch.float32):
    gen = torch.Generator().manual_seed(100 + step)
    return ([(torch.randn(s, generator=gen) * 1e-2).to(dtype) for s in ADAM_SHAPES],
            [(torch.randn(s, generator=gen) * 1e-2).to(dtype) for s in MUON_SHAPES])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ----------------------------------------------------------------- pure logic
def test_lpt_balances_ns_cost():
    from oracle.muon_adamw_oracle import llama_8b_shapes
    from triton_muon_adamw.distributed import lpt_assign, ns_cost
    _, muon = llama_8b_shapes()
    costs = [ns_cost(s) for s in muon]
    for n in (2, 4, 8):
        owner = lpt_assign(costs, n)
        load = [sum(c for c, o in zip(costs, owner) if o == r) for r in range(n)]
        assert max(load) / (sum(costs) / n) < 1.02, (n, load)
        assert owner == lpt_assign(costs, n)          # deterministic on every rank


def test_split_buckets_increasing_and_decreasing():
    """Decreasing buckets (the sharded exchange) and increasing ones (the host-gradient pipeline)."""
    from triton_muon_adamw.distributed import split_buckets
    costs = [1.0] * 150
    for increasing in (False, True):
        b = split_buckets(costs, 5, increasing=increasing)
        assert b == sorted(b) and set(b) == set(range(5))            # contiguous, every bucket used
        sizes = [b.count(k) for k in range(5)]
        assert sizes == sorted(sizes, reverse=not increasing), sizes
        assert abs(sizes[0] - (10 if increasing else 50)) <= 1 and abs(sizes[-1] - (50 if increasing else 10)) <= 1


def test_zero1_pieces_partition_every_element_once():
    from triton_muon_adamw.distributed import ALIGN, shard_pieces, zero1_layout
    numels = [100, 37, 192, 5, 129, 4096, 1]
    for n in (1, 2, 3, 8):
        offsets, shard, total = zero1_layout(numels, n)
        assert shard % ALIGN == 0 and total == shard * n and all(o % ALIGN == 0 for o in offsets)
        covered = [torch.zeros(k, dtype=torch.int32) for k in numels]
        for r in range(n):
            for i, start, length, sh in shard_pieces(offsets, numels, r * shard, (r + 1) * shard):
                assert 0 <= sh and sh + length <= shard
                covered[i][start:start + length] += 1
        assert all(bool((c == 1).all()) for c in covered)


def test_muon_layout_segments_do_not_overlap():
    from triton_muon_adamw.distributed import ALIGN, muon_layout
    for n, nb in ((2, 2), (3, 4), (8, 4)):
        slots, segs = muon_layout(MUON_SHAPES, n, nb)
        for b, seg in enumerate(segs):
            ranges = sorted((s.offset, s.offset + s.numel) for s in slots if s.bucket == b)
            for (a0, a1), (b0, _) in zip(ranges, ranges[1:]):
                assert a1 <= b0
            for s in slots:
                if s.bucket == b:
                    assert s.offset % ALIGN == 0
                    assert s.owner * seg <= s.offset and s.offset + s.numel <= (s.owner + 1) * seg


# ----------------------------------------------------------------- gloo ranks
def _worker(rank, world, port, mode, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        from triton_muon_adamw import AdamConfig, MuonConfig
        from triton_muon_adamw.distributed import ShardedMuonAdamW
        dtype = torch.bfloat16 if mode in ("bf16", "reduce_bf16", "master") else torch.float32
        reduce = mode.startswith("reduce")
        master = mode == "master"
        adam, muon = _make(dtype=dtype)
        # Master mode: the reference is a float32 run on the masters with the bf16 gradients widened.
        ref_dtype = torch.float32 if master else dtype
        ref = OracleMuonAdamW([p.detach().to(ref_dtype) for p in adam], [p.detach().to(ref_dtype) for p in muon],
                              adam=ADAM, muon=MUON)
        opt = ShardedMuonAdamW(adam, muon, MuonConfig(**MUON), AdamConfig(**ADAM), dist.group.WORLD, n_buckets=2,
                               backend=OracleBackend(), reduce_grads="mean" if reduce else None,
                               master_weights=master)
        if mode == "die" and rank == 1:
            raise SystemExit(0)     # leaves before the first collective
        for step in range(2):
            ga, gm = _grads(step, dtype)
            if reduce:
                # Data-parallel: rank r holds its own gradients; the step uses their mean.
                per_rank = [[(g.float() * (1 + 0.25 * r) + 1e-3 * r).to(dtype) for g in ga + gm]
                            for r in range(world)]
                mean = [(sum(per_rank[r][i].float() for r in range(world)) * torch.tensor(1.0 / world)).to(dtype)
                        for i in range(len(ga + gm))]
                mine = per_rank[rank]
                for i, (p, g) in enumerate(zip(adam + muon, mine)):
                    if step == 0 and i % 2 == 0:
                        p.grad = g.clone()       # a gradient outside the arena: copied in at step()
                    else:
                        p.grad.copy_(g)          # in place, inside the arena
                ga, gm = mean[:len(ga)], mean[len(ga):]
            else:
                for p, g in zip(adam + muon, ga + gm):
                    p.grad = g.clone()
            opt.step()
            if master:
                ga, gm = [g.float() for g in ga], [g.float() for g in gm]
            ref.step(ga, gm)
        for p, r in zip(adam + muon, ref.params_adam + ref.params_muon):
            want = r.to(dtype) if master else r
            assert p.dtype == dtype and torch.equal(p.detach(), want), f"rank {rank}: parameter {tuple(p.shape)} differs"
        sd = opt.state_dict()
        for i, (m, v) in enumerate(zip(ref.exp_avg, ref.exp_avg_sq)):
            assert torch.equal(sd["adam"]["state"][i]["exp_avg"], m)
            assert torch.equal(sd["adam"]["state"][i]["exp_avg_sq"], v)
        for i, mom in enumerate(ref.momentum):
            assert torch.equal(sd["muon"]["state"][i]["momentum_buffer"], mom)
        if master:
            for i, r in enumerate(ref.params_adam):
                assert torch.equal(sd["adam"]["state"][i]["master_param"], r)
            for i, r in enumerate(ref.params_muon):
                assert torch.equal(sd["muon"]["state"][i]["master_param"], r)
        # round trip: zero the shards, load the gathered dict back, gather again
        opt.exp_avg.zero_()
        for t in opt.mom_segs:
            t.zero_()
        opt.load_state_dict(sd)
        sd2 = opt.state_dict()
        assert torch.equal(sd2["adam"]["state"][0]["exp_avg"], sd["adam"]["state"][0]["exp_avg"])
        assert torch.equal(sd2["muon"]["state"][3]["momentum_buffer"], sd["muon"]["state"][3]["momentum_buffer"])
        # Gathered to one rank in host memory, then scattered back from it (the others pass None).
        sd0 = opt.state_dict(to_rank=0, cpu=True)
        if rank != 0:
            assert sd0 == {}
        opt.exp_avg.zero_()
        opt.exp_avg_sq.zero_()
        for t in opt.mom_segs + list(opt.master_segs):
            t.zero_()
        opt.load_state_dict(sd0 if rank == 0 else None, from_rank=0)
        sd5 = opt.state_dict()
        for br in ("adam", "muon"):
            assert sorted(sd5[br]["state"]) == sorted(sd[br]["state"])
            for i, st in sd[br]["state"].items():
                for name, t in st.items():
                    assert torch.equal(sd5[br]["state"][i][name], t), (br, i, name)
        if master:
            # A dict without masters (PyTorchMuonAdamW's layout) after the model's parameters changed: the
            # masters restart from the current bf16 parameters, and the next step continues from them.
            with torch.no_grad():
                for p in adam + muon:
                    p.mul_(0.5)
            bare = {k: {"state": {i: {n: t for n, t in st.items() if n != "master_param"}
                                  for i, st in sd[k]["state"].items()},
                        "param_groups": sd[k]["param_groups"]} for k in ("adam", "muon")}
            opt.load_state_dict(bare)
            sd3 = opt.state_dict()
            for k, ps in (("adam", adam), ("muon", muon)):
                for i, p in enumerate(ps):
                    assert torch.equal(sd3[k]["state"][i]["master_param"], p.detach().float()), (k, i)
            for r, p in zip(ref.params_adam + ref.params_muon, adam + muon):
                r.copy_(p.detach().float())
            ga, gm = _grads(2, dtype)
            for p, g in zip(adam + muon, ga + gm):
                p.grad = g.clone()
            opt.step()
            ref.step([g.float() for g in ga], [g.float() for g in gm])
            for p, r in zip(adam + muon, ref.params_adam + ref.params_muon):
                assert torch.equal(p.detach(), r.to(dtype)), f"rank {rank}: {tuple(p.shape)} after a master-less load"
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except SystemExit:
        q.put((rank, "left"))
    except Exception as e:  # reported to the parent
        q.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-800:]}"))


def _worker_edge(rank, world, port, case, q):
    """Degenerate layouts: a branch without parameters, more ranks and buckets than Muon matrices."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        from triton_muon_adamw import AdamConfig, MuonConfig
        from triton_muon_adamw.distributed import ShardedMuonAdamW
        adam, muon = _make()
        if case == "no_adam":
            adam = []
        elif case == "no_muon":
            muon = []
        elif case == "few_muon":
            muon = muon[:2]
        ref = OracleMuonAdamW([p.detach().clone() for p in adam], [p.detach().clone() for p in muon],
                              adam=ADAM, muon=MUON)
        opt = ShardedMuonAdamW(adam, muon, MuonConfig(**MUON), AdamConfig(**ADAM), dist.group.WORLD, n_buckets=5,
                               backend=OracleBackend())
        for step in range(2):
            ga, gm = _grads(step)
            ga, gm = ga[:len(adam)], [g for g, _ in zip(gm, muon)]
            for p, g in zip(adam + muon, ga + gm):
                p.grad = g.clone()
            opt.step()
            ref.step(ga, gm)
        for p, r in zip(adam + muon, ref.params_adam + ref.params_muon):
            assert torch.equal(p.detach(), r), f"rank {rank}: {case} parameter {tuple(p.shape)} differs"
        sd = opt.state_dict()
        assert len(sd["adam"]["state"]) == len(adam) and len(sd["muon"]["state"]) == len(muon)
        opt.load_state_dict(sd)
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        q.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-800:]}"))


def _run(world, mode, target=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target or _worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    out = {}
    while not q.empty():
        r, msg = q.get()
        out[r] = msg
    return out


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_step_matches_single_process_oracle(world):
    out = _run(world, "normal")
    assert out == {r: "ok" for r in range(world)}, out


def test_sharded_step_bf16_parameters():
    """bf16 parameters: bf16 flat buffers and momentum, float32 AdamW moment shards."""
    out = _run(2, "bf16")
    assert out == {0: "ok", 1: "ok"}, out


@pytest.mark.parametrize("world,case", [(2, "no_adam"), (2, "no_muon"), (3, "few_muon")])
def test_sharded_step_degenerate_layouts(world, case):
    out = _run(world, case, target=_worker_edge)
    assert out == {r: "ok" for r in range(world)}, out


def test_sharded_step_master_weights():
    """bf16 parameters with float32 masters on the owners: bit-identical to a float32 run on the masters."""
    out = _run(2, "master")
    assert out == {0: "ok", 1: "ok"}, out


@pytest.mark.parametrize("world,mode", [(2, "reduce"), (3, "reduce"), (2, "reduce_bf16")])
def test_sharded_step_reduces_per_rank_gradients(world, mode):
    """reduce_grads="mean": each rank's own gradients, read from the gradient arenas of all ranks at the
    owner's offsets, summed in rank order -- the result equals one step on the mean gradients."""
    out = _run(world, mode)
    assert out == {r: "ok" for r in range(world)}, out


def test_rank_that_leaves_surfaces_as_collective_error():
    """A rank that exits before the exchange: the survivor's step fails with an error, it does not hang."""
    out = _run(2, "die")
    assert out.get(1) == "left"
    assert out.get(0, "").split(":")[0] in ("RuntimeError", "DistBackendError", "DistError"), out


def test_cuda_backend_offers_every_call_the_sharded_step_makes():
    """The CPU runs above use OracleBackend; the CUDA backend must take the same calls."""
    import inspect

    from triton_muon_adamw.distributed import CudaBackend
    def params(fn):
        return [(p.name, p.kind, p.default) for p in inspect.signature(fn).parameters.values()]

    for name in ("adamw", "muon", "grad_arena"):
        assert params(getattr(CudaBackend, name)) == params(getattr(OracleBackend, name)), name
    for name in ("status", "param_arena", "push_segment"):
        assert callable(getattr(CudaBackend, name, None)), name
    with pytest.raises(ValueError):
        CudaBackend(push="tree")


def test_sms_handed_to_the_nccl_exchange():
    """reserve_sms=0 (default) keeps the caller's group for the NCCL all-gathers (NCCL's own CTA
    count, every SM for the GEMMs); a reserve applies to the NCCL exchange only."""
    from triton_muon_adamw.distributed import CudaBackend

    sentinel = object()
    b = CudaBackend(push="nccl")
    assert b.reserve_sms == 0
    assert b.param_arena(1 << 20, torch.device("cpu"), None) is None
    assert b.exchange_group(sentinel) is sentinel
    assert CudaBackend(push="copy_engine", reserve_sms=8).exchange_group(sentinel) is sentinel
    with pytest.raises(ValueError):
        CudaBackend(push="nccl", reserve_sms=65)


def test_mixed_exchange_sends_the_early_exchanges_by_copy_engine():
    """push="mixed": the first ce_exchanges exchanges of a step are written into the peers'
    replicas (copy engines), the later ones go by NCCL all-gather; the other modes are uniform."""
    from triton_muon_adamw.distributed import CudaBackend

    b = CudaBackend(push="mixed")
    assert [b.exchange_kind(i) for i in range(6)] == ["push"] * 3 + ["nccl"] * 3
    b = CudaBackend(push="mixed", ce_exchanges=1)
    assert [b.exchange_kind(i) for i in range(3)] == ["push", "nccl", "nccl"]
    assert CudaBackend(push="copy_engine").exchange_kind(9) == "push"
    n = CudaBackend(push="nccl")
    n.param_arena(1 << 20, torch.device("cpu"), None)
    assert n.exchange_kind(0) == "nccl"
    with pytest.raises(ValueError):
        CudaBackend(push="mixed", ce_exchanges=-1)
