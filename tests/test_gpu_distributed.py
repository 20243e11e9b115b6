"""Sharded MuonAdamW over NCCL on 2, 4 and 8 GPUs vs the single-GPU step (needs >= 2 B200s).

Every kernel is deterministic and a matrix's result does not depend on which
rank or bucket computes it, so the sharded step must reproduce the single-GPU
step bit for bit on every rank.  The fused gradient reduction is also held to
the CPU oracle's step on the mean gradients (the reference's tolerances:
AdamW atol 1e-4 / rtol 1e-3, Muon atol/rtol 1e-2).
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

pytestmark = pytest.mark.gpu

COEFFS = (3.4445, -4.7750, 2.0315)
ADAM_SHAPES = [(1000, 64), (64,), (300,), (64,)]
MUON_SHAPES = [(256, 64), (64, 256), (512, 512), (128, 96), (1024, 256), (96, 96), (300, 200), (64, 64)]


def _params(device):
    gen = torch.Generator().manual_seed(0)
    adam = [torch.nn.Parameter((torch.randn(s, generator=gen) * 0.02).to(device)) for s in ADAM_SHAPES]
    muon = [torch.nn.Parameter((torch.randn(s, generator=gen) * 0.02).to(device)) for s in MUON_SHAPES]
    return adam, muon


def _grads(step, device):
    gen = torch.Generator().manual_seed(50 + step)
    return [(torch.randn(s, generator=gen) * 1e-3).to(device) for s in ADAM_SHAPES + MUON_SHAPES]


def _worker_reduce(rank, world, port, q, dtype):
    """reduce_grads="mean": per-rank gradients read over NVLink vs one single-GPU step on their mean."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
        from triton_muon_adamw import AdamConfig, MuonAdamW, MuonConfig
        mc, ac = MuonConfig(coeffs=COEFFS), AdamConfig(lr=3e-4, betas=(0.9, 0.95))
        adam, muon = _params(dev)
        adam, muon = ([torch.nn.Parameter(p.detach().to(dtype)) for p in ps] for ps in (adam, muon))
        sharded = MuonAdamW({"adam": adam, "muon": muon}, muon_config=mc, adam_config=ac,
                            parameter_split="explicit", process_group=dist.group.WORLD, reduce_grads="mean")
        adam1, muon1 = _params(dev)
        adam1, muon1 = ([torch.nn.Parameter(p.detach().to(dtype)) for p in ps] for ps in (adam1, muon1))
        single = MuonAdamW({"adam": adam1, "muon": muon1}, muon_config=mc, adam_config=ac, parameter_split="explicit")
        for step in range(3):
            base = _grads(step, dev)
            per_rank = [[(g * (1 + 0.5 * r) + 1e-4 * r).to(dtype) for g in base] for r in range(world)]
            for i, (p, g) in enumerate(zip(adam + muon, per_rank[rank])):
                if step == 1 and i % 3 == 0:
                    p.grad = g.clone()           # outside the shared buffer: copied in by step()
                else:
                    p.grad.copy_(g)
            for i, p1 in enumerate(adam1 + muon1):
                acc = per_rank[0][i].float()
                for r in range(1, world):
                    acc = acc + per_rank[r][i].float()
                p1.grad = (acc * (1.0 / world)).to(dtype)
            sharded.step()
            single.step()
        torch.cuda.synchronize()
        for p, p1 in zip(adam + muon, adam1 + muon1):
            assert torch.equal(p.detach(), p1.detach()), f"rank {rank}: {tuple(p.shape)} {dtype} differs"
        assert sharded.device_status() == 0 and single.device_status() == 0
        if dtype == torch.float32:
            # The oracle's step on the mean gradients (rank-order float32 sum, as the kernels form it).
            from oracle.muon_adamw_oracle import OracleMuonAdamW
            a0, m0 = _params(torch.device("cpu"))
            ref = OracleMuonAdamW([p.detach().clone() for p in a0], [p.detach().clone() for p in m0],
                                  adam=dict(lr=ac.lr, betas=ac.betas, eps=ac.eps, weight_decay=ac.weight_decay),
                                  muon=dict(lr=mc.lr, beta=mc.beta, eps=mc.eps, weight_decay=mc.weight_decay,
                                            coeffs=mc.coeffs, nesterov=mc.nesterov, ns_steps=mc.ns_steps,
                                            normalize="fold"))
            for step in range(3):
                base = [g.cpu() for g in _grads(step, dev)]
                mean = []
                for g in base:
                    acc = g.float()
                    for r in range(1, world):
                        acc = acc + (g * (1 + 0.5 * r) + 1e-4 * r).float()
                    mean.append(acc * (1.0 / world))
                ref.step(mean[:len(ADAM_SHAPES)], mean[len(ADAM_SHAPES):])
            for p, r in zip(adam, ref.params_adam):
                torch.testing.assert_close(p.detach().cpu(), r, atol=1e-4, rtol=1e-3)
            for p, r in zip(muon, ref.params_muon):
                torch.testing.assert_close(p.detach().cpu(), r, atol=1e-2, rtol=1e-2)
        sharded.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        q.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-1500:]}"))


def _worker_master(rank, world, port, q):
    """master_weights=True sharded (bf16 exchange, float32 masters on the owners) vs single-GPU master mode."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
        from triton_muon_adamw import AdamConfig, MuonAdamW, MuonConfig
        mc, ac = MuonConfig(coeffs=COEFFS), AdamConfig(lr=3e-4, betas=(0.9, 0.95))

        def bf16_params():
            adam, muon = _params(dev)
            return ([torch.nn.Parameter(p.detach().to(torch.bfloat16)) for p in ps] for ps in (adam, muon))

        adam, muon = bf16_params()
        sharded = MuonAdamW({"adam": adam, "muon": muon}, muon_config=mc, adam_config=ac, parameter_split="explicit",
                            process_group=dist.group.WORLD, master_weights=True)
        adam1, muon1 = bf16_params()
        single = MuonAdamW({"adam": adam1, "muon": muon1}, muon_config=mc, adam_config=ac,
                           parameter_split="explicit", master_weights=True)
        for step in range(3):
            gs = [g.to(torch.bfloat16) for g in _grads(step, dev)]
            for p, p1, g in zip(adam + muon, adam1 + muon1, gs):
                p.grad, p1.grad = g.clone(), g.clone()
            sharded.step()
            single.step()
        torch.cuda.synchronize()
        for p, p1 in zip(adam + muon, adam1 + muon1):
            assert torch.equal(p.detach(), p1.detach()), f"rank {rank}: {tuple(p.shape)} differs"
        sd, ref = sharded.state_dict(), single.state_dict()
        for br in ("adam", "muon"):
            for i in ref[br]["state"]:
                assert torch.equal(sd[br]["state"][i]["master_param"], ref[br]["state"][i]["master_param"]), (br, i)
        sharded.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        q.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-1500:]}"))


def _worker_host(rank, world, port, q):
    """Sharded step_from_host (host gradients, copies overlapped) vs the single-GPU step()."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
        from triton_muon_adamw import AdamConfig, MuonAdamW, MuonConfig
        mc, ac = MuonConfig(coeffs=COEFFS), AdamConfig(lr=3e-4, betas=(0.9, 0.95))
        adam, muon = _params(dev)
        sharded = MuonAdamW({"adam": adam, "muon": muon}, muon_config=mc, adam_config=ac,
                            parameter_split="explicit", process_group=dist.group.WORLD)
        adam1, muon1 = _params(dev)
        single = MuonAdamW({"adam": adam1, "muon": muon1}, muon_config=mc, adam_config=ac, parameter_split="explicit")
        for step in range(3):
            gs = _grads(step, dev)
            sharded.step_from_host({p: g.cpu().pin_memory() for p, g in zip(adam + muon, gs)})
            for p1, g in zip(adam1 + muon1, gs):
                p1.grad = g.clone()
            single.step()
        torch.cuda.synchronize()
        for p, p1 in zip(adam + muon, adam1 + muon1):
            assert torch.equal(p.detach(), p1.detach()), f"rank {rank}: {tuple(p.shape)} differs"
        sharded.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        q.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-1500:]}"))


def _worker(rank, world, port, q, push="auto"):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
        from triton_muon_adamw import AdamConfig, MuonAdamW, MuonConfig
        mc, ac = MuonConfig(coeffs=COEFFS), AdamConfig(lr=3e-4, betas=(0.9, 0.95))
        adam, muon = _params(dev)
        sharded = MuonAdamW({"adam": adam, "muon": muon}, muon_config=mc, adam_config=ac,
                            parameter_split="explicit", process_group=dist.group.WORLD, peer_push=push)
        adam1, muon1 = _params(dev)
        single = MuonAdamW({"adam": adam1, "muon": muon1}, muon_config=mc, adam_config=ac, parameter_split="explicit")
        for step in range(3):
            gs = _grads(step, dev)
            for p, p1, g in zip(adam + muon, adam1 + muon1, gs):
                p.grad, p1.grad = g.clone(), g.clone()
            sharded.step()
            single.step()
        torch.cuda.synchronize()
        for p, p1 in zip(adam + muon, adam1 + muon1):
            assert torch.equal(p.detach(), p1.detach()), f"rank {rank}: {tuple(p.shape)} differs"
        assert sharded.device_status() == 0 and single.device_status() == 0
        sd = sharded.state_dict()
        ref = single.state_dict()
        for i in ref["muon"]["state"]:
            assert torch.equal(sd["muon"]["state"][i]["momentum_buffer"], ref["muon"]["state"][i]["momentum_buffer"])
        for i in ref["adam"]["state"]:
            assert torch.equal(sd["adam"]["state"][i]["exp_avg_sq"], ref["adam"]["state"][i]["exp_avg_sq"])
        # A sharded checkpoint resumes on one GPU: a fresh single-GPU optimizer over the current
        # parameters loads the gathered dict and steps exactly as the sharded one does.
        resumed = [torch.nn.Parameter(p.detach().clone()) for p in adam + muon]
        na = len(adam)
        one = MuonAdamW({"adam": resumed[:na], "muon": resumed[na:]}, muon_config=mc, adam_config=ac,
                        parameter_split="explicit")
        one.load_state_dict(sd)
        gs = _grads(3, dev)
        for p, p1, g in zip(adam + muon, resumed, gs):
            p.grad, p1.grad = g.clone(), g.clone()
        sharded.step()
        one.step()
        torch.cuda.synchronize()
        for p, p1 in zip(adam + muon, resumed):
            assert torch.equal(p.detach(), p1.detach()), f"rank {rank}: {tuple(p.shape)} after a sharded checkpoint"
        sharded.close()
        for p, p1 in zip(adam + muon, resumed):            # parameters survive close() as private copies
            assert torch.equal(p.detach(), p1.detach())
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        q.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-1500:]}"))


def _spawn(target, world, *extra):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=target, args=(r, world, port, q, *extra)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    out = {}
    while not q.empty():
        r, msg = q.get()
        out[r] = msg
    return out


@pytest.mark.parametrize("world,push", [(2, "auto"), (2, "nccl"), (2, "kernel"), (2, "hybrid"), (2, "mixed"),
                                        (4, "auto"), (8, "auto"), (8, "copy_engine"), (8, "mixed")])
def test_sharded_step_is_bit_identical(world, push):
    """Every way of exchanging the updated parameters (peer_push), at 2, 4 and 8 ranks -- 8 with the
    NCCL all-gather that "auto" picks there, as in the scaling runs -- gives the single-GPU result."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = _spawn(_worker, world, push)
    assert out == {r: "ok" for r in range(world)}, out


@pytest.mark.parametrize("world,dtype", [(2, torch.float32), (2, torch.bfloat16), (4, torch.float32),
                                         (8, torch.float32)])
def test_fused_gradient_reduction(world, dtype):
    """Each rank's own gradients, summed over NVLink inside the AdamW and Muon-prep kernels."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = _spawn(_worker_reduce, world, dtype)
    assert out == {r: "ok" for r in range(world)}, out


def test_two_gpu_master_weights_sharded_step():
    """bf16 parameters exchanged between ranks, float32 masters kept by their owners."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = _spawn(_worker_master, 2)
    assert out == {0: "ok", 1: "ok"}, out


def test_two_gpu_step_from_host_matches_step():
    """Host-resident gradients: each rank copies the pieces it owns, overlapped with the work."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = _spawn(_worker_host, 2)
    assert out == {0: "ok", 1: "ok"}, out
