"""Benchmark: one full MuonAdamW optimizer step on the Llama-3-8B-shaped parameter set.

    python bench.py [--gpus N --steps K --warmup W] [--config 8b|1b3|prof] [--impl ours|reference|reference-triton]

A step is one ``MuonAdamW.step()`` (AdamW branch + Muon branch with ns_steps
Newton-Schulz iterations) over the whole synthetic parameter set, already in
HBM.  ``value`` is the device-timed ms/step (CUDA events, max over ranks);
``e2e`` repeats the step through the public API with this step's gradients
copied in from pinned host memory and a small result read back, all inside
the timed region.  ``roofline`` reports the dominant kernel (the tcgen05
Newton-Schulz update GEMM) against the measured peaks in MEASURED_PEAKS.json,
timed live with CUDA events on the launching stream; ``kernels`` has every
kernel family.  ``cpu_baseline`` times the reference's CPU path
(``torch.optim`` AdamW(fused) + Muon, the PyTorchMuonAdamW wrapper, restated
under oracle/) on a bounded sample and extrapolates to the full step.

At N>1 the line also carries ``grad_reduce``: the step with per-rank
(data-parallel) gradients reduced inside its first kernels (``reduce_grads``)
against an NCCL all-reduce of the same gradient bytes (``--no-grad-reduce``
skips it); ``--push`` picks how updated parameters reach the other ranks
(``MuonAdamW(peer_push=...)``, default ``auto``).

With ``--impl reference`` only that CPU measurement runs (rank 0), each step a
bounded sample extrapolated to the full step.  ``--impl reference-triton``
times the reference's own Triton ``MuonAdamW`` (the unmodified package
installed under ``baseline/_ref``) on this GPU with the same shapes and
synthetic data (rank 0 only; the reference is single-GPU).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "triton-muonadamw_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402
import torch.nn as nn  # noqa: E402

COEFFS = (3.4445, -4.7750, 2.0315)
HBM_FALLBACK, TF_FALLBACK, TF_SUSTAINED_FALLBACK = 6650.0, 1590.0, 1400.0


# ----------------------------------------------------------------- configs
def llama_shapes(d, layers, n_heads, n_kv_heads, ffn, vocab, tied=False):
    hd = d // n_heads
    adam = [("embed", (vocab, d))] + ([] if tied else [("head", (vocab, d))])
    muon = []
    for i in range(layers):
        adam += [(f"l{i}.attn_norm", (d,)), (f"l{i}.ffn_norm", (d,))]
        muon += [(f"l{i}.wq", (n_heads * hd, d)), (f"l{i}.wk", (n_kv_heads * hd, d)),
                 (f"l{i}.wv", (n_kv_heads * hd, d)), (f"l{i}.wo", (d, n_heads * hd)),
                 (f"l{i}.gate", (ffn, d)), (f"l{i}.up", (ffn, d)), (f"l{i}.down", (d, ffn))]
    adam.append(("final_norm", (d,)))
    return adam, muon


def profiling_shapes():
    """Small case for ncu captures: one matrix of each 8B Muon orientation (about 2 GB on the device)."""
    return [("embed", (4096, 4096)), ("final_norm", (4096,))], [("wide", (4096, 14336)), ("tall", (14336, 4096)),
                                                                 ("square", (4096, 4096))]


CONFIGS = {
    "8b": dict(name="llama3-8b-shaped", shapes=lambda: llama_shapes(4096, 32, 32, 8, 14336, 128256),
               adam=dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01)),
    "1b3": dict(name="llama-1.3b", shapes=lambda: llama_shapes(2048, 24, 16, 16, 5504, 32000),
                adam=dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01)),
    "prof": dict(name="profiling-case (3 Muon matrices of the 8B shapes)", shapes=profiling_shapes,
                 adam=dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01)),
}


class ShapedParams(nn.Module):
    """Parameter container with the named shapes; embed/head exposed for the auto split."""

    def __init__(self, adam, muon, device, seed):
        super().__init__()
        gen = torch.Generator(device=device).manual_seed(seed)
        self.names = []
        for name, shape in adam + muon:
            t = torch.empty(shape, device=device, dtype=torch.float32)
            t.normal_(0.0, 0.02, generator=gen)
            self.register_parameter(name.replace(".", "_"), nn.Parameter(t))
            self.names.append(name.replace(".", "_"))
        self._embed = nn.Module()
        self._embed.weight = self.embed
        self._head = nn.Module() if hasattr(self, "head") else None
        if self._head is not None:
            self._head.weight = self.head

    def get_input_embeddings(self):
        return self._embed

    def get_output_embeddings(self):
        return self._head


# ----------------------------------------------------------------- helpers
def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return HBM_FALLBACK, TF_FALLBACK, TF_SUSTAINED_FALLBACK, "fallback"


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.3)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        load = [s for s in sm if smax and s > 0.5 * max(smax)] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


class PhaseTimer:
    """CUDA events around each launch of the step, on the launching (current) stream."""

    def __init__(self):
        self.events = []

    def mark(self, label):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.events.append((label, e))

    def durations(self):
        out = {}
        for (label, a), (_, b) in zip(self.events, self.events[1:]):
            if label is None:
                continue
            out.setdefault(label, []).append(a.elapsed_time(b))
        return out


def ns_flops_sym(shape):
    m, n = min(shape), max(shape)
    return {"gram": float(m) * m * n, "poly": float(m) ** 3, "update": 2.0 * m * m * n}


# Launches of each NS phase per step: ns_steps of Gram and polynomial, ns_steps - 1 plain updates
# and one last update (which writes the parameters).
def ns_phase_launches(phase, ns_steps):
    return {"gram": ns_steps, "poly": ns_steps, "update": ns_steps - 1, "update_last": 1}[phase]


# ----------------------------------------------------------------- CPU baseline
def cpu_sample(cfg_key, adam_cfg, ns_steps):
    """Time the reference's CPU path on one matrix per distinct Muon shape + an AdamW chunk; extrapolate."""
    from oracle.muon_adamw_oracle import ReferenceWrapperCPU  # noqa: PLC0415
    torch.set_num_threads(os.cpu_count() or 1)
    adam, muon = CONFIGS[cfg_key]["shapes"]()
    counts = {}
    for _, s in muon:
        counts[s] = counts.get(s, 0) + 1
    gen = torch.Generator().manual_seed(0)
    muon_cfg = dict(lr=1e-3, beta=0.95, eps=1e-7, weight_decay=0.1, nesterov=True, ns_steps=ns_steps,
                    adjust_lr_fn="original")
    total_ms, detail = 0.0, {}
    for shape, cnt in counts.items():
        p = nn.Parameter(torch.randn(shape, generator=gen) * 0.02)
        p.grad = torch.randn(shape, generator=gen) * 1e-3
        w = ReferenceWrapperCPU([], [p], adam=adam_cfg, muon=muon_cfg)
        t0 = time.perf_counter()
        w.step()
        dt = (time.perf_counter() - t0) * 1e3
        detail[f"{shape[0]}x{shape[1]}"] = round(dt, 1)
        total_ms += dt * cnt
    adam_elems = sum(math.prod(s) for _, s in adam)
    chunk = 1 << 24
    p = nn.Parameter(torch.randn(chunk, generator=gen) * 0.02)
    p.grad = torch.randn(chunk, generator=gen) * 1e-3
    w = ReferenceWrapperCPU([p], [], adam=adam_cfg, muon=muon_cfg)
    w.step()
    t0 = time.perf_counter()
    w.step()
    dt = (time.perf_counter() - t0) * 1e3
    detail["adamw_16M"] = round(dt, 1)
    total_ms += dt * adam_elems / chunk
    sample = (f"one matrix per distinct Muon shape ({', '.join(detail)}) through torch.optim.Muon, one 16M-element "
              f"chunk through torch.optim.AdamW(fused); extrapolated by shape counts and element count")
    return total_ms, sample, torch.get_num_threads(), detail


# ----------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="8b", choices=sorted(CONFIGS) + list(SWEEPS),
                    help="8b (default: the Llama-3-8B-shaped step), 1b3, prof (small ncu case), or the "
                         "isolated sweeps adamw_sweep (C2) and ns_isolated (C3)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-triton"])
    ap.add_argument("--ns-steps", type=int, default=5)
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--push", default="auto", choices=["auto", "nccl", "copy_engine", "kernel", "hybrid", "mixed"],
                    help="at N>1, how updated parameters reach the other ranks (MuonAdamW peer_push)")
    ap.add_argument("--no-grad-reduce", action="store_true",
                    help="at N>1, skip timing the step with per-rank gradients reduced inside it (reduce_grads)")
    ap.add_argument("--no-reference-triton", action="store_true",
                    help="at N=1, skip timing the reference's own Triton MuonAdamW on this GPU after our arm")
    ap.add_argument("--reserve-sms", type=int, default=0,
                    help="at N>1 with the NCCL exchange, SMs handed to it: the Newton-Schulz GEMMs leave them free "
                         "and NCCL is capped to as many CTAs (MuonAdamW reserve_sms)")
    ap.add_argument("--realloc-grads", action="store_true",
                    help="alternate every step between two sets of gradient tensors (new .grad addresses each "
                         "step, as zero_grad(set_to_none=True) + backward gives): the plans patch the addresses")
    ap.add_argument("--cases", default=None,
                    help="sweeps only: comma-separated case names to run (adamw_sweep: 1M,16M,64M,256M,ragged_10k; "
                         "ns_isolated: SHAPExBATCH, e.g. 4096x14336x32)")
    ap.add_argument("--impls", default=None,
                    help="adamw_sweep only: comma-separated implementations (ours,reference_triton,torch_fused); "
                         "profiler captures leave out the reference's ragged case (10,000 launches a step)")
    ap.add_argument("--no-verify", action="store_true",
                    help="at N>1, skip the post-timing check of every replica against a single-GPU recomputation")
    args = ap.parse_args()
    if args.config in SWEEPS:
        if int(os.environ.get("RANK", "0")) == 0:
            SWEEPS[args.config](args)
        return
    cfg = CONFIGS[args.config]

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        run_reference_arm(args, cfg, world)
        return
    if args.impl == "reference-triton":
        if rank != 0:
            return
        run_reference_triton_arm(args, cfg, world, local_rank)
        return

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    pg = None
    if world > 1:
        from datetime import timedelta  # noqa: PLC0415
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
        pg = dist.group.WORLD

    from triton_muon_adamw import AdamConfig, MuonAdamW, MuonConfig  # noqa: PLC0415

    adam_shapes, muon_shapes = cfg["shapes"]()
    model = ShapedParams(adam_shapes, muon_shapes, dev, seed=0)
    ggen = torch.Generator(device=dev).manual_seed(1)
    for p in model.parameters():
        p.grad = torch.empty_like(p).normal_(0.0, 1e-3, generator=ggen)
    mcfg = MuonConfig(lr=1e-3, beta=0.95, eps=1e-7, weight_decay=0.1, coeffs=COEFFS, nesterov=True,
                      ns_steps=args.ns_steps)
    acfg = AdamConfig(**cfg["adam"])
    opt = MuonAdamW(model, muon_config=mcfg, adam_config=acfg, parameter_split="auto", process_group=pg,
                    peer_push=args.push, reserve_sms=args.reserve_sms)
    push_mode = opt.distributed.backend.push if opt.distributed is not None else None   # "auto" resolved
    reserve_sms = opt.distributed.backend.reserve_sms if opt.distributed is not None else 0
    n_muon, n_adam = len(opt.muon.model_params), len(opt.adamw.model_params)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    step_params = [p for p in model.parameters() if p.grad is not None]
    grad_sets = None
    if args.realloc_grads:
        grad_sets = [[p.grad for p in step_params], [p.grad.clone() for p in step_params]]

    def timed_step(i):
        if grad_sets is not None:
            for p, g in zip(step_params, grad_sets[i % 2]):
                p.grad = g
        opt.step()

    for i in range(args.warmup):
        timed_step(i)
    barrier()

    clocks = ClockSampler(local_rank)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    start.record()
    for i in range(args.steps):
        timed_step(i)
    end.record()
    barrier()
    clock_info = clocks.stop()
    ms_local = start.elapsed_time(end) / args.steps
    ms = ms_local
    if world > 1:
        t = torch.tensor([ms_local], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    if grad_sets is not None:
        for p, g in zip(step_params, grad_sets[0]):
            p.grad = g
        grad_sets = None
    # Per-kernel timing: one more pass with CUDA events between every launch.
    timer = PhaseTimer()
    opt_branch_timer(opt, timer)
    timing_steps = max(1, min(args.steps, 3))
    barrier()
    for _ in range(timing_steps):
        opt.step()
    barrier()
    opt_branch_timer(opt, None)
    per = timer.durations()

    # Work accounting (this rank's share), per step.
    owned = owned_shapes(opt)
    flops = {"gram": 0.0, "poly": 0.0, "update": 0.0, "update_last": 0.0}
    elems_muon = 0
    for s in owned:
        f = ns_flops_sym(s)
        for k in flops:
            flops[k] += f["update" if k == "update_last" else k] * ns_phase_launches(k, args.ns_steps)
        elems_muon += math.prod(s)
    adam_elems = adam_elems_local(opt)
    hbm, tf_burst, tf_sus, peak_src = measured_peaks()
    kernels = {}

    def phase(label):
        d = per.get(label, [])
        return (sum(d) / timing_steps, len(d) / timing_steps) if d else (0.0, 0.0)

    for k in ("gram", "poly", "update", "update_last"):
        ms_k, n_k = phase(k)
        if n_k:
            tfl = flops[k] / (ms_k * 1e-3) / 1e12
            kernels[f"ns_gemm_{k}"] = {"launches_per_step": n_k, "ms_per_step": round(ms_k, 3),
                                       "avg_launch_ms": round(ms_k / n_k, 4), "tflops": round(tfl, 1),
                                       "frac_sustained": round(tfl / tf_sus, 3)}
    ms_a, n_a = phase("adamw")
    if n_a:
        gbs = 28.0 * adam_elems / (ms_a * 1e-3) / 1e9
        kernels["adamw_multi"] = {"launches_per_step": n_a, "ms_per_step": round(ms_a, 3), "gbs": round(gbs, 1),
                                  "frac": round(gbs / hbm, 3), "bytes_per_elem": 28}
    ms_p, n_p = phase("prep")
    if n_p:
        gbs = 14.0 * elems_muon / (ms_p * 1e-3) / 1e9
        kernels["muon_prep"] = {"launches_per_step": 2 * n_p, "includes": "muon_norm_kernel", "ms_per_step": round(ms_p, 3), "gbs": round(gbs, 1),
                                "frac": round(gbs / hbm, 3), "bytes_per_elem": 14}
    ns_ms = sum(phase(k)[0] for k in ("gram", "poly", "update", "update_last"))
    ns_total = sum(flops.values())
    upd = kernels.get("ns_gemm_update", {})
    traffic, traffic_how = ncu_traffic("ns_gemm_update", args.config)
    roofline = {"kernel": "ns_gemm_kernel<UPDATE> (tcgen05 B·X + a·X epilogue)", "bound": "tensor",
                "achieved": upd.get("tflops"), "peak": tf_sus, "unit": "TFLOP/s",
                "frac": upd.get("frac_sustained"), "peak_kind": f"{peak_src} sustained bf16",
                "traffic": traffic, "traffic_source": traffic_how, "ns_all_tflops": round(ns_total / (ns_ms * 1e-3) / 1e12, 1) if ns_ms else None,
                "ns_all_frac_sustained": round(ns_total / (ns_ms * 1e-3) / 1e12 / tf_sus, 3) if ns_ms else None,
                "ns_ms_per_step": round(ns_ms, 3), "ns_flops_per_step": ns_total}
    # Kernel launches per timed phase: the prep phase is the prep kernel plus the per-matrix norm kernel.
    kernels_per_phase = {"prep": 2}
    launches_per_step = sum(len(v) * kernels_per_phase.get(k, 1) for k, v in per.items()) / timing_steps

    # At N>1: one more (untimed) step, checked -- replicas bit-identical on every rank, and rank 0
    # recomputes matrices and AdamW tensors owned by other ranks with the single-GPU optimizer.
    parity = None
    if world > 1 and not args.no_verify:
        parity = verify_sharded_step(opt, rank, world, barrier)

    # End to end: this step's gradients from pinned host memory, result read back.
    e2e = run_e2e(opt, model, dev, args, barrier, world)

    grad_reduce = None
    if not args.no_grad_reduce and world > 1:
        opt.close()
        del opt
        grad_reduce = run_grad_reduce(model, mcfg, acfg, args, dev, pg, world, rank, barrier)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, sample, cores, detail = cpu_sample(args.config, cfg["adam"], args.ns_steps)
        cpu = {"value": round(v, 1), "unit": "ms/step", "cores": cores, "kind": "port", "sample": sample,
               "per_shape_ms": detail, "extrapolated": True}

    # The reference's own Triton MuonAdamW on this GPU, same config, in a child process once our
    # state is freed (both do not fit in HBM together at 8B).
    ref_triton = None
    if world == 1 and not args.no_reference_triton:
        import gc  # noqa: PLC0415
        opt_branch_timer(opt, None)
        del opt, model
        gc.collect()
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        ref_triton = run_reference_triton_child(args)

    if rank == 0:
        line = {
            "metric": f"MuonAdamW ms/step ({cfg['name']})", "value": round(ms, 3), "unit": "ms/step",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp32 params/grads/moments/momentum (elementwise fp32); Newton-Schulz bf16 (fp32 accumulate)",
            "data": "synthetic (seeded N(0,0.02) params, N(0,1e-3) grads; no dataset)",
            "config": {"workload": f"{cfg['name']} MuonAdamW optimizer step", "muon_matrices": n_muon,
                       "adamw_tensors": n_adam, "ns_steps": args.ns_steps, "coeffs": list(COEFFS),
                       "parallelism": "single-gpu" if world == 1 else f"muon-owner+zero1-adamw x{world}",
                       "param_push": push_mode, "realloc_grads": bool(args.realloc_grads),
                       "reserve_sms": reserve_sms,
                       "l2": "inputs (fp32 grads/params/momentum, > 100 GB) exceed L2; no flush needed",
                       "elementwise_dtype": "fp32"},
            "roofline": roofline, "kernels": kernels, "e2e": e2e, "gpu_launches": int(round(launches_per_step * args.steps)),
            "clocks": clock_info, "cpu_baseline": cpu,
        }
        if clock_info.get("sm_mhz"):
            # Under the 1 kW cap the sampled SM clock differs from box to box; time x clock
            # compares runs (and N) per clock cycle.
            line["ms_x_sm_ghz"] = round(ms * clock_info["sm_mhz"] / 1000.0, 1)
        if grad_reduce is not None:
            line["grad_reduce"] = grad_reduce
        if parity is not None:
            line["parity"] = parity["status"]
            line["parity_detail"] = parity
        if ref_triton is not None:
            line["reference_triton"] = ref_triton
            rv = ref_triton.get("value")
            if rv:
                line["vs_reference_triton"] = round(rv / ms, 3)
                ours_mhz, ref_mhz = clock_info.get("sm_mhz"), (ref_triton.get("clocks") or {}).get("sm_mhz")
                if ours_mhz and ref_mhz:
                    # cycles per step, ours vs the reference's: the ratio with each arm's own SM clock taken out
                    line["vs_reference_triton_per_clock"] = round(rv * ref_mhz / (ms * ours_mhz), 3)
        print(json.dumps(line), flush=True)
    if parity is not None and parity["status"] != "ok":
        if world > 1:
            dist.destroy_process_group()
        sys.exit(1)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def opt_branch_timer(opt, timer):
    target = opt.distributed if getattr(opt, "distributed", None) is not None else opt
    for br in (target.adamw, target.muon):
        br._timer = timer


def owned_shapes(opt):
    if getattr(opt, "distributed", None) is not None:
        return opt.distributed.owned_muon_shapes()
    return [tuple(p.shape) for p in opt.muon.model_params if p.grad is not None]


def adam_elems_local(opt):
    if getattr(opt, "distributed", None) is not None:
        return opt.distributed.adam_shard_numel()
    return sum(p.numel() for p in opt.adamw.model_params if p.grad is not None)


def ncu_traffic(kernel, config):
    """DRAM bytes per launch of `kernel` from the committed ncu summary (None if not captured)."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return None, None
    try:
        d = json.loads(p.read_text()).get(config, {}).get(kernel)
    except (ValueError, OSError):
        return None, None
    return (d["bytes_per_launch"], d["how"]) if d else (None, None)


def run_e2e(opt, model, dev, args, barrier, world):
    """The same step through the public API with this step's gradients in pinned host memory.

    ``MuonAdamW.step_from_host`` copies each gradient (only the pieces this
    rank reads) to the device on a side stream, overlapped with the previous
    buckets' work; the final-norm parameters are copied back.  All of it is
    inside the device-timed region.
    """
    params = [p for p in model.parameters() if p.grad is not None]
    flat = torch.empty(sum(p.numel() for p in params), dtype=torch.float32, pin_memory=True)
    host, off = {}, 0
    for p in params:
        host[p] = flat[off:off + p.numel()].view(p.shape)
        host[p].copy_(p.grad)
        off += p.numel()
    h2d = sum(g.numel() for g in e2e_grad_tensors(opt, model)) * 4
    probe = model.final_norm
    out = torch.empty(probe.numel(), dtype=torch.float32, pin_memory=True)
    steps = max(1, args.e2e_steps)
    opt.step_from_host(host)       # warm-up: bucket plans
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        opt.step_from_host(host)
        out.copy_(probe.detach(), non_blocking=True)
    end.record()
    barrier()
    ms = start.elapsed_time(end) / steps
    # What the host link gives one plain copy: 1 GiB of the same pinned buffer to the device,
    # on every rank at once (the ranks share the host's memory and PCIe switches).
    n = min(flat.numel(), (1 << 30) // 4)
    dst = torch.empty(n, dtype=torch.float32, device=dev)
    dst.copy_(flat[:n], non_blocking=True)
    barrier()
    start.record()
    for _ in range(3):
        dst.copy_(flat[:n], non_blocking=True)
    end.record()
    barrier()
    copy_gbs = 3 * n * 4 / (start.elapsed_time(end) * 1e-3) / 1e9
    del dst
    if world > 1:
        t = torch.tensor([ms, -copy_gbs], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, copy_gbs = float(t[0].item()), -float(t[1].item())
    return {"value": round(ms, 3), "unit": "ms/step", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(out.numel() * 4), "steps": steps,
            "h2d_gbs": round(h2d / (ms * 1e-3) / 1e9, 1),
            "h2d_copy_gbs": round(copy_gbs, 1),
            "h2d_bound_ms": round(h2d / (copy_gbs * 1e9) * 1e3, 1),
            "what": "MuonAdamW.step_from_host (grads H2D from pinned memory, overlapped) + final-norm D2H, "
                    "device-timed; h2d_gbs = this rank's gradient bytes / step time, h2d_copy_gbs = a plain "
                    "1 GiB pinned copy on every rank at once (slowest rank), h2d_bound_ms = the step's "
                    "gradient bytes at that rate"}


def run_grad_reduce(model, mcfg, acfg, args, dev, pg, world, rank, barrier):
    """Data-parallel gradients, different on every rank: the step with the reduction fused into its
    first kernels (reduce_grads="mean", peer reads over NVLink) vs an NCCL all-reduce of the same
    gradient bytes, which a data-parallel step without it needs first."""
    import gc  # noqa: PLC0415

    from triton_muon_adamw import MuonAdamW  # noqa: PLC0415
    for p in model.parameters():
        p.grad = None
    gc.collect()
    torch.cuda.empty_cache()
    opt = MuonAdamW(model, muon_config=mcfg, adam_config=acfg, parameter_split="auto", process_group=pg,
                    reduce_grads="mean", peer_push=args.push)
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    for p in model.parameters():
        p.grad.normal_(0.0, 1e-3, generator=gen)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            fn()
        end.record()
        barrier()
        t = torch.tensor([start.elapsed_time(end) / args.steps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    fused = timed(opt.step)
    # Per-kernel split of the fused step (events between launches) and the NVLink read rate of the
    # two kernels that sum the peers' copies.
    timer = PhaseTimer()
    opt_branch_timer(opt, timer)
    barrier()
    for _ in range(2):
        opt.step()
    barrier()
    opt_branch_timer(opt, None)
    phases = {k: sum(v) / 2 for k, v in timer.durations().items()}
    es = torch.empty((), dtype=opt.distributed.dtype).element_size()
    peer_bytes = {"adamw": adam_elems_local(opt) * (world - 1) * es,
                  "prep": sum(math.prod(sh) for sh in owned_shapes(opt)) * (world - 1) * es}
    peer = {k: {"ms_per_step": round(phases.get(k, 0.0), 3), "peer_bytes": int(b),
                "peer_read_gbs": round(b / (phases[k] * 1e-3) / 1e9, 1) if phases.get(k) else None}
            for k, b in peer_bytes.items()}
    arena = opt.distributed.arena.tensor
    grads = arena.view(opt.distributed.dtype)
    allreduce = timed(lambda: dist.all_reduce(grads, op=dist.ReduceOp.AVG, group=pg))
    opt.close()
    return {"fused_step_ms": round(fused, 3), "nccl_allreduce_ms": round(allreduce, 3),
            "gradient_bytes_per_rank": int(arena.numel()), "reduce_kernels": peer,
            "gemm_ms_per_step": round(sum(phases.get(k, 0.0) for k in ("gram", "poly", "update", "update_last")), 3),
            "what": "step with per-rank gradients summed inside the AdamW/Muon-prep kernels (peer loads over "
                    "NVLink) vs the NCCL all-reduce (AVG) of the same gradient bytes that a step on reduced "
                    "gradients needs first; compare fused_step_ms with nccl_allreduce_ms + value"}


@torch.no_grad()
def verify_sharded_step(opt, rank, world, barrier):
    """One more sharded step, checked (N>1; collective).

    * Replicas: a bit-exact checksum (int64 sum of each parameter's raw bits)
      of every parameter on every rank; all ranks must agree.
    * Recomputation: rank 0 snapshots up to three Muon matrices owned by other
      ranks (momentum sent by the owner) and two AdamW tensors (moments
      gathered from the ZeRO-1 shards), steps them with the single-GPU
      ``TritonMuon`` / ``TritonAdamW`` on the same gradients, and requires the
      result to equal its replica bit for bit: the sharded step is the
      single-GPU step, whatever rank owns a matrix or a range.
    """
    from triton_muon_adamw.adamw import TritonAdamW  # noqa: PLC0415
    from triton_muon_adamw.muon import TritonMuon  # noqa: PLC0415
    sh = opt.distributed
    mu, ad = sh.muon, sh.adamw
    # Muon matrices owned elsewhere, one per distinct shape, owners spread out.
    picks, seen = [], set()
    for i, s in enumerate(sh.slots):
        shape = tuple(mu.model_params[i].shape)
        if s.owner != 0 and shape not in seen and mu.model_params[i].grad is not None:
            picks.append(i)
            seen.add(shape)
        if len(picks) == 3:
            break
    snaps = []
    for i in picks:
        p, s = mu.model_params[i], sh.slots[i]
        mom = mu.momentum[p].clone() if s.owner == rank else torch.empty_like(p, dtype=sh.mom_segs[0].dtype)
        dist.broadcast(mom, src=s.owner, group=sh.pg)
        if rank == 0:
            snaps.append((i, p.detach().clone(), mom, p.grad.clone()))
        else:
            del mom
    adam_picks = [0, len(ad.model_params) - 1] if ad.model_params else []
    full_m = torch.empty(sh.adam_shard * world, dtype=torch.float32, device=sh.device)
    full_v = torch.empty_like(full_m)
    dist.all_gather_into_tensor(full_m, sh.exp_avg, group=sh.pg)
    dist.all_gather_into_tensor(full_v, sh.exp_avg_sq, group=sh.pg)
    adam_snaps = []
    if rank == 0:
        for i in adam_picks:
            p, o, n = ad.model_params[i], sh.adam_offsets[i], sh.adam_numels[i]
            adam_snaps.append((i, p.detach().clone(), full_m[o:o + n].view_as(p).clone(),
                               full_v[o:o + n].view_as(p).clone(), p.grad.clone()))
    del full_m, full_v
    step_before = ad.step_num
    barrier()
    opt.step()
    barrier()

    def bits(t):
        raw = t.detach().reshape(-1)
        raw = raw.view(torch.int32) if raw.element_size() == 4 else raw.view(torch.int16)
        return raw.to(torch.int64).sum()

    params = list(ad.model_params) + list(mu.model_params)
    sums = torch.stack([bits(p) for p in params])
    every = [torch.empty_like(sums) for _ in range(world)]
    dist.all_gather(every, sums, group=sh.pg)
    mismatched = [r for r in range(world) if not torch.equal(every[r], every[0])]
    out = {"replicas_identical": not mismatched, "ranks_checked": world, "params_checked": len(params),
           "muon_recomputed": [], "adamw_recomputed": []}
    problems = [f"replica of rank {r} differs from rank 0" for r in mismatched]
    if rank == 0:
        for i, p0, mom, g in snaps:
            p = mu.model_params[i]
            q = torch.nn.Parameter(p0)
            single = TritonMuon([q], lr=mu.lr, weight_decay=mu.weight_decay, coeffs=(mu.a, mu.b, mu.c),
                                nesterov=mu.is_nesterov, beta=mu.beta, ns_steps=mu.steps, eps=mu.eps,
                                adjust_lr_fn=mu.adjust_lr_fn)
            single.momentum[q].copy_(mom)
            q.grad = g
            single.step()
            ok = torch.equal(q.detach(), p.detach())
            out["muon_recomputed"].append({"index": i, "shape": list(p.shape), "owner": sh.slots[i].owner,
                                           "bit_equal": ok})
            if not ok:
                problems.append(f"Muon matrix {i} {tuple(p.shape)} (owner {sh.slots[i].owner}) differs")
        for i, p0, m, v, g in adam_snaps:
            p = ad.model_params[i]
            q = torch.nn.Parameter(p0)
            single = TritonAdamW([q], lr=ad.lr, betas=(ad.beta1, ad.beta2), weight_decay=ad.weight_decay, eps=ad.eps)
            single.m[q].copy_(m)
            single.v[q].copy_(v)
            single.step_num = step_before
            q.grad = g
            single.step()
            ok = torch.equal(q.detach(), p.detach())
            out["adamw_recomputed"].append({"index": i, "numel": p.numel(), "bit_equal": ok})
            if not ok:
                problems.append(f"AdamW tensor {i} ({p.numel()} elements) differs")
        torch.cuda.synchronize()
    status = "ok" if not problems else "FAIL: " + "; ".join(problems)
    flag = torch.tensor([0 if status == "ok" else 1], device=sh.device)
    dist.all_reduce(flag, group=sh.pg)
    out["status"] = "ok" if int(flag.item()) == 0 else (status if status != "ok" else "FAIL on another rank")
    return out


def run_reference_triton_child(args):
    """``bench.py --impl reference-triton`` as a child process; its JSON line (or why it is missing)."""
    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT")}
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference-triton", "--steps", str(args.steps),
           "--warmup", str(args.warmup), "--config", args.config, "--ns-steps", str(args.ns_steps)]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=1800)
    except subprocess.TimeoutExpired:
        return {"unavailable": "reference-triton child run exceeded 1800 s"}
    for line in reversed(r.stdout.strip().splitlines()):
        if line.startswith("{"):
            d = json.loads(line)
            keep = ("value", "unit", "steps", "warmup", "clocks", "unavailable", "config")
            return {k: d[k] for k in keep if k in d}
    return {"unavailable": f"reference-triton child exited {r.returncode}: {r.stderr.strip()[-300:]}"}


def e2e_grad_tensors(opt, model):
    if getattr(opt, "distributed", None) is not None:
        return opt.distributed.local_grad_tensors()
    return [p.grad for p in model.parameters() if p.grad is not None]


def c1_cpu_direct(steps=10):
    """The C1 config (17M GPT, tied embedding) through the reference wrapper's CPU path, timed directly."""
    from oracle.muon_adamw_oracle import ReferenceWrapperCPU, gpt_c1_shapes  # noqa: PLC0415
    adam_shapes, muon_shapes = gpt_c1_shapes()
    gen = torch.Generator().manual_seed(0)
    adam = [nn.Parameter(torch.randn(s, generator=gen) * 0.02) for s in adam_shapes]
    muon = [nn.Parameter(torch.randn(s, generator=gen) * 0.02) for s in muon_shapes]
    for p in adam + muon:
        p.grad = torch.randn(p.shape, generator=gen) * 1e-3
    w = ReferenceWrapperCPU(adam, muon, adam=dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-7, weight_decay=0.01),
                            muon=dict(lr=1e-3, beta=0.95, eps=1e-7, weight_decay=0.1, nesterov=True, ns_steps=5,
                                      adjust_lr_fn="original"))
    w.step()
    t0 = time.perf_counter()
    for _ in range(steps):
        w.step()
    return {"value": round((time.perf_counter() - t0) * 1e3 / steps, 2), "unit": "ms/step", "steps": steps,
            "params": sum(p.numel() for p in adam + muon),
            "what": "C1 (17M GPT, d=512, 4 layers, vocab 8192 tied) through the wrapper's CPU path, timed "
                    "directly, not extrapolated"}


def run_reference_arm(args, cfg, world):
    """The reference's CPU path on the host cores, bounded sample per step, extrapolated.

    Each of the K "steps" is one sampled round: one matrix per distinct Muon
    shape and one AdamW chunk, timed and scaled by the shape counts -- the
    8B step does not fit in host memory.  The line says so (``extrapolated``,
    ``sampled_rounds``) and adds C1 timed directly as a cross-check.
    """
    vals, sample, cores = [], "", 1
    for i in range(args.warmup + args.steps):
        v, sample, cores, _ = cpu_sample(args.config, cfg["adam"], args.ns_steps)
        if i >= args.warmup:
            vals.append(v)
    ms = statistics.mean(vals)
    line = {"metric": f"MuonAdamW ms/step ({cfg['name']})", "value": round(ms, 1), "unit": "ms/step",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 1),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp32 params/state; Newton-Schulz bf16 (torch CPU)", "data": "synthetic", "impl": "reference",
            "extrapolated": True, "sampled_rounds": args.steps,
            "config": {"workload": f"{cfg['name']} MuonAdamW optimizer step", "ns_steps": args.ns_steps,
                       "parallelism": "host cores"},
            "cpu_baseline": {"value": round(ms, 1), "unit": "ms/step", "cores": cores, "kind": "port",
                             "sample": sample, "extrapolated": True},
            "c1_direct": c1_cpu_direct(),
            "e2e": {"value": round(ms, 1), "unit": "ms/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_reference_triton_arm(args, cfg, world, local_rank):
    """The reference's own Triton MuonAdamW on this GPU: same shapes, data and hyperparameters as ours."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "triton_muon_adamw" / "optimizer.py").exists():
        print(json.dumps({"impl": "reference-triton", "unavailable": "baseline/_ref holds no reference install"}))
        return
    ours = (ROOT / "triton-muonadamw_b200").resolve()
    sys.path[:] = [p for p in sys.path if Path(p or ".").resolve() != ours]
    sys.path.insert(0, str(ref))
    import triton_muon_adamw as R  # noqa: PLC0415  (the reference package, not ours)
    assert Path(R.__file__).resolve().is_relative_to(ref.resolve()), R.__file__
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    adam_shapes, muon_shapes = cfg["shapes"]()
    model = ShapedParams(adam_shapes, muon_shapes, dev, seed=0)
    ggen = torch.Generator(device=dev).manual_seed(1)
    for p in model.parameters():
        p.grad = torch.empty_like(p).normal_(0.0, 1e-3, generator=ggen)
    opt = R.MuonAdamW(model, muon_config=R.MuonConfig(lr=1e-3, beta=0.95, eps=1e-7, weight_decay=0.1, coeffs=COEFFS,
                                                      nesterov=True, ns_steps=args.ns_steps),
                      adam_config=R.AdamConfig(**cfg["adam"]), parameter_split="auto")
    for _ in range(args.warmup):
        opt.step()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        opt.step()
    end.record()
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    ms = start.elapsed_time(end) / args.steps
    line = {"metric": f"MuonAdamW ms/step ({cfg['name']})", "value": round(ms, 3), "unit": "ms/step",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) params, N(0,1e-3) grads; no dataset)", "impl": "reference-triton",
            "config": {"workload": f"{cfg['name']} MuonAdamW optimizer step", "ns_steps": args.ns_steps,
                       "coeffs": list(COEFFS), "parallelism": "single-gpu",
                       "muon_matrices": len(opt.muon.model_params), "adamw_tensors": len(opt.adamw.model_params),
                       "source": "reference package, unmodified, from baseline/_ref"},
            "clocks": clock_info}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- isolated sweeps (C2, C3)
def _event_ms(fn, steps, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def run_adamw_sweep(args):
    """C2: the AdamW branch alone on flat float32 tensors of 1M, 16M, 64M and 256M elements and on 10,000
    ragged tensors of 1..65536 elements (seeded; ~3.3e8 elements), moments from 5 warm-up steps.

    Per case: our one-launch multi-tensor step (``TritonAdamW``), the reference's own ``TritonAdamW`` (one
    Triton launch per tensor, from baseline/_ref) and ``torch.optim.AdamW(fused=True)``, all on this GPU
    with CUDA events; GB/s = 28 B/element / time, against the measured HBM copy bandwidth.  Inputs of the
    large cases exceed L2; the 1M case fits in L2 (reported as is)."""
    import importlib.util  # noqa: PLC0415
    from triton_muon_adamw.adamw import TritonAdamW  # noqa: PLC0415
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hbm, _, _, peak_src = measured_peaks()
    ref_mod = None
    init = ROOT / "baseline" / "_ref" / "triton_muon_adamw" / "__init__.py"
    if init.exists():
        spec = importlib.util.spec_from_file_location("ref_triton_muon_adamw", init,
                                                      submodule_search_locations=[str(init.parent)])
        ref_mod = importlib.util.module_from_spec(spec)
        sys.modules["ref_triton_muon_adamw"] = ref_mod
        spec.loader.exec_module(ref_mod)
    hp = dict(lr=3e-4, betas=(0.9, 0.999), weight_decay=0.01, eps=1e-8)
    gen = torch.Generator(device=dev).manual_seed(0)
    cases = [("1M", [1 << 20]), ("16M", [1 << 24]), ("64M", [1 << 26]), ("256M", [1 << 28])]
    rg = torch.Generator().manual_seed(7)
    cases.append(("ragged_10k", torch.randint(1, 65537, (10000,), generator=rg).tolist()))
    if args.cases:
        cases = [c for c in cases if c[0] in args.cases.split(",")]
    out = []
    for name, sizes in cases:
        numel = sum(sizes)
        row = {"case": name, "tensors": len(sizes), "elements": numel, "bytes_per_step": 28 * numel}
        impls = [("ours", lambda ps: TritonAdamW(ps, **hp))]
        if ref_mod is not None:
            impls.append(("reference_triton", lambda ps: ref_mod.adamw.triton_adam.TritonAdamW(ps, **hp)))
        impls.append(("torch_fused", lambda ps: torch.optim.AdamW(ps, fused=True, **hp)))
        if args.impls:
            impls = [i for i in impls if i[0] in args.impls.split(",")]
        for impl, make in impls:
            # The reference launches grid (rows, cdiv(cols, 512)) per tensor (triton_adam.py:92-94), and a 1-D
            # tensor is one row: beyond 65535 * 512 elements grid.y exceeds the CUDA limit and the launch fails.
            # It runs those cases on the same elements viewed as rows of 4096 (the update is elementwise).
            as_rows = impl == "reference_triton" and max(sizes) > 65535 * 512
            if as_rows:
                row["reference_triton_layout"] = "rows of 4096 (a flat tensor this long exceeds its grid limit)"
            params = [nn.Parameter(torch.empty((n // 4096, 4096) if as_rows and n % 4096 == 0 else (n,), device=dev)
                                   .normal_(0, 0.02, generator=gen)) for n in sizes]
            for q in params:
                q.grad = torch.empty_like(q).normal_(0, 1e-2, generator=gen)
            opt = make(params)
            for _ in range(5):                       # moments from 5 warm-up steps
                opt.step()
            ms = _event_ms(opt.step, max(3, args.steps), 2)
            gbs = 28.0 * numel / (ms * 1e-3) / 1e9
            row[impl] = {"ms": round(ms, 4), "gbs": round(gbs, 1), "frac_hbm": round(gbs / hbm, 3)}
            del opt, params
            torch.cuda.empty_cache()
        if "reference_triton" in row and "ours" in row:
            row["speedup_vs_reference_triton"] = round(row["reference_triton"]["ms"] / row["ours"]["ms"], 2)
        if "torch_fused" in row and "ours" in row:
            row["speedup_vs_torch_fused"] = round(row["torch_fused"]["ms"] / row["ours"]["ms"], 2)
        out.append(row)
        print(json.dumps(row), file=sys.stderr, flush=True)
    big = next((r for r in out if r["case"] == "256M" and "ours" in r), None) or next(r for r in out if "ours" in r)
    print(json.dumps({"metric": f"AdamW HBM GB/s (C2 sweep; value: {big['case']} case)", "value": big["ours"]["gbs"],
                      "unit": "GB/s", "higher_is_better": True, "n_gpus": 1, "steps": max(3, args.steps),
                      "dtype": "fp32", "data": "synthetic (seeded; params N(0,0.02), grads N(0,1e-2))",
                      "peak": hbm, "peak_kind": f"{peak_src} HBM copy", "config": {"workload": "C2 AdamW sweep"},
                      "cases": out}), flush=True)


def run_ns_sweep(args):
    """C3: Newton-Schulz in isolation -- bf16-valued N(0,1) matrices of 1024x1024, 4096x4096, 4096x14336 and
    14336x4096 (tall: transposed), batches of 1, 8 and 32 in one plan, ns_steps 5 and 6.

    One ``TritonMuon`` step per timed iteration (beta=0, no Nesterov: X is the gradient itself), its
    launches timed with CUDA events on the launching stream; TFLOP/s over the Gram, polynomial and update
    GEMMs = (3m^2n + m^3 per iteration, triangles counted once) / their time, against the measured
    sustained bf16 peak; the dense-equivalent 4m^2n + 2m^3 rate is reported beside it."""
    from triton_muon_adamw.muon import TritonMuon  # noqa: PLC0415
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _, tf_burst, tf_sus, peak_src = measured_peaks()
    gen = torch.Generator(device=dev).manual_seed(0)
    out = []
    wanted = set(args.cases.split(",")) if args.cases else None
    for shape in [(1024, 1024), (4096, 4096), (4096, 14336), (14336, 4096)]:
        for batch in (1, 8, 32):
            if wanted is not None and f"{shape[0]}x{shape[1]}x{batch}" not in wanted:
                continue
            for ns in (5, 6):
                params = []
                for _ in range(batch):
                    q = nn.Parameter(torch.zeros(shape, device=dev))
                    q.grad = torch.empty(shape, device=dev).normal_(0, 1, generator=gen).bfloat16().float()
                    params.append(q)
                opt = TritonMuon(params, lr=1e-3, weight_decay=0.0, coeffs=COEFFS, nesterov=False, beta=0.0,
                                 ns_steps=ns, eps=1e-7)
                for _ in range(2):
                    opt.step()
                timer = PhaseTimer()
                opt._timer = timer
                steps = max(2, min(args.steps, 5))
                torch.cuda.synchronize()
                for _ in range(steps):
                    opt.step()
                torch.cuda.synchronize()
                opt._timer = None
                per = timer.durations()
                ns_ms = sum(sum(per.get(k, [])) for k in ("gram", "poly", "update", "update_last")) / steps
                prep_ms = sum(per.get("prep", [])) / steps
                m, n = min(shape), max(shape)
                sym = batch * ns * (3.0 * m * m * n + float(m) ** 3)
                dense = batch * ns * (4.0 * m * m * n + 2.0 * float(m) ** 3)
                tf = sym / (ns_ms * 1e-3) / 1e12
                row = {"shape": list(shape), "batch": batch, "ns_steps": ns, "ns_ms": round(ns_ms, 3),
                       "prep_ms": round(prep_ms, 3), "tflops": round(tf, 1),
                       "frac_sustained": round(tf / tf_sus, 3), "frac_burst": round(tf / tf_burst, 3),
                       "dense_equiv_tflops": round(dense / (ns_ms * 1e-3) / 1e12, 1)}
                st = opt.device_status()
                if st:
                    row["device_status"] = st
                out.append(row)
                print(json.dumps(row), file=sys.stderr, flush=True)
                del opt, params
                torch.cuda.empty_cache()
    best = max(out, key=lambda r: r["tflops"])
    head = next((r for r in out if r["shape"] == [4096, 14336] and r["batch"] == 32 and r["ns_steps"] == 5), best)
    print(json.dumps({"metric": f"Newton-Schulz TFLOP/s (C3; value: {head['batch']} x {head['shape'][0]}x"
                                f"{head['shape'][1]}, ns {head['ns_steps']})", "value": head["tflops"],
                      "unit": "TFLOP/s", "higher_is_better": True, "n_gpus": 1, "dtype": "bf16 (fp32 accumulate)",
                      "data": "synthetic (bf16-valued N(0,1) matrices, seeded)", "peak_sustained": tf_sus,
                      "peak_burst": tf_burst, "peak_kind": f"{peak_src} bf16", "best_case": best,
                      "config": {"workload": "C3 Newton-Schulz isolated"}, "cases": out}), flush=True)


SWEEPS = {"adamw_sweep": run_adamw_sweep, "ns_isolated": run_ns_sweep}


if __name__ == "__main__":
    main()
