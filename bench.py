#!/usr/bin/env python
"""Benchmark of the NVFP4 dual GEMM  C = silu(A B1^T) * (A B2^T).

One step = one dual-GEMM call on one batch of seeded synthetic NVFP4 input
(randn -> e2m1 codes + e4m3 per-16 scales).  Default workload: BASELINE
config 2, the decode shape M=256, N=4096, K=7168.  Prints ONE JSON line on
rank 0.

Timed region: the K steps are captured once in a CUDA graph and replayed
between two CUDA events (barrier + synchronize on both sides); inputs rotate
over enough independent sets that the data touched between two uses of a set
exceeds the 126 MB L2, so every call streams its operands from HBM.

Multi-GPU (torchrun, one process per GPU): for the c2/c3/c4 workloads every
rank owns its own N-slice of a wider problem of the same per-rank shape (A
replicated, no collective: weak scaling); for c5 the fixed N = 28672 is split
over the ranks (strong scaling).  Time = max over ranks.

  --impl reference  times the reference's own implementation on the same
                    workload: its kernel compiled from its sources
                    (oracle/_ref, shapes of its dispatch table), else the CPU
                    port of its algorithm in oracle/.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

WORKLOADS = {
    "c2": dict(M=256, N=4096, K=7168, a=1.0, w=1.0,
               name="C2 decode 256x4096x7168 (BASELINE configs[1])"),
    "c3": dict(M=512, N=3072, K=7168, a=1.0, w=1.0,
               name="C3 mid 512x3072x7168 (BASELINE configs[2])"),
    "c4": dict(M=4096, N=14336, K=4096, a=0.5, w=0.02,
               name="C4 prefill 4096x14336x4096 (BASELINE configs[3])"),
    "c5": dict(M=8192, N=28672, K=8192, a=0.5, w=0.02, strong=True,
               name="C5 N-sharded 8192x28672x8192 (BASELINE configs[4])"),
}
METRIC = ("dual-GEMM µs & effective TFLOPS (% of FP4/HBM roofline), "
          "geomean over shapes")
L2_BYTES = 126 * 2 ** 20


def algo_bytes(m, n, k):
    """A + B1 + B2 codes, their e4m3 scales and the fp16 C."""
    return m * k // 2 + n * k + m * k // 16 + 2 * (n * k // 16) + 2 * m * n


def algo_flops(m, n, k):
    return 4.0 * m * n * k


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return {"hbm_gbs": float(pk["hbm_gbs"]),
                "bf16_tflops": float(pk["bf16_tflops"]),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def load_traffic(workload):
    """DRAM bytes per launch from a committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", "dram_traffic.json")
    try:
        with open(path) as f:
            v = json.load(f).get(workload)
        return None if v is None else float(v)
    except Exception:
        return None


class ClockSampler:
    """Polls NVML (SM clock, throttle reasons) from a thread while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting",
        0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x10: "sync_boost",
        0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index, period_s=0.002):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._period = period_s
        self._h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(
                self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._h = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _sample(self):
        nv = self._nv
        self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
        self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(self._period)

    def __enter__(self):
        if self._h is not None:
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._h is not None:
            self._t.join()
            try:
                self._sample()
            except Exception:
                pass

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [],
                    "samples": 0}
        names = [v for k, v in self.REASONS.items()
                 if self.reasons & k and v != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


# --------------------------------------------------------------------------
# distributed plumbing
# --------------------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    from nvfp4_dual_gemm_b200.shard import max_over_ranks as _max
    return _max(x, device="cuda")


# --------------------------------------------------------------------------
# inputs
# --------------------------------------------------------------------------
def rank_problem(wl, world, rank):
    m, n, k = wl["M"], wl["N"], wl["K"]
    if wl.get("strong"):
        if n % (64 * world):
            raise SystemExit(f"N={n} does not split into {world} x 64")
        n = n // world
    return m, n, k


def make_sets(dg, m, n, k, wl, rank, min_sets=2):
    per = algo_bytes(m, n, k)
    nsets = max(min_sets, math.ceil(2 * L2_BYTES / per))
    sets = [dg.generate_input(m, n, k, seed=1000 * rank + s, a_scale=wl["a"],
                              w_scale=wl["w"]) for s in range(nsets)]
    torch.cuda.synchronize()
    return sets, nsets


def time_graph(step_fn, steps, warmup, world):
    """Warm up eagerly, capture `steps` calls in one CUDA graph, replay it in
    the timed region.  Returns (ms, clock summary)."""
    for i in range(warmup):
        step_fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for i in range(steps):
                step_fn(i)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()  # one untimed replay: first-replay setup is not part of a step
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    dev = torch.cuda.current_device()
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(dev) as clk:
        start.record()
        g.replay()
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = start.elapsed_time(end)
    del g
    return ms, clk.summary()


def time_eager(step_fn, steps, warmup, world):
    """Warm up, then time `steps` back-to-back eager calls between two events
    on the current (default) stream.  Used for implementations whose launches
    cannot be captured in a CUDA graph."""
    for i in range(warmup):
        step_fn(i)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(torch.cuda.current_device()) as clk:
        start.record()
        for i in range(steps):
            step_fn(i)
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    return start.elapsed_time(end), clk.summary()


def copy_call_copy(call, host_inputs, dev_inputs, c_dev, c_host):
    """One end-to-end step through a device-buffer API: pinned H2D of the
    inputs, the call, D2H of C, one after another on the current stream."""
    def one():
        for h, d in zip(host_inputs, dev_inputs):
            d.copy_(h, non_blocking=True)
        call()
        c_host.copy_(c_dev, non_blocking=True)
    return one


def time_e2e(one, host_inputs, c_host, steps, world):
    """Events around `steps` end-to-end steps (each uploads its inputs from
    pinned host memory and downloads C); returns (ms, H2D and D2H bytes per
    step)."""
    stream = torch.cuda.current_stream()
    h2d = sum(t.numel() * t.element_size() for t in host_inputs)
    d2h = c_host.numel() * c_host.element_size()
    one()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(steps):
        one()
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return start.elapsed_time(end), h2d, d2h


def cpu_baseline(host_a, host_sfa, host_b1, host_sfb1, host_b2, host_sfb2,
                 m, n, k, budget_s=20.0):
    """The oracle (CPU restatement of the path) on a bounded row sample,
    with all host threads for the matmuls."""
    from threadpoolctl import threadpool_info, threadpool_limits

    from oracle import nvfp4_oracle as O

    cores = os.cpu_count() or 1
    with threadpool_limits(limits=cores):
        threads = max([d.get("num_threads", 1) for d in threadpool_info()] or [1])
        rows = min(m, 32)
        t0 = time.perf_counter()
        O.dual_gemm(host_a[:rows], host_sfa[:rows], host_b1, host_sfb1,
                    host_b2, host_sfb2)
        dt = time.perf_counter() - t0
        reps = 1
        while time.perf_counter() - t0 + dt < min(budget_s, 10 * dt) and reps < 5:
            O.dual_gemm(host_a[:rows], host_sfa[:rows], host_b1, host_sfb1,
                        host_b2, host_sfb2)
            reps += 1
        total = time.perf_counter() - t0
    per_call = total / reps
    flops = algo_flops(rows, n, k)
    return {"value": flops / per_call / 1e12, "unit": "TFLOP/s",
            "cores": threads, "kind": "port",
            "sample": f"{rows} of {m} rows of A against all {n} rows of "
                      f"B1/B2 (dequantise + fp32 matmul + SiLU), {reps} reps",
            "us_per_call_full_shape_est": per_call * (m / rows) * 1e6}


# --------------------------------------------------------------------------
# arms
# --------------------------------------------------------------------------
def run_ours(args, world, rank):
    import nvfp4_dual_gemm_b200 as dg

    wl = WORKLOADS[args.workload]
    m, n, k = rank_problem(wl, world, rank)
    sets, nsets = make_sets(dg, m, n, k, wl, rank)
    # The timed calls never write the weights (inputs rotate over sets made
    # before timing), so they may be read before the dependency wait.
    from nvfp4_dual_gemm_b200 import _lib
    flags = args.flags | (0 if args.no_static_weights
                          else _lib.FLAG_STATIC_WEIGHTS)
    ws_bytes = dg.workspace_size(m, n, k, flags)
    ws = torch.zeros(max(ws_bytes, 256), dtype=torch.uint8, device="cuda")

    def step(i):
        d = sets[i % nsets]
        dg.dual_gemm(d[0], d[1], d[2], d[6], d[7], d[8], d[9], flags=flags,
                     workspace=ws)

    ms, clocks = time_graph(step, args.steps, args.warmup, world)
    ms = max_over_ranks(ms, world)
    ranks_flops = algo_flops(m, n, k) * world
    us_call = ms * 1e3 / args.steps
    tflops = ranks_flops * args.steps / (ms * 1e-3) / 1e12
    peaks = load_peaks()
    byts = algo_bytes(m, n, k)
    fp4_peak = 4.0 * peaks["bf16_tflops"]
    t_hbm = byts / (peaks["hbm_gbs"] * 1e9)
    t_tc = algo_flops(m, n, k) / (fp4_peak * 1e12)
    if t_hbm >= t_tc:
        ach = byts / (us_call * 1e-6) / 1e9
        roof = {"bound": "hbm", "achieved": round(ach, 1),
                "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(ach / peaks["hbm_gbs"], 4)}
    else:
        ach = algo_flops(m, n, k) / (us_call * 1e-6) / 1e12
        roof = {"bound": "tensor", "achieved": round(ach, 1),
                "peak": fp4_peak, "unit": "TFLOP/s",
                "frac": round(ach / fp4_peak, 4)}
    roof["traffic"] = load_traffic(args.workload)
    roof["algorithmic_bytes"] = byts
    roof["algorithmic_flops"] = algo_flops(m, n, k)
    roof["peak_source"] = (
        f"{peaks['source']} HBM copy GB/s; FP4 dense = 4 x {peaks['source']} "
        "bf16 cuBLAS TF/s")

    # end to end through the public host-buffer API: pinned host inputs and
    # output, the library uploads, computes and downloads (slab-pipelined)
    d = sets[0]
    dev_in = [d[0], d[1], d[2], d[6], d[7], d[8]]
    host_in = [t.cpu().view(torch.uint8).pin_memory() for t in dev_in]
    c_host = torch.empty(d[9].shape[:2], dtype=torch.float16).pin_memory()
    e2e_steps = max(1, min(args.steps, args.e2e_steps))

    def e2e_step():
        dg.dual_gemm_host(*host_in, c_host, flags=args.flags)

    e2e_ms, h2d, d2h = time_e2e(e2e_step, host_in, c_host, e2e_steps, world)
    e2e_ms = max_over_ranks(e2e_ms, world)
    e2e_val = ranks_flops * e2e_steps / (e2e_ms * 1e-3) / 1e12

    line = {
        "metric": METRIC, "value": round(tflops, 3), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "us_per_call": round(us_call, 3),
        "higher_is_better": True,
        "scaling": "strong" if wl.get("strong") else "weak",
        "vs_baseline": None,
        "dtype": "nvfp4 (e2m1 x e4m3/16, fp32 accumulate, fp16 out)",
        "data": "synthetic: seeded randn -> NVFP4 on the GPU",
        "config": {"workload": wl["name"], "M": m, "N_per_rank": n, "K": k,
                   "L": 1, "parallelism": f"N-sharded x{world}" if world > 1
                   else "single GPU", "plan": dg.plan(m, n, k, flags),
                   "l2": f"{nsets} rotating input sets of "
                         f"{algo_bytes(m, n, k) / 1e6:.1f} MB "
                         f"(> 2 x 126 MB L2 between reuses)",
                   "timed": "one CUDA graph of `steps` calls, replayed once",
                   "flags": (f"{flags:#x}" + (
                       " (STATIC_WEIGHTS: the weights, constant across the "
                       "timed calls, are copied before the dependency wait)"
                       if flags & _lib.FLAG_STATIC_WEIGHTS else ""))},
        "roofline": roof,
        "e2e": {"value": round(e2e_val, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps,
                "api": "nvfp4_dual_gemm_b200.dual_gemm_host "
                       "(C ABI nvfp4_dual_gemm_run_host)"},
        "gpu_launches": args.steps,
        "clocks": clocks,
    }
    if args.shapes and world == 1:
        line["shapes"] = shape_sweep(dg, args, flags)
        vals = [s["tflops"] for s in line["shapes"]]
        line["geomean_tflops"] = round(math.exp(sum(map(math.log, vals)) /
                                                len(vals)), 3)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        hd = [t.view(torch.uint8).squeeze(-1).cpu().numpy() for t in
              (d[0], d[3], d[1], d[4], d[2], d[5])]
        line["cpu_baseline"] = cpu_baseline(*hd, m, n, k)
    del sets
    return line


def shape_sweep(dg, args, flags=0):
    out = []
    peaks = load_peaks()
    for key in ("c2", "c3", "c4"):
        wl = WORKLOADS[key]
        m, n, k = wl["M"], wl["N"], wl["K"]
        sets, nsets = make_sets(dg, m, n, k, wl, 0)
        ws = torch.zeros(max(dg.workspace_size(m, n, k, flags), 256),
                         dtype=torch.uint8, device="cuda")
        steps = max(10, min(args.steps, 200))

        def step(i):
            d = sets[i % nsets]
            dg.dual_gemm(d[0], d[1], d[2], d[6], d[7], d[8], d[9],
                         workspace=ws, flags=flags)

        ms, _ = time_graph(step, steps, 3, 1)
        us = ms * 1e3 / steps
        t_roof = max(algo_bytes(m, n, k) / (peaks["hbm_gbs"] * 1e3),
                     algo_flops(m, n, k) / (4 * peaks["bf16_tflops"] * 1e6))
        out.append({"workload": key, "us": round(us, 3),
                    "tflops": round(algo_flops(m, n, k) / us / 1e6, 2),
                    "roofline_frac": round(t_roof / us, 4)})
        del sets, ws
        torch.cuda.empty_cache()
    return out


def run_reference(args, world, rank):
    """The reference's own implementation on the same workload."""
    wl = WORKLOADS[args.workload]
    m, n, k = rank_problem(wl, 1, 0)
    import nvfp4_dual_gemm_b200 as dg  # input generation only
    from oracle import build_ref

    mod = build_ref.load()
    line = {"metric": METRIC, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "impl": "reference",
            "scaling": "strong" if wl.get("strong") else "weak",
            "vs_baseline": None,
            "dtype": "nvfp4 (e2m1 x e4m3/16, fp32 accumulate, fp16 out)",
            "data": "synthetic: seeded randn -> NVFP4 on the GPU",
            "config": {"workload": wl["name"], "M": m, "N_per_rank": n, "K": k,
                       "L": 1, "parallelism": "rank 0 only"}}
    sets, nsets = make_sets(dg, m, n, k, wl, 0)
    d0 = sets[0]
    hd = [t.view(torch.uint8).squeeze(-1).cpu().numpy() for t in
          (d0[0], d0[3], d0[1], d0[4], d0[2], d0[5])]
    cpu = None if args.no_cpu_baseline else cpu_baseline(*hd, m, n, k)
    if mod is not None and (m, n, k) in build_ref.SAFE_SHAPES:
        def step(i):
            d = sets[i % nsets]
            mod.cuda_nvfp4_dual_gemm(d[0], d[1], d[2], d[6], d[7], d[8], d[9])

        # The reference launches on the legacy default stream
        # (nvfp4_dual_gemm.cu:368-372), which no CUDA graph can capture, so
        # its steps are timed as back-to-back eager calls.
        ms, clocks = time_eager(step, args.steps, args.warmup, 1)
        tflops = algo_flops(m, n, k) * args.steps / (ms * 1e-3) / 1e12
        dev_in = [d0[0], d0[1], d0[2], d0[6], d0[7], d0[8]]
        host_in = [t.cpu().pin_memory() for t in dev_in]
        c_host = torch.empty(d0[9].shape, dtype=torch.float16).pin_memory()
        e2e_steps = max(1, min(args.steps, args.e2e_steps))
        e2e_ms, h2d, d2h = time_e2e(
            copy_call_copy(
                lambda: mod.cuda_nvfp4_dual_gemm(d0[0], d0[1], d0[2], d0[6],
                                                 d0[7], d0[8], d0[9]),
                host_in, dev_in, d0[9], c_host),
            host_in, c_host, e2e_steps, 1)
        line.update({
            "value": round(tflops, 3), "ms_per_step": ms / args.steps,
            "us_per_call": round(ms * 1e3 / args.steps, 3),
            "reference_kind": "the reference's CUDA kernel, compiled from its "
                              "sources by oracle/build_ref.py, called through "
                              "its cuda_nvfp4_dual_gemm entry",
            "timed": "back-to-back eager calls (legacy default stream, "
                     "not capturable in a CUDA graph)",
            "e2e": {"value": round(algo_flops(m, n, k) * e2e_steps /
                                   (e2e_ms * 1e-3) / 1e12, 3),
                    "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps},
            "clocks": clocks, "cpu_baseline": cpu})
    else:
        why = ("oracle/_ref not built" if mod is None else
               "shape outside the reference kernel's dispatch table")
        if cpu is None:
            cpu = cpu_baseline(*hd, m, n, k)
        line.update({
            "value": cpu["value"], "ms_per_step": None,
            "reference_kind": f"CPU port of the reference algorithm ({why})",
            "cpu_baseline": cpu,
            "e2e": {"value": cpu["value"], "unit": "TFLOP/s",
                    "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    return line


PLUMBING = {
    "quantize": dict(rows=8192, K=7168, dtype="bfloat16",
                     name="activation quantiser: 8192 x 7168 bf16 rows -> "
                          "NVFP4 codes + blocked scales"),
    "scales": dict(rows=14336, K=7168,
                   name="scale layout converter: plain -> blocked, "
                        "14336 x 448 scales"),
    "batched": dict(rows=256, K=7168, N=4096, L=8,
                    name="batched dual GEMM, L = 8 problems of C2's shape "
                         "(256x4096x7168) in one launch vs 8 launches"),
    "grouped": dict(rows=[512, 300, 128, 64, 40, 8, 0, 200], K=7168,
                    N=2048,
                    name="grouped dual GEMM (MoE FFN): 8 experts, N = 2048, "
                         "K = 7168, 1252 tokens in skewed groups, one launch "
                         "vs one launch per expert"),
    "nvfp4_out": dict(rows=256, K=7168, N=4096,
                      name="dual GEMM with NVFP4 output (C2 256x4096x7168): "
                           "fused quantising epilogue vs fp16 C + quantiser"),
}


def run_plumbing(args):
    """Time one of the kernels beside the dual GEMM (SURVEY-style 'next'
    rows): the activation quantiser or the scale layout converter, in a
    CUDA graph over rotating buffers larger than 2 x L2; one JSON line with
    GB/s against the measured HBM copy bandwidth."""
    import nvfp4_dual_gemm_b200 as dg
    from nvfp4_dual_gemm_b200 import _lib

    torch.cuda.set_device(0)
    cfg = PLUMBING[args.plumbing]
    rows, k = cfg["rows"], cfg["K"]
    lib = _lib.load()
    stream = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731
    if args.plumbing == "nvfp4_out":
        return run_nvfp4_out(args, cfg)
    if args.plumbing == "batched":
        return run_batched(args, cfg)
    if args.plumbing == "grouped":
        return run_grouped(args, cfg)
    blocked = ((rows + 127) // 128) * (k // 64) * 512
    if args.plumbing == "quantize":
        dt = getattr(torch, cfg["dtype"])
        per = rows * k * 2 + rows * k // 2 + blocked
        nsets = max(2, -(-2 * L2_BYTES // per))
        xs = [torch.randn((rows, k), device="cuda").to(dt) for _ in range(nsets)]
        codes = [torch.empty((rows, k // 2), dtype=torch.uint8, device="cuda")
                 for _ in range(nsets)]
        blks = [torch.empty((blocked,), dtype=torch.uint8, device="cuda")
                for _ in range(nsets)]

        def step(i):
            j = i % nsets
            rc = lib.nvfp4_quantize_rows(
                xs[j].data_ptr(), _lib.DTYPE_BF16, rows, k, k,
                codes[j].data_ptr(), None, blks[j].data_ptr(), stream())
            assert rc == 0, _lib.last_error()
    else:
        per = rows * (k // 16) + blocked
        nsets = max(2, -(-2 * L2_BYTES // per))
        sfs = [torch.randint(0, 256, (rows, k // 16), dtype=torch.uint8,
                             device="cuda") for _ in range(nsets)]
        blks = [torch.empty((blocked,), dtype=torch.uint8, device="cuda")
                for _ in range(nsets)]

        def step(i):
            j = i % nsets
            rc = lib.nvfp4_scales_to_blocked(sfs[j].data_ptr(), rows, k,
                                             k // 16, blks[j].data_ptr(),
                                             stream())
            assert rc == 0, _lib.last_error()
    ms, clocks = time_graph(step, args.steps, args.warmup, 1)
    us = ms * 1e3 / args.steps
    gbs = per / (us * 1e-6) / 1e9
    peaks = load_peaks()
    return {
        "metric": cfg["name"], "value": round(gbs, 1), "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "us_per_call": round(us, 3),
        "higher_is_better": True, "data": "synthetic",
        "config": {"workload": args.plumbing, "rows": rows, "K": k,
                   "bytes_per_call": per,
                   "l2": f"{nsets} rotating buffer sets (> 2 x 126 MB L2)",
                   "timed": "one CUDA graph of `steps` calls, replayed once"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(gbs / peaks["hbm_gbs"], 4),
                     "peak_source": f"{peaks['source']} HBM copy GB/s"},
        "gpu_launches": args.steps, "clocks": clocks,
    }


def run_batched(args, cfg):
    """L problems of one shape (a batch, e.g. the experts of an MoE layer
    with equal token counts) in one launch, against L back-to-back launches
    of the unbatched problems on the same buffers; both graph-timed over
    rotating input sets larger than 2 x L2."""
    import nvfp4_dual_gemm_b200 as dg

    m, n, k, L = cfg["rows"], cfg["N"], cfg["K"], cfg["L"]
    per = L * algo_bytes(m, n, k)
    nsets = max(2, math.ceil(2 * L2_BYTES / per))
    sets = [dg.generate_input(m, n, k, l=L, seed=s) for s in range(nsets)]
    torch.cuda.synchronize()
    blk_a = ((m + 127) // 128) * (k // 64) * 512
    blk_b = ((n + 127) // 128) * (k // 64) * 512
    ws = torch.zeros(max(dg.workspace_size(m, n, k, L=L),
                         dg.workspace_size(m, n, k), 256),
                     dtype=torch.uint8, device="cuda")

    def one_launch(i):
        d = sets[i % nsets]
        dg.dual_gemm(d[0], d[1], d[2], d[6], d[7], d[8], d[9], workspace=ws)

    def per_batch(i):
        d = sets[i % nsets]
        for b in range(L):
            dg.dual_gemm(d[0][..., b], d[1][..., b], d[2][..., b],
                         d[6][b * blk_a:(b + 1) * blk_a],
                         d[7][b * blk_b:(b + 1) * blk_b],
                         d[8][b * blk_b:(b + 1) * blk_b], d[9][..., b],
                         workspace=ws)

    ms_1, clocks = time_graph(one_launch, args.steps, args.warmup, 1)
    ms_l, _ = time_graph(per_batch, args.steps, args.warmup, 1)
    us_1 = ms_1 * 1e3 / args.steps
    us_l = ms_l * 1e3 / args.steps
    flops = L * algo_flops(m, n, k)
    peaks = load_peaks()
    gbs = per / (us_1 * 1e-6) / 1e9
    return {
        "metric": cfg["name"], "value": round(flops / (us_1 * 1e-6) / 1e12, 3),
        "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_1 / args.steps,
        "us_per_call": round(us_1, 3),
        "separate_launches_us_per_call": round(us_l, 3),
        "higher_is_better": True, "data": "synthetic: seeded randn -> NVFP4",
        "config": {"workload": "batched", "M": m, "N": n, "K": k, "L": L,
                   "l2": f"{nsets} rotating input sets (> 2 x 126 MB L2)",
                   "timed": "one CUDA graph of `steps` calls, replayed once"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(gbs / peaks["hbm_gbs"], 4),
                     "algorithmic_bytes": per,
                     "peak_source": f"{peaks['source']} HBM copy GB/s"},
        "gpu_launches": args.steps, "clocks": clocks,
    }


def run_grouped(args, cfg):
    """Experts with their own token counts in one launch
    (``dual_gemm_grouped``) against one launch per non-empty expert on the
    same buffers; both graph-timed over rotating input sets > 2 x L2."""
    import nvfp4_dual_gemm_b200 as dg

    rows, n, k = cfg["rows"], cfg["N"], cfg["K"]
    G = len(rows)
    row0 = dg.group_offsets(rows)
    R = max(r + m for r, m in zip(row0, rows) if m)
    blk_a = ((R + 127) // 128) * (k // 64) * 512
    blk_b = ((n + 127) // 128) * (k // 64) * 512
    per = R * k // 2 + blk_a + G * (n * k + 2 * blk_b) + 2 * R * n
    nsets = max(2, math.ceil(2 * L2_BYTES / per))
    sets = []
    for s_ in range(nsets):
        a = dg.generate_input(R, n, k, l=1, seed=100 + s_)  # A rows, SFA
        w = dg.generate_input(128, n, k, l=G, seed=200 + s_)  # experts
        sets.append((a[0].squeeze(-1), w[1], w[2], a[6], w[7], w[8],
                     torch.empty((R, n), dtype=torch.float16, device="cuda")))
    torch.cuda.synchronize()
    ws = torch.zeros(1 << 24, dtype=torch.uint8, device="cuda")
    # one problem per expert: slices of the same buffers
    def per_expert(i):
        d = sets[i % nsets]
        for g in range(G):
            if rows[g] == 0:
                continue
            rs = slice(row0[g], row0[g] + rows[g])
            dg.dual_gemm(d[0][rs], d[1][..., g], d[2][..., g],
                         d[3][(row0[g] // 128) * (k // 64) * 512:],
                         d[4][g * blk_b:(g + 1) * blk_b],
                         d[5][g * blk_b:(g + 1) * blk_b], d[6][rs],
                         workspace=ws)

    wsg = torch.zeros(max(dg.grouped_workspace_size(rows, n, k), 256),
                      dtype=torch.uint8, device="cuda")

    def grouped(i):
        d = sets[i % nsets]
        dg.dual_gemm_grouped(*d, rows, workspace=wsg)

    ms_g, clocks = time_graph(grouped, args.steps, args.warmup, 1)
    ms_e, _ = time_graph(per_expert, args.steps, args.warmup, 1)
    us_g = ms_g * 1e3 / args.steps
    us_e = ms_e * 1e3 / args.steps
    flops = 4 * sum(rows) * n * k
    peaks = load_peaks()
    return {
        "metric": cfg["name"], "value": round(flops / (us_g * 1e-6) / 1e12, 3),
        "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_g / args.steps,
        "us_per_call": round(us_g, 3),
        "per_expert_launches_us_per_call": round(us_e, 3),
        "higher_is_better": True, "data": "synthetic: seeded randn -> NVFP4",
        "config": {"workload": "grouped", "group_rows": rows, "N": n, "K": k,
                   "l2": f"{nsets} rotating input sets (> 2 x 126 MB L2)",
                   "timed": "one CUDA graph of `steps` calls, replayed once"},
        "roofline": {"bound": "hbm",
                     "achieved": round(per / (us_g * 1e-6) / 1e9, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(per / (us_g * 1e-6) / 1e9 /
                                   peaks["hbm_gbs"], 4),
                     "algorithmic_bytes": per,
                     "peak_source": f"{peaks['source']} HBM copy GB/s"},
        "gpu_launches": args.steps, "clocks": clocks,
    }


def run_nvfp4_out(args, cfg):
    """The dual GEMM emitting NVFP4 (codes + blocked scales of fp16(h)) for
    the next GEMM: the fused epilogue (one launch) against the unfused
    sequence (fp16 C, then the activation quantiser over C), both graph-timed
    over the same rotating input sets."""
    import nvfp4_dual_gemm_b200 as dg
    from nvfp4_dual_gemm_b200 import _lib

    lib = _lib.load()
    m, n, k = cfg["rows"], cfg["N"], cfg["K"]
    wl = WORKLOADS["c2"]
    sets, nsets = make_sets(dg, m, n, k, wl, 0)
    cq = torch.empty((m, n // 2), dtype=torch.uint8, device="cuda")
    sfc = torch.empty((((m + 127) // 128) * (n // 64) * 512,),
                      dtype=torch.uint8, device="cuda")

    def fused(i):
        d = sets[i % nsets]
        dg.dual_gemm_nvfp4(d[0], d[1], d[2], d[6], d[7], d[8], cq, sfc)

    def unfused(i):
        d = sets[i % nsets]
        dg.dual_gemm(d[0], d[1], d[2], d[6], d[7], d[8], d[9])
        rc = lib.nvfp4_quantize_rows(
            d[9].data_ptr(), _lib.DTYPE_F16, m, n, n, cq.data_ptr(), None,
            sfc.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert rc == 0, _lib.last_error()

    ms_f, clocks = time_graph(fused, args.steps, args.warmup, 1)
    ms_u, _ = time_graph(unfused, args.steps, args.warmup, 1)
    us_f = ms_f * 1e3 / args.steps
    us_u = ms_u * 1e3 / args.steps
    tflops = algo_flops(m, n, k) / (us_f * 1e-6) / 1e12
    peaks = load_peaks()
    # bytes: the inputs plus the NVFP4 output (codes + scales) instead of C
    byts = algo_bytes(m, n, k) - 2 * m * n + m * n // 2 + sfc.numel()
    gbs = byts / (us_f * 1e-6) / 1e9
    return {
        "metric": cfg["name"], "value": round(tflops, 3), "unit": "TFLOP/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_f / args.steps, "us_per_call": round(us_f, 3),
        "unfused_us_per_call": round(us_u, 3),
        "higher_is_better": True, "data": "synthetic: seeded randn -> NVFP4",
        "config": {"workload": "nvfp4_out", "M": m, "N": n, "K": k,
                   "plan": dg.plan(m, n, k),
                   "l2": f"{nsets} rotating input sets (> 2 x 126 MB L2)",
                   "timed": "one CUDA graph of `steps` calls, replayed once"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(gbs / peaks["hbm_gbs"], 4),
                     "algorithmic_bytes": byts,
                     "peak_source": f"{peaks['source']} HBM copy GB/s"},
        "gpu_launches": args.steps, "clocks": clocks,
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c2")
    ap.add_argument("--flags", type=int, default=0,
                    help="NVFP4DG_FLAG_* bits (0 = automatic schedule)")
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--shapes", action="store_true",
                    help="also time C2/C3/C4 and report their geomean")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-static-weights", action="store_true",
                    help="time without NVFP4DG_FLAG_STATIC_WEIGHTS (weight "
                         "copies then also wait for the previous kernel)")
    ap.add_argument("--plumbing", choices=sorted(PLUMBING),
                    help="time the activation quantiser or the scale layout "
                         "converter instead of the dual GEMM (1 GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.plumbing:
        print(json.dumps(run_plumbing(args)), flush=True)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        line = run_reference(args, world, rank)
        print(json.dumps(line), flush=True)
        return
    world, rank, _ = dist_setup()
    try:
        line = run_ours(args, world, rank)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
