#!/usr/bin/env python
"""Benchmark of the NVFP4 dual GEMM  C = silu(A B1^T) * (A B2^T).

The metric is BASELINE's: dual-GEMM us per call and effective TFLOP/s (as a
fraction of the FP4-tensor / HBM roofline), geomean over shapes.  The
default workload is every benchmark shape in one run:

  C2 decode   256 x  4096 x 7168   (HBM-bound)
  C3 mid      512 x  3072 x 7168
  C4 prefill 4096 x 14336 x 4096   (tensor-bound)
  C5 N-sharded FFN 8192 x 28672 x 8192, N split over the ranks

One step = one call of each shape (through the reference-compatible entry
point ``custom_kernel(data)``, one call at a time, as the reference's harness
calls it); ``value`` is the geomean over the shapes of the whole job's
TFLOP/s.  Inputs: seeded randn fp32 quantised to NVFP4 (e2m1 codes, e4m3
per-16 scale = amax / 6, blocked scale layout) by plain torch operations on
the GPU (``make_data``), the same bytes for both arms.

Timing: per shape, W untimed calls, then `repeats` timed regions of exactly
K back-to-back calls, each between two CUDA events on the launching stream
with a barrier and a synchronize on both sides; the region's median is the
shape's time (max over ranks).  Inputs rotate over enough independent sets
that more than 2 x the 126 MB L2 is touched between two uses of a set.
Beside it, per shape: the same calls captured in a CUDA graph, end to end
through the host-buffer API (pinned host inputs and output), and cold
single calls (`cold_us_per_call`: each call after a 256 MB write that
evicts L2, timed alone with its launch latency, median of `--cold-reps`),
the way a harness that clears L2 before every call times it.

Multi-GPU (torchrun, one process per GPU): C2/C3/C4 run the full shape on
every rank (weak scaling); C5's N = 28672 is split over the ranks (strong
scaling: rank r owns B1/B2 rows [r N/w, (r+1) N/w) and their scale bytes,
A is replicated).  No collective on the timed path.

  --impl reference  the reference's own implementation of the path on the
                    same inputs: its kernel, compiled from its sources
                    (oracle/_ref; its dispatch entry for C2/C3, its launcher
                    template instantiated for C4/C5), called eagerly the way
                    its custom_kernel calls it.  Under torchrun rank 0 alone
                    runs it, on one rank's shapes (n_gpus 1).
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
ALL = ["c2", "c3", "c4", "c5"]
METRIC = ("dual-GEMM µs & effective TFLOPS (% of FP4/HBM roofline), "
          "geomean over shapes")
L2_BYTES = 126 * 2 ** 20
EAGER_TIMED = ("per shape: `repeats` regions of exactly `steps` back-to-back "
               "eager calls, CUDA events on the launching stream, barrier + "
               "synchronize around each region; median region")
GRAPH_TIMED = ("`repeats` replays of one CUDA graph of `steps` calls, CUDA "
               "events around each replay; median replay")


def algo_bytes(m, n, k):
    """A + B1 + B2 codes, their e4m3 scales and the fp16 C."""
    return m * k // 2 + n * k + m * k // 16 + 2 * (n * k // 16) + 2 * m * n


def algo_flops(m, n, k):
    return 4.0 * m * n * k


def geomean(vals):
    vals = [v for v in vals if v is not None and v > 0]
    if not vals:
        return None
    return math.exp(sum(map(math.log, vals)) / len(vals))


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return {"hbm_gbs": float(pk["hbm_gbs"]),
                "bf16_tflops": float(pk["bf16_tflops"]),
                "bf16_tflops_sustained": float(
                    pk.get("bf16_tflops_sustained", pk["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0,
                "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def load_traffic(workload):
    """DRAM bytes per launch from a committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", "dram_traffic.json")
    try:
        with open(path) as f:
            v = json.load(f).get(workload)
        return None if v is None else float(v)
    except Exception:
        return None


def roofline(m, n, k, us, peaks, workload):
    """Roofline object of one call of m x n x k taking `us`: the slower of
    the FP4-tensor bound (4 x the measured bf16 rate, NVIDIA's dense FP4:bf16
    ratio; the burst figure for short calls, the sustained one for calls of
    a millisecond or more) and the HBM bound (measured copy bandwidth)."""
    byts = algo_bytes(m, n, k)
    flops = algo_flops(m, n, k)
    bf16 = peaks["bf16_tflops"] if us < 1000 else peaks["bf16_tflops_sustained"]
    fp4 = 4.0 * bf16
    t_hbm = byts / (peaks["hbm_gbs"] * 1e9)
    t_tc = flops / (fp4 * 1e12)
    if t_hbm >= t_tc:
        ach = byts / (us * 1e-6) / 1e9
        r = {"bound": "hbm", "achieved": round(ach, 1),
             "peak": peaks["hbm_gbs"], "unit": "GB/s",
             "frac": round(ach / peaks["hbm_gbs"], 4)}
    else:
        ach = flops / (us * 1e-6) / 1e12
        r = {"bound": "tensor", "achieved": round(ach, 1), "peak": fp4,
             "unit": "TFLOP/s", "frac": round(ach / fp4, 4)}
    r["traffic"] = load_traffic(workload)
    r["traffic_source"] = ("dram__bytes_read.sum + dram__bytes_write.sum per "
                           "launch from an earlier ncu capture of this "
                           "workload (profiles/dram_traffic.json), not "
                           "measured in this run")
    r["algorithmic_bytes"] = byts
    r["algorithmic_flops"] = flops
    r["peak_source"] = (
        f"{peaks['source']} HBM copy GB/s; FP4 dense = 4 x {peaks['source']} "
        f"bf16 cuBLAS TF/s ({'burst' if us < 1000 else 'sustained'})")
    return r


class ClockSampler:
    """Polls NVML (SM clock, throttle reasons) from a thread while running;
    samples accumulate over every timed region it brackets."""

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
        self._period = period_s
        self._h = None
        self._stop = None
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(
                self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._h = None

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
            self._stop = threading.Event()
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._h is not None:
            self._stop.set()
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
        # keep stdout to the one JSON line (NCCL prints its version at INFO)
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def gather_ranks(x, world):
    """Every rank's value of x (a float), in rank order."""
    if world == 1:
        return [x]
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device="cuda")
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(v.item()) for v in out]


# --------------------------------------------------------------------------
# inputs: NVFP4 quantisation in plain torch (no library code), the same
# recipe as the oracle's quantiser (oracle/nvfp4_oracle.py: quantize,
# to_blocked); tests/test_bench_inputs.py checks the bytes against it.
# --------------------------------------------------------------------------
_E2M1_CUTS = (0.25, float(np.nextafter(np.float32(0.75), np.float32(0))), 1.25,
              float(np.nextafter(np.float32(1.75), np.float32(0))), 2.5,
              float(np.nextafter(np.float32(3.5), np.float32(0))), 5.0)


def nvfp4_quantize_torch(x):
    """[rows, K] float32 -> (codes [rows, K/2] uint8, element 2i in the low
    nibble; scales [rows, K/16] uint8 e4m3).  Scale = e4m3(amax / 6) (round
    to nearest even, saturating at 448); code = e2m1(x / scale) rounded to
    nearest with ties to the even code, saturating at 6, sign kept; a block
    whose scale is 0 gets zero codes."""
    rows, k = x.shape
    blk = x.reshape(rows, k // 16, 16)
    amax = blk.abs().amax(dim=2)
    sf = (amax / 6.0).clamp(max=448.0).to(torch.float8_e4m3fn)
    sd = sf.to(torch.float32).unsqueeze(-1)
    q = torch.where(sd > 0, blk / sd, torch.zeros_like(blk))
    cuts = torch.tensor(_E2M1_CUTS, dtype=torch.float32, device=x.device)
    mag = torch.bucketize(q.abs(), cuts, right=False).to(torch.uint8)
    codes = (mag | (torch.signbit(q).to(torch.uint8) << 3)).reshape(rows, k)
    packed = codes[:, 0::2] | (codes[:, 1::2] << 4)
    return packed.contiguous(), sf.view(torch.uint8)


def blocked_torch(sf):
    """Plain scales [rows, K/16] uint8 -> the blocked layout (512-byte atoms
    of 128 rows x 4 scales, atom = rowblock * (K/64) + k64, byte
    (r % 32) * 16 + ((r % 128) // 32) * 4 + c % 4), padding rows zero."""
    rows, kb = sf.shape
    rb = (rows + 127) // 128
    pad = torch.zeros((rb * 128, kb), dtype=torch.uint8, device=sf.device)
    pad[:rows] = sf
    return (pad.view(rb, 4, 32, kb // 4, 4).permute(0, 3, 2, 1, 4)
            .contiguous().view(-1))


def make_data(m, n, k, seed, a_scale, w_scale, device, chunk=4096):
    """The reference's ``data`` 10-tuple (a, b1, b2, sfa, sfb1, sfb2,
    sfa_blocked, sfb1_blocked, sfb2_blocked, c) for one seeded problem:
    operands float4_e2m1fn_x2 [rows, K/2, 1], plain scales float8_e4m3fn
    [rows, K/16, 1], blocked scales float8_e4m3fn (flat), c float16
    [m, n, 1]."""
    gen = torch.Generator(device=device)
    out, plain, blocked = [], [], []
    for idx, (rows, scale) in enumerate(((m, a_scale), (n, w_scale),
                                         (n, w_scale))):
        gen.manual_seed(seed * 1000003 + idx)
        codes = torch.empty((rows, k // 2), dtype=torch.uint8, device=device)
        sf = torch.empty((rows, k // 16), dtype=torch.uint8, device=device)
        for r0 in range(0, rows, chunk):
            r1 = min(rows, r0 + chunk)
            x = torch.randn((r1 - r0, k), generator=gen, device=device,
                            dtype=torch.float32)
            if scale != 1.0:
                x.mul_(scale)
            codes[r0:r1], sf[r0:r1] = nvfp4_quantize_torch(x)
            del x
        out.append(codes.view(torch.float4_e2m1fn_x2).unsqueeze(-1))
        plain.append(sf.view(torch.float8_e4m3fn).unsqueeze(-1))
        blocked.append(blocked_torch(sf).view(torch.float8_e4m3fn))
    c = torch.empty((m, n, 1), dtype=torch.float16, device=device)
    return (out[0], out[1], out[2], plain[0], plain[1], plain[2],
            blocked[0], blocked[1], blocked[2], c)


def shard_data(d, n, k, world, rank):
    """Rank `rank`'s slice of a full problem for N-sharding: B1/B2 rows
    [r N/w, (r+1) N/w) and the matching bytes of their blocked scales (one
    contiguous range when N/w is a multiple of 128; views, no copies), A and
    SFA replicated, a local C [m, N/w, 1]."""
    if world == 1:
        return d
    rows = n // world
    if rows % 128:
        raise SystemExit(f"N / world = {rows} is not a multiple of 128")
    n0 = rank * rows
    per_rb = (k // 64) * 512
    s0, s1 = (n0 // 128) * per_rb, ((n0 + rows) // 128) * per_rb
    c = torch.empty((d[9].size(0), rows, 1), dtype=torch.float16,
                    device=d[9].device)
    return (d[0], d[1][n0:n0 + rows], d[2][n0:n0 + rows], d[3],
            d[4][n0:n0 + rows], d[5][n0:n0 + rows], d[6], d[7][s0:s1],
            d[8][s0:s1], c)


def rank_shape(key, world):
    wl = WORKLOADS[key]
    n = wl["N"] // world if wl.get("strong") else wl["N"]
    return wl["M"], n, wl["K"]


def make_sets(key, world, rank, device, seed0=0):
    """Rotating input sets for one workload on this rank: enough that more
    than 2 x L2 is touched between two uses of a set.  For the strong
    (N-sharded) workload each set is generated in full and sliced."""
    wl = WORKLOADS[key]
    m, n, k = rank_shape(key, world)
    nsets = max(2, math.ceil(2 * L2_BYTES / algo_bytes(m, n, k)))
    sets = []
    for s in range(nsets):
        seed = seed0 + 100 * s + (0 if wl.get("strong") else rank)
        if wl.get("strong"):
            full = make_data(wl["M"], wl["N"], wl["K"], seed, wl["a"],
                             wl["w"], device)
            sets.append(shard_data(full, wl["N"], wl["K"], world, rank))
        else:
            sets.append(make_data(m, n, k, seed, wl["a"], wl["w"], device))
    torch.cuda.synchronize()
    return sets


# --------------------------------------------------------------------------
# timing
# --------------------------------------------------------------------------
def _region(fn, world, clk=None):
    """One timed region: barrier + synchronize, events around fn(),
    synchronize + barrier; returns ms."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    start.record()
    fn()
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    return start.elapsed_time(end)


def time_eager(step_fn, steps, warmup, world, repeats):
    """W untimed calls, then `repeats` regions of exactly `steps`
    back-to-back calls; returns (median ms per region, every region's ms,
    clock summary)."""
    for i in range(warmup):
        step_fn(i)
    torch.cuda.synchronize()

    def region():
        for i in range(steps):
            step_fn(i)

    times = []
    with ClockSampler(torch.cuda.current_device()) as clk:
        for _ in range(repeats):
            times.append(_region(region, world))
    return statistics.median(times), times, clk.summary()


COLD_TIMED = ("per shape: `cold_reps` single calls, each after a 256 MB "
              "device write that evicts L2 (2 x its 126 MB), CUDA events "
              "around that one call on the launching stream; median call "
              "(the way a harness that clears L2 between calls times it)")
_FLUSH = []


def time_cold(step_fn, reps, world):
    """`reps` single calls, each preceded by a write of a buffer twice the
    L2 size and bracketed by its own CUDA events; returns the median ms of
    one call, max over ranks (the launch latency of the call is inside)."""
    if not _FLUSH:
        _FLUSH.append(torch.empty(256 << 20, dtype=torch.uint8,
                                  device="cuda"))
    buf = _FLUSH[0]
    step_fn(0)
    torch.cuda.synchronize()
    evs = []
    for i in range(reps):
        buf.zero_()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        step_fn(i)
        e.record()
        evs.append((s, e))
    torch.cuda.synchronize()
    ms = statistics.median(s.elapsed_time(e) for s, e in evs)
    return max(gather_ranks(ms, world))


def time_allgather(d, key, world, rank, reps):
    """The optional all-gather of the N-sharded C (NCCL, after the kernels,
    not part of `value`): shard.gather_columns of this rank's [M, N/w] slice
    into the full [M, N], `reps` calls between events, median per call, max
    over ranks; bus bandwidth as NCCL counts it for an all-gather."""
    from nvfp4_dual_gemm_b200 import shard

    wl = WORKLOADS[key]
    spec = shard.shard_spec(wl["N"], wl["K"], world, rank)
    c_local = d[9].squeeze(-1)
    shard.gather_columns(c_local, spec)  # warm-up (NCCL channels)
    times = []
    for _ in range(reps):
        times.append(_region(lambda: shard.gather_columns(c_local, spec),
                             world))
    ms = max(gather_ranks(statistics.median(times), world))
    full = c_local.numel() * c_local.element_size() * world
    return {"us": round(ms * 1e3, 1),
            "bytes_out_per_rank": full,
            "busbw_gbs": round(full * (world - 1) / world / (ms * 1e-3) / 1e9,
                               1),
            "what": "nvfp4_dual_gemm_b200.shard.gather_columns: NCCL "
                    "all_gather of the [M, N/w] fp16 slices + column "
                    "assembly into [M, N]; reported separately, not in "
                    "value"}


def time_graph(step_fn, steps, warmup, world, repeats=1):
    """Warm up eagerly, capture `steps` calls in one CUDA graph, replay it
    `repeats` times, each replay a timed region; returns (median ms per
    replay, clock summary)."""
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
    times = []
    with ClockSampler(torch.cuda.current_device()) as clk:
        for _ in range(repeats):
            times.append(_region(g.replay, world))
    del g
    return statistics.median(times), clk.summary()


def time_e2e(one, h2d, d2h, steps, world):
    """Events around `steps` end-to-end steps (each uploads its inputs from
    pinned host memory and downloads C); returns ms."""
    one()
    torch.cuda.synchronize()

    def region():
        for _ in range(steps):
            one()

    return _region(region, world)


def merge_clocks(parts):
    samples = sum(p.get("samples", 0) for p in parts)
    mhz = [p["sm_mhz"] for p in parts if p.get("sm_mhz") is not None]
    reasons = sorted({r for p in parts for r in p.get("reasons", [])})
    return {"sm_mhz": statistics.median(mhz) if mhz else None,
            "sm_max_mhz": next((p["sm_max_mhz"] for p in parts
                                if p.get("sm_max_mhz")), None),
            "reasons": reasons, "samples": samples,
            "per_workload_sm_mhz": [p.get("sm_mhz") for p in parts]}


# --------------------------------------------------------------------------
# CPU baseline: the oracle (CPU restatement of the path) on a bounded sample
# --------------------------------------------------------------------------
def cpu_baseline(d, key, budget_s=6.0):
    """Dequantise-to-fp32 + fp32 BLAS matmuls + SiLU (oracle/) on a row
    sample of one workload, all host threads; dequantisation and matmuls
    timed separately (median of up to 5 repetitions)."""
    from threadpoolctl import threadpool_info, threadpool_limits

    from oracle import nvfp4_oracle as O

    m, n, k = d[0].size(0), d[1].size(0), 2 * d[0].size(1)
    rows = min(m, 32 if n <= 4096 else 16)
    cols = min(n, 4096 if n <= 4096 else 2048)
    host = [t.view(torch.uint8).squeeze(-1)[:r].cpu().numpy()
            for t, r in ((d[0], rows), (d[3], rows), (d[1], cols),
                         (d[4], cols), (d[2], cols), (d[5], cols))]
    cores = os.cpu_count() or 1
    t_dq, t_mm = [], []
    with threadpool_limits(limits=cores):
        threads = max([i.get("num_threads", 1) for i in threadpool_info()]
                      or [1])
        t_start = time.perf_counter()
        while len(t_dq) < 5 and (len(t_dq) < 1 or
                                 time.perf_counter() - t_start < budget_s):
            t0 = time.perf_counter()
            a = O.dequantize(host[0], host[1])
            b1 = O.dequantize(host[2], host[3])
            b2 = O.dequantize(host[4], host[5])
            t1 = time.perf_counter()
            with np.errstate(over="ignore"):
                O.silu_mul(a @ b1.T, a @ b2.T).astype(np.float16)
            t2 = time.perf_counter()
            t_dq.append(t1 - t0)
            t_mm.append(t2 - t1)
    dq, mm = statistics.median(t_dq), statistics.median(t_mm)
    flops = algo_flops(rows, cols, k)
    return {"workload": key, "value": flops / (dq + mm) / 1e12,
            "unit": "TFLOP/s", "cores": threads,
            "sample": f"{rows} rows of A x {cols} rows of B1/B2, K = {k}",
            "dequantise_s": dq, "matmul_silu_s": mm, "reps": len(t_dq)}


def cpu_baseline_all(data_by_key):
    per = [cpu_baseline(d, key) for key, d in data_by_key.items()]
    return {"value": geomean([p["value"] for p in per]), "unit": "TFLOP/s",
            "cores": max(p["cores"] for p in per), "kind": "port",
            "sample": "geomean over the shapes of the oracle (dequantise + "
                      "fp32 matmul + SiLU) on a row sample of each: " +
                      "; ".join(f"{p['workload']}: {p['sample']}" for p in per),
            "shapes": per}


# --------------------------------------------------------------------------
# arms
# --------------------------------------------------------------------------
def _host_copies(d):
    """Pinned host copies of one set's six inputs (uint8) and of C."""
    dev_in = [d[0], d[1], d[2], d[6], d[7], d[8]]
    host_in = [t.view(torch.uint8).cpu().pin_memory() for t in dev_in]
    c_host = torch.empty(d[9].shape, dtype=torch.float16).pin_memory()
    return dev_in, host_in, c_host


def _nbytes(ts):
    return sum(t.numel() * t.element_size() for t in ts)


def run_ours(args, world, rank):
    import nvfp4_dual_gemm_b200 as dg

    keys = ALL if args.workload == "all" else [args.workload]
    peaks = load_peaks()
    shapes, clocks, cpu = [], [], []
    h2d_total = d2h_total = 0
    launches = 0
    for key in keys:
        m, n, k = rank_shape(key, world)
        sets = make_sets(key, world, rank, "cuda")
        ns = len(sets)

        def step(i):
            dg.custom_kernel(sets[i % ns])

        ms, regions, clk = time_eager(step, args.steps, args.warmup, world,
                                      args.repeats)
        clocks.append(clk)
        launches += args.steps * args.repeats
        ranks_ms = gather_ranks(ms, world)
        us = max(ranks_ms) * 1e3 / args.steps
        flops_job = algo_flops(m, n, k) * world
        ent = {"workload": key, "name": WORKLOADS[key]["name"], "M": m,
               "N_per_rank": n, "K": k,
               "us_per_call": round(us, 3),
               "us_per_call_ranks": [round(v * 1e3 / args.steps, 3)
                                     for v in ranks_ms],
               "us_per_call_min_region": round(min(regions) * 1e3 /
                                               args.steps, 3),
               "tflops": round(flops_job / (us * 1e-6) / 1e12, 2),
               "roofline": roofline(m, n, k, us, peaks, key),
               "plan": dg.plan(m, n, k), "input_sets": ns,
               "l2": f"{ns} rotating input sets of "
                     f"{algo_bytes(m, n, k) / 1e6:.1f} MB (> 2 x 126 MB L2 "
                     "between reuses)"}
        if args.cold_reps > 0:
            ent["cold_us_per_call"] = round(
                time_cold(step, args.cold_reps, world) * 1e3, 3)
            launches += args.cold_reps + 1
        if WORKLOADS[key].get("strong") and world > 1:
            ent["allgather"] = time_allgather(sets[0], key, world, rank,
                                              max(3, args.steps // 2))
        # the same calls captured in a CUDA graph (caller workspace, so the
        # capture allocates nothing), with and without STATIC_WEIGHTS
        if not args.no_graph:
            from nvfp4_dual_gemm_b200 import _lib
            for tag, fl in (("graph", 0),
                            ("graph_static_weights", _lib.FLAG_STATIC_WEIGHTS)):
                ws = torch.zeros(max(dg.workspace_size(m, n, k, fl), 256),
                                 dtype=torch.uint8, device="cuda")

                def gstep(i, fl=fl, ws=ws):
                    d = sets[i % ns]
                    dg.dual_gemm(d[0], d[1], d[2], d[6], d[7], d[8], d[9],
                                 flags=fl, workspace=ws)

                gms, _ = time_graph(gstep, args.steps, args.warmup, world,
                                    args.repeats)
                ent[f"{tag}_us_per_call"] = round(
                    max(gather_ranks(gms, world)) * 1e3 / args.steps, 3)
                del ws
        # end to end through the public host-buffer API: pinned host inputs
        # and output; the library uploads, computes and downloads
        if args.e2e_steps > 0:
            dev_in, host_in, c_host = _host_copies(sets[0])
            c_host = c_host.squeeze(-1)
            e2e_steps = max(1, min(args.steps, args.e2e_steps))

            def one():
                dg.dual_gemm_host(*host_in, c_host)

            e_ms = max(gather_ranks(time_e2e(one, None, None, e2e_steps,
                                             world), world))
            ent["e2e_tflops"] = round(flops_job * e2e_steps /
                                      (e_ms * 1e-3) / 1e12, 3)
            h2d_total += _nbytes(host_in)
            d2h_total += _nbytes([c_host])
            del host_in, c_host
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            cpu.append(cpu_baseline(sets[0], key))
        shapes.append(ent)
        del sets
        torch.cuda.empty_cache()

    value = geomean([s["tflops"] for s in shapes])
    head = next((s for s in shapes if s["workload"] == "c2"), shapes[0])
    roof = dict(head["roofline"])
    roof["workload"] = head["workload"]
    roof["geomean_frac_over_shapes"] = round(
        geomean([s["roofline"]["frac"] for s in shapes]), 4)
    strong = [k for k in keys if WORKLOADS[k].get("strong")]
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "repeats": args.repeats,
        "ms_per_step": sum(s["us_per_call"] for s in shapes) / 1e3,
        "us_per_call": {s["workload"]: s["us_per_call"] for s in shapes},
        "cold_us_per_call": {s["workload"]: s.get("cold_us_per_call")
                             for s in shapes},
        "higher_is_better": True,
        "scaling": "weak",
        "scaling_by_workload": {k: ("strong" if WORKLOADS[k].get("strong")
                                    else "weak") for k in keys},
        "vs_baseline": None,
        "dtype": "nvfp4 (e2m1 x e4m3/16, fp32 accumulate, fp16 out)",
        "data": "synthetic: seeded randn -> NVFP4 by torch ops on the GPU",
        "config": {
            "workload": ("all four benchmark shapes (C2, C3, C4, C5)"
                         if args.workload == "all"
                         else WORKLOADS[args.workload]["name"]),
            "shapes": keys, "L": 1,
            "parallelism": (f"{world} ranks: " +
                            ("C5 N-sharded (strong), " if strong else "") +
                            "C2-C4 one full problem per rank (weak)")
            if world > 1 else "single GPU",
            "step": "one call of each shape",
            "api": "custom_kernel(data) -> torch binding _C -> C ABI "
                   "nvfp4_dual_gemm_run, default flags",
            "timed": EAGER_TIMED,
            "cold": COLD_TIMED,
            "l2": "per shape, rotating input sets touching > 2 x 126 MB "
                  "between reuses of a set"},
        "shapes": shapes,
        "roofline": roof,
        "e2e": {"value": round(geomean([s.get("e2e_tflops") for s in shapes])
                               or 0.0, 3),
                "unit": "TFLOP/s", "h2d_bytes_per_step": h2d_total,
                "d2h_bytes_per_step": d2h_total,
                "api": "nvfp4_dual_gemm_b200.dual_gemm_host (C ABI "
                       "nvfp4_dual_gemm_run_host), geomean over the shapes"},
        "gpu_launches": launches,
        "gpu_launches_note": "dual GEMM kernel launches in the eager timed "
                             "regions that give `value` (one per call) and "
                             "in the cold single-call timings",
        "clocks": merge_clocks(clocks),
    }
    if cpu:
        line["cpu_baseline"] = {
            "value": geomean([p["value"] for p in cpu]), "unit": "TFLOP/s",
            "cores": max(p["cores"] for p in cpu), "kind": "port",
            "sample": "geomean over the shapes of the oracle (dequantise + "
                      "fp32 matmul + SiLU) on a row sample of each: " +
                      "; ".join(f"{p['workload']}: {p['sample']}"
                                for p in cpu),
            "shapes": cpu}
    return line


def ref_custom_kernel(entry, data):
    """The reference's custom_kernel (submission.py:1153-1157): unpack the
    10-tuple and call its torch-extension function with the blocked
    scales."""
    a, b1, b2, _sfa, _sfb1, _sfb2, sfa_b, sfb1_b, sfb2_b, c = data
    return entry(a, b1, b2, sfa_b, sfb1_b, sfb2_b, c)


def run_reference(args, world):
    """The reference's own implementation on rank 0's shapes: its kernel
    built from its sources (oracle/_ref), called eagerly as its
    custom_kernel calls it; the CPU port of its algorithm where no kernel
    is available.  Never imports this repository's package."""
    from oracle import build_ref

    mod = build_ref.load()
    keys = ALL if args.workload == "all" else [args.workload]
    peaks = load_peaks()
    shapes, clocks, cpu = [], [], []
    h2d_total = d2h_total = 0
    missing = []
    for key in keys:
        m, n, k = rank_shape(key, world)
        entry = build_ref.entry(mod, (m, n, k))
        sets = make_sets(key, world, 0, "cuda")
        ns = len(sets)
        if entry is None:
            missing.append(key)
            cpu.append(cpu_baseline(sets[0], key))
            shapes.append({"workload": key, "M": m, "N_per_rank": n, "K": k,
                           "tflops": cpu[-1]["value"],
                           "kind": "CPU port (no reference kernel)"})
            del sets
            continue

        def step(i):
            ref_custom_kernel(entry, sets[i % ns])

        ms, regions, clk = time_eager(step, args.steps, args.warmup, 1,
                                      args.repeats)
        clocks.append(clk)
        us = ms * 1e3 / args.steps
        ent = {"workload": key, "name": WORKLOADS[key]["name"], "M": m,
               "N_per_rank": n, "K": k, "us_per_call": round(us, 3),
               "us_per_call_min_region": round(min(regions) * 1e3 /
                                               args.steps, 3),
               "tflops": round(algo_flops(m, n, k) / (us * 1e-6) / 1e12, 2),
               "roofline": roofline(m, n, k, us, peaks, key),
               "entry": ("cuda_nvfp4_dual_gemm (its dispatch table)"
                         if (m, n, k) in build_ref.SAFE_SHAPES else
                         "cuda_nvfp4_dual_gemm_generic (its launcher "
                         "template, instantiated for this shape)")}
        if args.cold_reps > 0:
            ent["cold_us_per_call"] = round(
                time_cold(step, args.cold_reps, 1) * 1e3, 3)
        if args.e2e_steps > 0:
            d0 = sets[0]
            dev_in, host_in, c_host = _host_copies(d0)
            e2e_steps = max(1, min(args.steps, args.e2e_steps))

            def one():
                for h, dv in zip(host_in, dev_in):
                    dv.view(torch.uint8).copy_(h, non_blocking=True)
                ref_custom_kernel(entry, d0)
                c_host.copy_(d0[9], non_blocking=True)

            e_ms = time_e2e(one, None, None, e2e_steps, 1)
            ent["e2e_tflops"] = round(algo_flops(m, n, k) * e2e_steps /
                                      (e_ms * 1e-3) / 1e12, 3)
            h2d_total += _nbytes(host_in)
            d2h_total += _nbytes([c_host])
        if not args.no_cpu_baseline and world == 1:
            cpu.append(cpu_baseline(sets[0], key))
        shapes.append(ent)
        del sets
        torch.cuda.empty_cache()

    value = geomean([s["tflops"] for s in shapes])
    head = next((s for s in shapes if s["workload"] == "c2"), shapes[0])
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s",
        "n_gpus": 1, "ranks_in_job": world, "impl": "reference",
        "steps": args.steps, "warmup": args.warmup, "repeats": args.repeats,
        "ms_per_step": sum(s.get("us_per_call", 0.0) for s in shapes) / 1e3,
        "us_per_call": {s["workload"]: s.get("us_per_call") for s in shapes},
        "cold_us_per_call": {s["workload"]: s.get("cold_us_per_call")
                             for s in shapes},
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "nvfp4 (e2m1 x e4m3/16, fp32 accumulate, fp16 out)",
        "data": "synthetic: seeded randn -> NVFP4 by torch ops on the GPU "
                "(the same bytes as the other arm)",
        "config": {"workload": ("all four benchmark shapes (C2, C3, C4, C5)"
                                if args.workload == "all"
                                else WORKLOADS[args.workload]["name"]),
                   "shapes": keys, "L": 1,
                   "parallelism": ("rank 0 alone, on one rank's shapes "
                                   f"(C5 N / {world})" if world > 1 else
                                   "single GPU"),
                   "timed": EAGER_TIMED, "cold": COLD_TIMED},
        "reference_kind": ("the reference's CUDA kernel compiled from its "
                           "sources by oracle/build_ref.py, called as its "
                           "custom_kernel calls it (submission.py:1153-1157)"
                           if mod is not None else
                           "CPU port of the reference algorithm "
                           "(oracle/_ref not built)"),
        "shapes": shapes,
        "roofline": dict(head.get("roofline", {}), workload=head["workload"]),
        "e2e": {"value": round(geomean([s.get("e2e_tflops") for s in shapes])
                               or 0.0, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d_total,
                "d2h_bytes_per_step": d2h_total,
                "api": "pinned H2D of the inputs, the reference's entry, "
                       "D2H of C, on the current stream"},
        "clocks": merge_clocks(clocks) if clocks else None,
    }
    if missing:
        line["cpu_port_for"] = missing
    if cpu:
        line["cpu_baseline"] = {
            "value": geomean([p["value"] for p in cpu]), "unit": "TFLOP/s",
            "cores": max(p["cores"] for p in cpu), "kind": "port",
            "sample": "; ".join(f"{p['workload']}: {p['sample']}"
                                for p in cpu),
            "note": "the reference's own CPU path (its harness's dequantise-"
                    "to-fp32 check) is not part of the reference; this is "
                    "the oracle's restatement of it",
            "shapes": cpu}
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
    """Time one of the kernels beside the dual GEMM (the formats and callers
    on either side of it): the activation quantiser or the scale layout
    converter, in a
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
    ms, clocks = time_graph(step, args.steps, args.warmup, 1, args.repeats)
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
                   "timed": GRAPH_TIMED},
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

    ms_1, clocks = time_graph(one_launch, args.steps, args.warmup, 1, args.repeats)
    ms_l, _ = time_graph(per_batch, args.steps, args.warmup, 1, args.repeats)
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
                   "timed": GRAPH_TIMED},
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

    ms_g, clocks = time_graph(grouped, args.steps, args.warmup, 1, args.repeats)
    ms_e, _ = time_graph(per_expert, args.steps, args.warmup, 1, args.repeats)
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
                   "timed": GRAPH_TIMED},
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
    sets = make_sets("c2", 1, 0, "cuda")
    nsets = len(sets)
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

    ms_f, clocks = time_graph(fused, args.steps, args.warmup, 1, args.repeats)
    ms_u, _ = time_graph(unfused, args.steps, args.warmup, 1, args.repeats)
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
                   "timed": GRAPH_TIMED},
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
    ap.add_argument("--steps", type=int, default=20,
                    help="calls per timed region (per shape)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--repeats", type=int, default=50,
                    help="timed regions per shape; the median is reported")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["all"] + ALL, default="all")
    ap.add_argument("--e2e-steps", type=int, default=10,
                    help="end-to-end steps per shape (0: skip)")
    ap.add_argument("--no-graph", action="store_true",
                    help="skip the CUDA-graph timings beside the eager ones")
    ap.add_argument("--cold-reps", type=int, default=30,
                    help="single calls after an L2 flush per shape, timed "
                         "one by one (0: skip)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--plumbing", choices=sorted(PLUMBING),
                    help="time one of the kernels beside the dual GEMM "
                         "instead (1 GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    args.repeats = max(1, args.repeats)
    if args.plumbing:
        print(json.dumps(run_plumbing(args)), flush=True)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        # rank 0 alone runs the reference arm; the other ranks have no work
        if rank != 0:
            return
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        print(json.dumps(run_reference(args, world)), flush=True)
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
