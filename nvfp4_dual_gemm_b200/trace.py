"""Pipeline trace of the dual GEMM kernels (maintainer tool).

Builds a variant of the library compiled with ``-DNVFP4DG_TRACE`` (the
kernels then record the SM clock at each hand-off of the first 64 K blocks
of every CTA and at the epilogue's start and end), runs one problem and
prints the median per-CTA timeline in SM cycles::

    python -m nvfp4_dual_gemm_b200.trace 256 4096 7168 [--flags F] [--calls N]

Columns: first MMA (cycles from the producer's first copy to the first MMA),
period (cycles between consecutive K blocks at the MMA issuer), the MMA
issuer's per-block issue time, the scale warps' store time, the time from the
producer's empty-slot wait to the scales landing, and the epilogue's length;
then, from global-timer stamps (ns), the spread of CTA start times, the
prologue up to the dependency wait, a CTA's median life and the kernel's span
from the first CTA's start to the last CTA's exit.
The traced build is slower than the product build (every stamp is a global
store); use it for where the cycles go, not for absolute speed.
"""
from __future__ import annotations

import argparse
import ctypes
import os
import subprocess
import sys

import numpy as np

from . import build as _build

TRACE_LIB = os.path.join(_build.PKG_DIR, "libnvfp4dg_trace.so")
CTAS, ROLES, SLOTS = 160, 10, 64


def build_trace_lib(force: bool = False) -> str:
    src = os.path.join(_build.CSRC, "dual_gemm.cu")
    deps = [os.path.join(_build.CSRC, d) for d in _build.DEPS]
    if (not force and os.path.exists(TRACE_LIB) and
            all(os.path.getmtime(d) <= os.path.getmtime(TRACE_LIB)
                for d in deps)):
        return TRACE_LIB
    cmd = [_build.nvcc_path(), "-DNVFP4DG_TRACE", *_build.ARCH_FLAGS,
           *_build.NVCC_FLAGS, "-shared", "-I", _build.INCLUDE, "-I",
           _build.CSRC, src, "-o", TRACE_LIB]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{res.stderr}")
    return TRACE_LIB


def summarise(buf: np.ndarray) -> dict:
    rows = []
    for c in range(buf.shape[0]):
        t = buf[c]
        nkb = int((t[2] > 0).sum())
        if nkb < 4:
            continue
        hi = min(nkb, SLOTS)
        t0 = t[0, 0]
        rows.append([
            t[2, 0] - t0,
            np.diff(t[2, 2:hi]).mean(),
            (t[3, 2:hi] - t[2, 2:hi]).mean(),
            (t[7, 2:hi] - t[6, 2:hi]).mean(),
            (t[6, 2:hi] - t[0, 2:hi]).mean(),
            t[5, 0] - t[4, 0],
            nkb,
        ])
    if not rows:
        return {}
    med = np.median(np.array(rows, dtype=np.float64), axis=0)
    keys = ["first_mma", "period", "mma_issue", "scale_store", "scale_land",
            "epilogue", "kblocks"]
    out = {k: float(v) for k, v in zip(keys, med)}
    out["ctas"] = len(rows)
    # global-timer stamps (ns) of every CTA: entry, past the dependency wait,
    # exit
    ent = buf[:, 5, 61]
    ok = ent > 0
    if ok.any():
        ent, dep, ext = ent[ok], buf[ok, 5, 62], buf[ok, 5, 63]
        out["ns_entry_skew"] = float(ent.max() - ent.min())
        out["ns_prologue"] = float(np.median(dep - ent))
        out["ns_cta_span"] = float(np.median(ext - ent))
        out["ns_kernel_span"] = float(ext.max() - ent.min())
        clk = buf[ok, 4, 63] - buf[ok, 4, 61]
        out["sm_mhz"] = float(np.median(clk / np.maximum(ext - ent, 1)) * 1e3)
        # SM cycles from entry to the first copy, and from the end of the
        # epilogue (role 5 slot 0) to exit, of CTAs that ran an epilogue
        first = buf[ok, 0, 0]
        epi_end = buf[ok, 5, 0]
        has = (first > 0) & (epi_end > 0)
        if has.any():
            out["cyc_entry_to_first_copy"] = float(
                np.median(first[has] - buf[ok, 4, 61][has]))
        # producer's prologue milestones (1-SM kernel): past __syncthreads,
        # before and after the dependency wait (slots 60-62 of role 1, which
        # the per-block stamps reach when a CTA runs 60 or more K blocks)
        sync, pre, post = buf[ok, 1, 60], buf[ok, 1, 61], buf[ok, 1, 62]
        if (sync > 0).any() and out.get("kblocks", 0) < 60:
            e = buf[ok, 4, 61]
            out["cyc_entry_to_sync"] = float(np.median((sync - e)[sync > 0]))
            out["cyc_sync_to_depwait"] = float(
                np.median((pre - sync)[pre > 0]))
            out["cyc_depwait"] = float(np.median((post - pre)[post > 0]))
            out["cyc_depwait_to_first_copy"] = float(
                np.median((first - post)[(post > 0) & (first > 0)]))
            out["cyc_epilogue_to_exit"] = float(
                np.median(buf[ok, 4, 63][has] - epi_end[has]))
    return out


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("m", type=int)
    ap.add_argument("n", type=int)
    ap.add_argument("k", type=int)
    ap.add_argument("--flags", type=lambda s: int(s, 0), default=0)
    ap.add_argument("--calls", type=int, default=4,
                    help="warm-up calls before the traced one")
    args = ap.parse_args(argv)

    import torch

    from . import api

    lib = ctypes.CDLL(build_trace_lib())
    lib.nvfp4_dual_gemm_run.argtypes = ([ctypes.c_void_p] * 7 +
                                        [ctypes.c_int] * 4 +
                                        [ctypes.c_uint, ctypes.c_void_p])
    lib.nvfp4_dual_gemm_trace_read.argtypes = [ctypes.c_void_p,
                                               ctypes.c_size_t]
    buf = np.zeros((CTAS, ROLES, SLOTS), np.int64)
    m, n, k = args.m, args.n, args.k
    sets = [api.generate_input(m, n, k, seed=s) for s in range(4)]

    def call(i):
        d = sets[i % len(sets)]
        rc = lib.nvfp4_dual_gemm_run(
            *[t.data_ptr() for t in (d[0], d[1], d[2], d[6], d[7], d[8],
                                     d[9])],
            m, n, k, 1, args.flags,
            torch.cuda.current_stream().cuda_stream)
        if rc:
            raise RuntimeError(f"nvfp4_dual_gemm_run failed ({rc})")

    for i in range(args.calls):
        call(i)
    torch.cuda.synchronize()
    lib.nvfp4_dual_gemm_trace_read(buf.ctypes.data, buf.nbytes)  # clear
    call(args.calls)
    torch.cuda.synchronize()
    lib.nvfp4_dual_gemm_trace_read(buf.ctypes.data, buf.nbytes)
    print({"problem": [m, n, k], "flags": args.flags,
           "plan": api.plan(m, n, k, args.flags), **summarise(buf)})


if __name__ == "__main__":
    main(sys.argv[1:])
