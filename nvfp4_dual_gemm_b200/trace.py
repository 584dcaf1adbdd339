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
    # accumulator hold of whole-tile epilogues (ready -> released, role 8)
    # and the phases of the cluster split-K epilogue (role 8, slots 41-45)
    hold, split = [], []
    for c in range(buf.shape[0]):
        t = buf[c]
        for u in range(40):
            if t[4, u] > 0 and t[8, u] > 0:
                hold.append(t[8, u] - t[4, u])
        if t[4, 0] > 0 and t[8, 41] > 0 and t[8, 43] > 0:
            split.append([t[8, 41] - t[4, 0], t[8, 42] - t[8, 41],
                          t[8, 43] - t[8, 42], t[8, 44] - t[8, 43],
                          t[5, 0] - t[8, 44]])
    med = np.median(np.array(rows, dtype=np.float64), axis=0)
    keys = ["first_mma", "period", "mma_issue", "scale_store", "scale_land",
            "epilogue", "kblocks"]
    out = {k: float(v) for k, v in zip(keys, med)}
    out["ctas"] = len(rows)
    if hold:
        out["epilogue_hold"] = float(np.median(hold))
    # pair kernel prologue (role 9 slots 56-60, SM cycles from entry, role 4
    # slot 61): barriers initialised, producer past its CTA barrier, past
    # the cluster barrier, past the dependency wait, TMEM allocated (the
    # 1-SM kernel uses role 9 for per-block stamps instead)
    ent = buf[:, 4, 61]
    for slot, name in ((56, "pro_bar_init"), (57, "pro_prod_cta_bar"),
                       (58, "pro_prod_cluster_bar"), (59, "pro_prod_depwait"),
                       (60, "pro_tmem_alloc")):
        v = buf[:, 9, slot]
        ok_ = (v > 0) & (ent > 0)
        if ok_.sum() > 0:
            out[name] = float(np.median(v[ok_] - ent[ok_]))
    if split:
        sm = np.median(np.array(split, dtype=np.float64), axis=0)
        for k, v in zip(["split_peer_ready", "split_send", "split_own_ld",
                         "split_first_recv", "split_rest"], sm):
            out[k] = float(v)
    # global-timer stamps (ns) of every CTA: entry, end of the prologue,
    # exit
    ent = buf[:, 5, 61]
    ok = ent > 0
    if ok.any():
        ent, dep, ext = ent[ok], buf[ok, 5, 62], buf[ok, 5, 63]
        out["ns_entry_skew"] = float(ent.max() - ent.min())
        out["ns_prologue"] = float(np.median(dep - ent))
        out["ns_cta_span"] = float(np.median(ext - ent))
        out["ns_kernel_span"] = float(ext.max() - ent.min())
        # pair kernel (slots 50-53): from the earliest return of the
        # dependency wait (the previous grid's completion as this grid sees
        # it) to the last exit, and the teardown's phases
        dep = buf[ok, 5, 53]
        td0, td1, td2 = buf[ok, 5, 50], buf[ok, 5, 51], buf[ok, 5, 52]
        has = (dep > 0) & (td0 > 0) & (td1 > 0) & (td2 > 0)
        if has.any():
            rel = dep[has].min()
            out["ns_release_skew"] = float(np.median(dep[has]) - rel)
            out["ns_release_to_last_teardown"] = float(td0[has].max() - rel)
            out["ns_release_to_last_exit"] = float(ext.max() - rel)
            out["ns_store_read_wait"] = float(np.median(td1[has] - td0[has]))
            out["ns_final_cluster_sync"] = float(
                np.median(td2[has] - td1[has]))
            out["ns_dealloc_to_exit"] = float(np.median(ext[has] - td2[has]))
            # each warp's arrival at the teardown (role 9 slots 40-50, SM
            # cycles) relative to thread 0's, the latest warp per CTA
            t0 = buf[ok, 4, 50]
            arr = buf[ok, 9, 40:51]
            sel = (t0 > 0) & (arr > 0).all(axis=1)
            if sel.any():
                rel_w = arr[sel] - t0[sel][:, None]
                out["cyc_teardown_arrival_by_warp"] = [
                    float(v) for v in np.median(rel_w, axis=0)]
                out["cyc_teardown_latest_warp"] = float(
                    np.median(rel_w.max(axis=1)))
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
    ap.add_argument("--back-to-back", action="store_true",
                    help="no synchronize before the traced call: it starts "
                         "while the previous calls drain, as in a stream of "
                         "calls (the stamps of the last call win)")
    ap.add_argument("--raw", default=None,
                    help="also save the raw stamp buffer (.npy) here")
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
    if args.back_to_back:
        for i in range(args.calls):
            call(i)
    call(args.calls)
    torch.cuda.synchronize()
    lib.nvfp4_dual_gemm_trace_read(buf.ctypes.data, buf.nbytes)
    if args.raw:
        np.save(args.raw, buf)
    print({"problem": [m, n, k], "flags": args.flags,
           "plan": api.plan(m, n, k, args.flags), **summarise(buf)})


if __name__ == "__main__":
    main(sys.argv[1:])
