"""Build the in-tree C-ABI library ``libnvfp4dg.so`` for sm_100a.

The library is compiled with nvcc straight from ``csrc/`` and links the CUDA
runtime statically, so it loads on machines without a GPU driver (the
driver entry point it needs, cuTensorMapEncodeTiled, is resolved at run time
through cudaGetDriverEntryPoint).  Usage::

    python -m nvfp4_dual_gemm_b200.build          # rebuild if sources changed
    python -m nvfp4_dual_gemm_b200.build --force
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
LIB_NAME = "libnvfp4dg.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

SOURCES = ["dual_gemm.cu"]
DEPS = ["dual_gemm.cu", "schedule.h", "sm100_ptx.cuh"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-cudart",
    "static",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC")
    if cand:
        return cand
    found = shutil.which("nvcc")
    if found:
        return found
    default = "/usr/local/cuda/bin/nvcc"
    if os.path.exists(default):
        return default
    raise RuntimeError("nvcc not found (set NVCC or put it on PATH)")


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    lib_mtime = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC, d) for d in DEPS]
    deps.append(os.path.join(INCLUDE, "nvfp4_dual_gemm.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(d) > lib_mtime for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile libnvfp4dg.so in-tree; returns its path."""
    if not force and not _stale():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, "-shared",
           "-I", INCLUDE, "-I", CSRC,
           *[os.path.join(CSRC, s) for s in SOURCES], "-o", tmp]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(
            f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
