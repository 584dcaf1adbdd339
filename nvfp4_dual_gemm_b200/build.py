"""Build the in-tree C-ABI library ``libnvfp4dg.so`` for sm_100a and the
torch binding ``_C`` over it.

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
    # one name for both loaders (ctypes by path, the torch binding by its
    # DT_NEEDED entry), so they share one copy of the library's state
    "-Xlinker",
    "-soname=libnvfp4dg.so",
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


EXT_SOURCE = os.path.join(CSRC, "torch_ext.cpp")


def ext_path() -> str:
    import sysconfig

    return os.path.join(PKG_DIR, "_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_ext(force: bool = False, verbose: bool = False) -> str:
    """Compile the torch binding ``_C`` (pybind11 module over the C ABI,
    linked against libnvfp4dg.so beside it); returns its path."""
    out = ext_path()
    deps = [EXT_SOURCE, os.path.join(INCLUDE, "nvfp4_dual_gemm.h"),
            os.path.abspath(__file__), LIB_PATH]
    if (not force and os.path.exists(out) and
            all(os.path.getmtime(d) <= os.path.getmtime(out) for d in deps)):
        return out
    import sysconfig

    import torch
    from torch.utils import cpp_extension as ce

    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    torch_dir = os.path.dirname(os.path.abspath(torch.__file__))
    cuda_home = ce.CUDA_HOME or "/usr/local/cuda"
    incs = [os.path.join(torch_dir, "include"),
            os.path.join(torch_dir, "include", "torch", "csrc", "api",
                         "include"),
            os.path.join(cuda_home, "include"),
            sysconfig.get_paths()["include"], INCLUDE]
    tmp = out + ".tmp"
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-shared",
           "-fPIC", "-fvisibility=hidden", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{d}" for d in incs], EXT_SOURCE, "-o", tmp,
           f"-L{os.path.join(torch_dir, 'lib')}", f"-L{PKG_DIR}",
           "-lnvfp4dg", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
           "-ltorch_python", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(
            f"g++ failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, out)
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
    print(build_ext(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
