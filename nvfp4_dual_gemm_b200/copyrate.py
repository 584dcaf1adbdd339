"""Copy-rate microbenchmark of B200 (maintainer tool).

Builds ``csrc/copy_rate.cu`` and runs it on the current GPU::

    python -m nvfp4_dual_gemm_b200.copyrate

It prints, as CSV, for 1 to all SMs copying at once, copies of 2 KiB and
16 KiB and 1, 2 or 4 issuing warps per SM: the cycles a thread spends issuing
one bulk global->shared copy, the cycles per copy until all bytes landed,
and the bytes per cycle each SM received.  These are the two figures the
kernels' producers are designed around: a thread issues its copies one at a
time while different warps issue side by side, and the global->shared
bandwidth an SM gets falls as more SMs copy at the same time.  A second
table gives the distributed-shared-memory exchange rate of clusters of two
CTAs sending 64 KiB to each other (bulk copies of several sizes, and
16-byte st.async stores), the cluster split-K epilogue's pattern.
"""
from __future__ import annotations

import os
import subprocess
import sys

from . import build as _build

BIN = os.path.join(_build.PKG_DIR, "copy_rate")


def build_binary(force: bool = False) -> str:
    src = os.path.join(_build.CSRC, "copy_rate.cu")
    if (not force and os.path.exists(BIN) and
            os.path.getmtime(BIN) >= os.path.getmtime(src)):
        return BIN
    cmd = [_build.nvcc_path(), *_build.ARCH_FLAGS, "-O2", "-std=c++17", src,
           "-o", BIN]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{res.stderr}")
    return BIN


def main() -> int:
    return subprocess.call([build_binary()])


if __name__ == "__main__":
    sys.exit(main())
