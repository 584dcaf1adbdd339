"""Generate the golden vectors that pin the oracle to the reference kernel.

Run on a machine with a B200 and the reference kernel built into
``oracle/_ref`` (``python oracle/build_ref.py`` where the reference sources
are present)::

    python tests/golden/make_golden.py [MxNxK ...]

For each case the inputs come from ``oracle.nvfp4_oracle.make_problem`` (seeded
numpy, bit-reproducible on any machine), the output from the reference's own
``cuda_nvfp4_dual_gemm`` (nvfp4_dual_gemm.cu:381-446) on the GPU.  A fixture
keeps a sample of output rows, the SHA-256 of the full fp16 output and of the
inputs, and how the reference compares with the oracle over the full output.
Only shapes of the reference's dispatch table with K/256 >= 4 are run
(``oracle.build_ref.SAFE_SHAPES``); the others are out of bounds for it.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import nvfp4_oracle as O  # noqa: E402

# (M, N, K, seed, a_scale, w_scale, sampled rows); the last two are the
# benchmark's decode (C2) and mid (C3) shapes, both in the reference's
# dispatch table (nvfp4_dual_gemm.cu:404-406, 413-415; C3's output is
# column-major there and is read back in row-major order)
CASES = [
    (512, 768, 7168, 11, 1.0, 1.0, 8),
    (256, 3072, 4096, 12, 1.0, 1.0, 8),
    (512, 768, 7168, 14, 0.5, 0.02, 8),
    (256, 4096, 7168, 21, 1.0, 1.0, 64),
    (512, 3072, 7168, 22, 1.0, 1.0, 64),
]


def fixture_path(m, n, k, seed) -> str:
    return os.path.join(HERE, f"ref_{m}x{n}x{k}_s{seed}.npz")


def input_digest(p: dict) -> str:
    h = hashlib.sha256()
    for key in ("a", "b1", "b2", "sfa_blocked", "sfb1_blocked",
                "sfb2_blocked"):
        h.update(np.ascontiguousarray(p[key]).tobytes())
    return h.hexdigest()


def sample_rows(m: int, count: int, seed: int) -> np.ndarray:
    return np.sort(np.random.default_rng([seed, 99]).choice(
        m, size=count, replace=False)).astype(np.int64)


def main() -> None:
    import torch

    from oracle import build_ref
    sys.path.insert(0, os.path.dirname(HERE))
    from helpers import to_device

    ref = build_ref.load()
    if ref is None:
        raise SystemExit("reference module not built (oracle/_ref)")
    # optional filter: shapes as MxNxK (default: every case)
    only = set(sys.argv[1:])
    for (m, n, k, seed, a_s, w_s, nrows) in CASES:
        if only and f"{m}x{n}x{k}" not in only:
            continue
        assert (m, n, k) in build_ref.SAFE_SHAPES
        p = O.make_problem(m, n, k, seed=seed, a_scale=a_s, w_scale=w_s)
        d = to_device(p)
        out = ref.cuda_nvfp4_dual_gemm(d["a"], d["b1"], d["b2"],
                                       d["sfa_blocked"], d["sfb1_blocked"],
                                       d["sfb2_blocked"], d["c"])
        torch.cuda.synchronize()
        c = out.reshape(m, n).cpu().numpy().astype(np.float16)
        full = O.reference_output(p)
        ok, n_bad, worst = O.check_close(c, full)
        rows = sample_rows(m, nrows, seed)
        np.savez_compressed(
            fixture_path(m, n, k, seed),
            shape=np.array([m, n, k], dtype=np.int64),
            seed=np.array(seed, dtype=np.int64),
            scales=np.array([a_s, w_s], dtype=np.float64),
            rows=rows,
            c_rows=c[rows],
            c_sha256=np.array(hashlib.sha256(
                np.ascontiguousarray(c).tobytes()).hexdigest()),
            inputs_sha256=np.array(input_digest(p)),
            oracle_outside_tol=np.array(n_bad, dtype=np.int64),
            nonfinite=np.array(int((~np.isfinite(c)).sum()), dtype=np.int64))
        print(f"{m}x{n}x{k} seed {seed}: {n_bad} of {c.size} outputs outside "
              f"rtol=atol=1e-3 vs the oracle (worst {worst}) -> "
              f"{os.path.basename(fixture_path(m, n, k, seed))}", flush=True)


if __name__ == "__main__":
    main()
