"""GPU test of nvfp4_dual_gemm_run_noalloc, the entry point for callers that
cannot allocate device memory when they call (a custom arena or pool owns all
device memory, the framework's allocator must not be re-entered, or the call
sits on a path that must not block on the allocator).  Its scratch lives in a
static device array, so it is checked against the ordinary entry point
(nvfp4_dual_gemm_run, whose scratch comes from cudaMalloc) on the same inputs,
within the tolerance of the other parity tests, on two calls in a row — the
second call reuses the array with the previous call's contents in it.

This file is collected last so that a run stopping at the first failure has
already run every other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

import nvfp4_dual_gemm_b200 as dg
from nvfp4_dual_gemm_b200 import _lib
from oracle import nvfp4_oracle as O
from tests.helpers import assert_close, to_device

pytestmark = pytest.mark.gpu


def _noalloc(d, m, n, k, flags):
    lib = _lib.load()
    rc = lib.nvfp4_dual_gemm_run_noalloc(
        d["a"].data_ptr(), d["b1"].data_ptr(), d["b2"].data_ptr(),
        d["sfa_blocked"].data_ptr(), d["sfb1_blocked"].data_ptr(),
        d["sfb2_blocked"].data_ptr(), d["c"].data_ptr(), m, n, k, 1,
        flags | _lib.FLAG_SYNC_CHECK, torch.cuda.current_stream().cuda_stream)
    return rc


@pytest.mark.parametrize("flags", [
    # tiles split along K, so the static scratch is used
    5 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_BN64 | _lib.FLAG_NO_PAIR,
    6 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_BN128 | _lib.FLAG_PAIR,
    # the largest forced stream-K grid whose partials still fit the array
    31 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_BN64 | _lib.FLAG_NO_PAIR,
    # the automatic schedule (no scratch needed for this shape)
    0,
])
def test_noalloc_matches_run_twice(flags):
    m, n, k = 256, 512, 2048
    p = O.make_problem(m, n, k, seed=31)
    ref_plan = dg.plan(m, n, k, flags)
    if flags & _lib.FLAG_FORCE_STREAMK:
        assert ref_plan["sk_tiles"] > 0
        need = dg.workspace_size(m, n, k, flags)
        assert 0 < need <= _lib.NOALLOC_SCRATCH_BYTES
    d = to_device(p)
    dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                 d["sfb1_blocked"], d["sfb2_blocked"], d["c"],
                 flags=flags | _lib.FLAG_SYNC_CHECK)
    torch.cuda.synchronize()
    want = d["c"].cpu().numpy()
    assert_close(want, O.reference_output(p), "ordinary entry point")
    for call in range(2):
        d["c"].fill_(float("nan"))
        rc = _noalloc(d, m, n, k, flags)
        assert rc == _lib.OK, _lib.last_error()
        torch.cuda.synchronize()
        got = d["c"].cpu().numpy()
        assert_close(got, want, f"no-allocation call {call + 1}")


def _ordinary(d, flags=0):
    dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                 d["sfb1_blocked"], d["sfb2_blocked"], d["c"],
                 flags=flags | _lib.FLAG_SYNC_CHECK)
    torch.cuda.synchronize()
    return d["c"].cpu().numpy()


def test_noalloc_falls_back_to_whole_tiles_when_stream_k_does_not_fit():
    # the automatic schedule of this shape is stream-K over a full grid,
    # whose partials (~39 MB) exceed the array: the call runs whole tiles
    m, n, k = 512, 5120, 4096
    auto = dg.plan(m, n, k)
    assert auto["sk_tiles"] > 0
    assert dg.workspace_size(m, n, k) > _lib.NOALLOC_SCRATCH_BYTES
    p = O.make_problem(m, n, k, seed=33)
    d = to_device(p)
    want = _ordinary(d)
    for call in range(2):
        d["c"].fill_(float("nan"))
        rc = _noalloc(d, m, n, k, 0)
        assert rc == _lib.OK, _lib.last_error()
        torch.cuda.synchronize()
        assert_close(d["c"].cpu().numpy(), want,
                     f"no-allocation call {call + 1} (whole tiles)")


def test_noalloc_calls_with_different_shapes_in_a_row():
    # the second call finds the first one's partials and counters at other
    # offsets of the array
    cases = [
        (256, 512, 2048, 5 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_BN64 |
         _lib.FLAG_NO_PAIR, 41),
        (384, 768, 2048, 6 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_BN128 |
         _lib.FLAG_PAIR, 42),
        (256, 512, 2048, 31 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_BN64 |
         _lib.FLAG_NO_PAIR, 43),
    ]
    for m, n, k, flags, seed in cases:
        assert dg.plan(m, n, k, flags)["sk_tiles"] > 0
        d = to_device(O.make_problem(m, n, k, seed=seed))
        want = _ordinary(d, flags)
        d["c"].fill_(float("nan"))
        rc = _noalloc(d, m, n, k, flags)
        assert rc == _lib.OK, _lib.last_error()
        torch.cuda.synchronize()
        assert_close(d["c"].cpu().numpy(), want, f"{m}x{n}x{k}")


def test_noalloc_rejects_schedules_beyond_the_static_scratch():
    # a stream-K schedule forced by the caller is not replaced
    m, n, k = 256, 4096, 7168
    flags = 148 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_BN128 | _lib.FLAG_NO_PAIR
    assert dg.workspace_size(m, n, k, flags) > _lib.NOALLOC_SCRATCH_BYTES
    d = {name: torch.zeros(size, dtype=torch.uint8, device="cuda")
         for name, size in (("a", m * k // 2), ("b1", n * k // 2),
                            ("b2", n * k // 2),
                            ("sfa_blocked", (m // 128) * (k // 64) * 512),
                            ("sfb1_blocked", (n // 128) * (k // 64) * 512),
                            ("sfb2_blocked", (n // 128) * (k // 64) * 512))}
    d["c"] = torch.zeros((m, n), dtype=torch.float16, device="cuda")
    rc = _noalloc(d, m, n, k, flags)
    assert rc == _lib.ERR_WORKSPACE
    assert "scratch" in _lib.last_error()
    torch.cuda.synchronize()
    assert not d["c"].any()  # nothing was launched
