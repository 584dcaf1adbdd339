"""GPU parity of the host-buffer entry point (nvfp4_dual_gemm_run_host):
inputs and C in host memory, the library uploads the weights slab by slab,
runs one kernel per slab and downloads each slab of C while later slabs
upload.  Checked against the oracle at rtol = atol = 1e-3 for automatic and
forced slab counts, a last slab narrower than the others (N % 128 == 64),
page-locked and ordinary host memory, repeated calls through one staging
buffer, and K = 0."""
import numpy as np
import pytest
import torch

import nvfp4_dual_gemm_b200 as dg
from nvfp4_dual_gemm_b200 import _lib
from oracle import nvfp4_oracle as O
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu


def host_tensors(p, pin=True):
    h = {}
    for k in ("a", "b1", "b2", "sfa_blocked", "sfb1_blocked", "sfb2_blocked"):
        t = torch.from_numpy(np.ascontiguousarray(p[k]))
        h[k] = t.pin_memory() if pin else t.clone()
    c = torch.full((p["M"], p["N"]), float("nan"), dtype=torch.float16)
    h["c"] = c.pin_memory() if pin else c
    return h


def call(h, **kw):
    dg.dual_gemm_host(h["a"], h["b1"], h["b2"], h["sfa_blocked"],
                      h["sfb1_blocked"], h["sfb2_blocked"], h["c"], **kw)
    torch.cuda.current_stream().synchronize()
    return h["c"].numpy().copy()


@pytest.mark.parametrize("m,n,k,slabs", [
    (256, 1024, 2048, 0),
    (256, 1024, 2048, 1),
    (256, 1024, 2048, 3),       # 384 + 384 + 256 rows
    (200, 320, 1024, 2),        # 256 + 64 rows, ragged M
    (128, 4096, 7168, 0),       # decode-like, automatic slabs
    (640, 1536, 1024, 16),      # one 128-row group per slab
])
def test_host_entry_matches_oracle(m, n, k, slabs):
    p = O.make_problem(m, n, k, seed=m + n + k + slabs)
    h = host_tensors(p)
    got = call(h, slabs=slabs)
    assert_close(got, O.reference_output(p), f"host entry {m}x{n}x{k}/{slabs}")


@pytest.mark.parametrize("slabs", [1, 3])  # 1: everything on the caller's stream
def test_host_entry_pageable_memory_and_repeat_calls(slabs):
    m, n, k = 256, 768, 1536
    p = O.make_problem(m, n, k, seed=5)
    q = O.make_problem(m, n, k, seed=6)
    want_p, want_q = O.reference_output(p), O.reference_output(q)
    hp, hq = host_tensors(p, pin=False), host_tensors(q, pin=True)
    staging = torch.empty(dg.host_staging_size(m, n, k), dtype=torch.uint8,
                          device="cuda")
    for rep in range(2):
        # alternating problems through one staging buffer, queued back to
        # back before any synchronisation
        for h in (hp, hq):
            h["c"].fill_(float("nan"))
            dg.dual_gemm_host(h["a"], h["b1"], h["b2"], h["sfa_blocked"],
                              h["sfb1_blocked"], h["sfb2_blocked"], h["c"],
                              slabs=slabs, staging=staging)
        torch.cuda.current_stream().synchronize()
        assert_close(hp["c"].numpy(), want_p, f"pageable call {rep}")
        assert_close(hq["c"].numpy(), want_q, f"pinned call {rep}")


def test_host_entry_same_result_as_device_entry_without_k_split():
    # With whole single-CTA tiles of one width, each output is one K loop in
    # the same order whichever slab its tile falls in, so the two entry
    # points agree bit for bit.
    m, n, k = 384, 1024, 2048
    p = O.make_problem(m, n, k, seed=9)
    h = host_tensors(p)
    flags = (_lib.FLAG_NO_STREAMK | _lib.FLAG_NO_SPLITK | _lib.FLAG_NO_PAIR |
             _lib.FLAG_BN64)
    got = call(h, slabs=4, flags=flags)
    d = {key: v.cuda() for key, v in h.items()}
    dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                 d["sfb1_blocked"], d["sfb2_blocked"], d["c"], flags=flags)
    torch.cuda.synchronize()
    assert np.array_equal(got.view(np.uint16),
                          d["c"].cpu().numpy().view(np.uint16))


def test_host_entry_k_zero_writes_zeros():
    m, n = 64, 128
    a = torch.zeros(m, 0, dtype=torch.uint8)
    b = torch.zeros(n, 0, dtype=torch.uint8)
    sf = torch.zeros(0, dtype=torch.uint8)
    c = torch.full((m, n), float("nan"), dtype=torch.float16).pin_memory()
    dg.dual_gemm_host(a, b, b, sf, sf, sf, c)
    torch.cuda.current_stream().synchronize()
    assert torch.count_nonzero(c).item() == 0
