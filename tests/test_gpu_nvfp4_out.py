"""GPU tests of the NVFP4-output dual GEMM (``nvfp4_dual_gemm_run_nvfp4_out``).

The fused output must equal, bit for bit, the oracle's quantiser applied to
the fp16 C that ``nvfp4_dual_gemm_run`` produces for the same inputs and
schedule (the accumulation order, hence C, depends on the schedule, so both
calls get the same flags); that C itself is checked against the oracle's
product within rtol = atol = 1e-3.  Every epilogue path is covered: whole
tiles of the 1-SM and the 2-SM pair kernel, stream-K owners, and cluster
split-K in both kernels, with ragged M (padding rows whose scales must be 0)
and the odd CTA of a pair lying past M.
"""
import numpy as np
import pytest
import torch

import nvfp4_dual_gemm_b200 as dg
from nvfp4_dual_gemm_b200 import _lib
from oracle import nvfp4_oracle as O
from tests.helpers import assert_close, to_device

pytestmark = pytest.mark.gpu

BN64, BN128 = _lib.FLAG_BN64, _lib.FLAG_BN128
PATHS = {
    "1sm_bn64": BN64 | _lib.FLAG_NO_PAIR | _lib.FLAG_NO_STREAMK,
    "1sm_bn128": BN128 | _lib.FLAG_NO_PAIR | _lib.FLAG_NO_STREAMK,
    "pair_bn64": BN64 | _lib.FLAG_PAIR | _lib.FLAG_NO_STREAMK,
    "pair_bn128": BN128 | _lib.FLAG_PAIR | _lib.FLAG_NO_STREAMK,
    "streamk_1sm": 5 | BN128 | _lib.FLAG_NO_PAIR | _lib.FLAG_FORCE_STREAMK,
    "streamk_pair": 3 | BN64 | _lib.FLAG_PAIR | _lib.FLAG_FORCE_STREAMK,
    "splitk_1sm": BN128 | _lib.FLAG_NO_PAIR | _lib.FLAG_SPLITK,
    "splitk_pair": BN64 | _lib.FLAG_PAIR | _lib.FLAG_SPLITK,
    "auto": 0,
}


def _fp16_and_nvfp4(p, flags):
    d = to_device(p)
    dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                 d["sfb1_blocked"], d["sfb2_blocked"], d["c"],
                 flags=flags | _lib.FLAG_SYNC_CHECK)
    m, n = p["M"], p["N"]
    # poisoned outputs: every byte must be written
    cq = torch.full((m, n // 2), 0xAB, dtype=torch.uint8, device="cuda")
    sfc = torch.full((O.blocked_size(m, n),), 0xCD, dtype=torch.uint8,
                     device="cuda")
    dg.dual_gemm_nvfp4(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                       d["sfb1_blocked"], d["sfb2_blocked"], cq, sfc,
                       flags=flags | _lib.FLAG_SYNC_CHECK)
    torch.cuda.synchronize()
    return d["c"].cpu().numpy(), cq.cpu().numpy(), sfc.cpu().numpy()


def _check_quantised(c16, cq, sfc, what):
    codes, sf = O.quantize(c16.astype(np.float32))
    blk = O.to_blocked(sf)
    if not np.array_equal(cq, codes):
        bad = np.argwhere(cq != codes)
        raise AssertionError(f"{what}: {len(bad)} code bytes differ, first "
                             f"{bad[:4].tolist()}")
    if not np.array_equal(sfc, blk):
        bad = np.flatnonzero(sfc != blk)
        raise AssertionError(f"{what}: {len(bad)} scale bytes differ, first "
                             f"offsets {bad[:4].tolist()}")


@pytest.mark.parametrize("path", list(PATHS))
@pytest.mark.parametrize("m,n,k", [(256, 512, 2048), (200, 256, 768),
                                   (300, 384, 1024)])
def test_nvfp4_out_equals_quantised_fp16(path, m, n, k):
    flags = PATHS[path]
    if flags & BN128 and n % 128:
        pytest.skip("BN = 128 needs N % 128 == 0")
    p = O.make_problem(m, n, k, seed=3 * m + n + k)
    c16, cq, sfc = _fp16_and_nvfp4(p, flags)
    assert_close(c16, O.reference_output(p), f"{path} {m}x{n}x{k} fp16")
    _check_quantised(c16, cq, sfc, f"{path} {m}x{n}x{k}")


def test_nvfp4_out_decode_shape_and_overflow():
    # C2's shape: the auto plan (pair split-K); its seeded randn inputs give
    # products beyond the fp16 range, so blocks holding +-inf are covered
    p = O.make_problem(256, 4096, 7168, seed=21)
    c16, cq, sfc = _fp16_and_nvfp4(p, 0)
    assert np.isinf(c16).any()
    _check_quantised(c16, cq, sfc, "256x4096x7168")


def test_nvfp4_out_feeds_the_next_dual_gemm():
    # The output is a valid A operand: quantised h of one dual GEMM is the
    # input of another (N of the first = K of the second).
    p = O.make_problem(128, 512, 512, seed=4, a_scale=0.05, w_scale=0.05)
    d = to_device(p)
    cq, sfc = dg.dual_gemm_nvfp4(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                                 d["sfb1_blocked"], d["sfb2_blocked"])
    q = O.make_problem(128, 256, 512, seed=5)
    e = to_device(q)
    c2 = torch.empty((128, 256), dtype=torch.float16, device="cuda")
    dg.dual_gemm(cq, e["b1"], e["b2"], sfc, e["sfb1_blocked"],
                 e["sfb2_blocked"], c2, flags=_lib.FLAG_SYNC_CHECK)
    torch.cuda.synchronize()
    sf_plain = O.from_blocked(sfc.cpu().numpy(), 128, 512)
    ref = O.dual_gemm(cq.cpu().numpy(), sf_plain, q["b1"], q["sfb1"],
                      q["b2"], q["sfb2"])
    assert_close(c2.cpu().numpy(), ref, "chained")


def test_nvfp4_out_empty_k_and_invalid_args():
    p = O.make_problem(130, 128, 256, seed=1)
    d = to_device(p)
    cq = torch.full((130, 64), 0xAB, dtype=torch.uint8, device="cuda")
    sfc = torch.full((O.blocked_size(130, 128),), 0xCD, dtype=torch.uint8,
                     device="cuda")
    empty = torch.empty((130, 0), dtype=torch.uint8, device="cuda")
    emptyb = torch.empty((128, 0), dtype=torch.uint8, device="cuda")
    nothing = torch.empty((0,), dtype=torch.uint8, device="cuda")
    dg.dual_gemm_nvfp4(empty, emptyb, emptyb, nothing, nothing, nothing, cq,
                       sfc)
    torch.cuda.synchronize()
    assert not cq.cpu().numpy().any() and not sfc.cpu().numpy().any()
    lib = _lib.load()
    args = [d[k].data_ptr() for k in ("a", "b1", "b2", "sfa_blocked",
                                      "sfb1_blocked", "sfb2_blocked")]
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.nvfp4_dual_gemm_run_nvfp4_out(*args, None, sfc.data_ptr(), 130,
                                           128, 256, 1, 0, stream)
    assert rc == _lib.ERR_INVALID
    rc = lib.nvfp4_dual_gemm_run_nvfp4_out(*args, cq.data_ptr(), None, 130,
                                           128, 256, 1, 0, stream)
    assert rc == _lib.ERR_INVALID
    rc = lib.nvfp4_dual_gemm_run_nvfp4_out(*args, cq.data_ptr(),
                                           sfc.data_ptr() + 8, 130, 128, 256,
                                           1, 0, stream)
    assert rc == _lib.ERR_ALIGN
