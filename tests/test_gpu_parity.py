"""GPU parity tests: the CUDA path (through the C ABI) against the CPU oracle.

Tolerance: rtol = atol = 1e-3 on the fp16 output (the task's definition of a
correct result).  Small and mid shapes are compared in full; the large
benchmark shapes are compared on sampled rows x columns (the oracle computes
exactly those outputs) plus size-independent properties.
"""
import numpy as np
import pytest
import torch

import nvfp4_dual_gemm_b200 as dg
from nvfp4_dual_gemm_b200 import _lib
from oracle import nvfp4_oracle as O
from tests.helpers import (assert_close, data_tuple, near_midpoint_fp32,
                           to_device)

pytestmark = pytest.mark.gpu


# Stream-K over all 148 SMs (the grid forced), so that each tile of
# 256 x 512 x 7168 has 9 to 19 contributors.
MANY_CONTRIBUTOR_FLAGS = [
    148 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_NO_PAIR | _lib.FLAG_BN128,
    148 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_NO_PAIR | _lib.FLAG_BN64,
    148 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_PAIR | _lib.FLAG_BN128,
]


def run(p, flags=0, use_custom_kernel=False):
    d = to_device(p)
    if use_custom_kernel:
        out = dg.custom_kernel(data_tuple(d))
        assert out.data_ptr() == d["c"].data_ptr()
    else:
        dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                     d["sfb1_blocked"], d["sfb2_blocked"], d["c"],
                     flags=flags | _lib.FLAG_SYNC_CHECK)
    torch.cuda.synchronize()
    return d["c"].cpu().numpy()


VARIANTS = {
    "auto": 0,
    "bn64": _lib.FLAG_BN64 | _lib.FLAG_NO_PAIR,
    "bn128": _lib.FLAG_BN128 | _lib.FLAG_NO_PAIR,
    "pair_bn64": _lib.FLAG_BN64 | _lib.FLAG_PAIR,
    "pair_bn128": _lib.FLAG_BN128 | _lib.FLAG_PAIR,
    "whole_tiles": _lib.FLAG_NO_STREAMK,
}


@pytest.fixture(scope="module")
def config1():
    p = O.make_problem(128, 256, 256, seed=0)
    return p, O.reference_output(p)


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_config1_variants(config1, variant):
    p, ref = config1
    got = run(p, VARIANTS[variant])
    assert_close(got, ref, f"config1/{variant}")


def test_config1_custom_kernel_entry(config1):
    p, ref = config1
    assert_close(run(p, use_custom_kernel=True), ref, "custom_kernel")


@pytest.fixture(scope="module")
def streamk_problem():
    p = O.make_problem(256, 512, 2048, seed=11)
    return p, O.reference_output(p)


@pytest.mark.parametrize("grid", [1, 2, 3, 5, 7, 13])
@pytest.mark.parametrize("bn", [64, 128])
def test_stream_k_forced_grid(streamk_problem, grid, bn):
    p, ref = streamk_problem
    flag = (_lib.FLAG_BN64 if bn == 64 else _lib.FLAG_BN128) | \
        _lib.FLAG_FORCE_STREAMK | _lib.FLAG_NO_PAIR
    if grid in (3, 5, 7):
        assert dg.plan(256, 512, 2048, grid | flag)["sk_tiles"] > 0
    assert_close(run(p, grid | flag), ref, f"grid={grid} bn={bn}")


@pytest.mark.parametrize("grid", [2, 4, 6, 10, 14])
@pytest.mark.parametrize("bn", [64, 128])
def test_pair_stream_k_forced_grid(streamk_problem, grid, bn):
    p, ref = streamk_problem
    flag = (_lib.FLAG_BN64 if bn == 64 else _lib.FLAG_BN128) | \
        _lib.FLAG_FORCE_STREAMK | _lib.FLAG_PAIR
    pl = dg.plan(256, 512, 2048, grid | flag)
    assert pl["ctas"] == 2
    if grid in (6, 10, 14):
        assert pl["sk_tiles"] > 0
    assert_close(run(p, grid | flag), ref, f"pair grid={grid} bn={bn}")


@pytest.mark.parametrize("flags", MANY_CONTRIBUTOR_FLAGS)
def test_stream_k_many_contributors_per_tile(flags):
    # A long K split over every SM: each tile's owner adds the partials of
    # many other CTAs, more than its staging ring holds at once (the plan
    # itself is checked on the CPU in test_abi.py).
    m, n, k = 256, 512, 7168
    p = O.make_problem(m, n, k, seed=77)
    ref = O.reference_output(p)
    for _ in range(2):
        assert_close(run(p, flags | _lib.FLAG_SYNC_CHECK), ref,
                     f"many contributors {flags:#x}")


def test_stream_k_repeated_calls_reuse_counters(streamk_problem):
    # Each tile's owner resets its counter, so back-to-back launches on the
    # same workspace must all be correct.
    p, ref = streamk_problem
    d = to_device(p)
    for _ in range(3):
        d["c"].fill_(float("nan"))
        dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                     d["sfb1_blocked"], d["sfb2_blocked"], d["c"],
                     flags=5 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_SYNC_CHECK)
        torch.cuda.synchronize()
        assert_close(d["c"].cpu().numpy(), ref, "repeat")


@pytest.mark.parametrize("m,n,k", [(1, 128, 256), (64, 64, 256),
                                   (200, 256, 512), (130, 384, 768),
                                   (333, 192, 1024), (384, 256, 512)])
@pytest.mark.parametrize("pair", [_lib.FLAG_PAIR, _lib.FLAG_NO_PAIR])
def test_ragged_m_and_small_shapes(m, n, k, pair):
    p = O.make_problem(m, n, k, seed=m + n + k)
    assert_close(run(p, pair), O.reference_output(p), f"{m}x{n}x{k}")


@pytest.mark.parametrize("m,n,k,bn", [(256, 512, 2048, 128),
                                      (256, 512, 2048, 64),
                                      (200, 256, 768, 128),
                                      (333, 192, 1024, 64),
                                      (128, 128, 512, 128),
                                      (256, 4096, 7168, 128)])
@pytest.mark.parametrize("pair", [0, _lib.FLAG_PAIR])
def test_cluster_split_k(m, n, k, bn, pair):
    # single CTAs in clusters of two, or 2-SM pairs in clusters of four (the
    # odd CTA of a pair past M for the ragged shapes); K halves exchange
    # partial sums through distributed shared memory
    p = O.make_problem(m, n, k, seed=m + 7 * n + k)
    flags = _lib.FLAG_SPLITK | pair | (_lib.FLAG_BN64 if bn == 64 else
                                       _lib.FLAG_BN128) | _lib.FLAG_SYNC_CHECK
    pl = dg.plan(m, n, k, flags)
    assert pl["split"] == 2 and pl["ctas"] == (2 if pair else 1)
    ref = O.reference_output(p)
    d = to_device(p)
    for _ in range(2):  # twice: no state may leak between launches
        d["c"].fill_(float("nan"))
        dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                     d["sfb1_blocked"], d["sfb2_blocked"], d["c"], flags=flags)
        torch.cuda.synchronize()
        assert_close(d["c"].cpu().numpy(), ref, f"split {m}x{n}x{k} bn={bn}")


# The 13 shapes of the reference's dispatch table (nvfp4_dual_gemm.cu:403-442)
REFERENCE_SHAPES = [
    (256, 4096, 7168), (512, 4096, 7168), (256, 3072, 4096), (512, 3072, 7168),
    (1536, 512, 7168), (256, 512, 256), (3072, 1024, 1536), (7168, 1024, 256),
    (7168, 2304, 2048), (4608, 384, 7168), (7168, 384, 2304), (512, 768, 7168),
    (4096, 768, 512),
]


@pytest.mark.parametrize("m,n,k", REFERENCE_SHAPES)
def test_reference_dispatch_shapes(m, n, k):
    p = O.make_problem(m, n, k, seed=1)
    got = run(p)
    if m * n * k <= 16 * 2 ** 30:
        assert_close(got, O.reference_output(p), f"{m}x{n}x{k}")
    else:
        rng = np.random.default_rng(0)
        rows = np.sort(rng.choice(m, 96, replace=False))
        cols = np.sort(rng.choice(n, 256, replace=False))
        assert_close(got[np.ix_(rows, cols)],
                     O.reference_output(p, rows=rows, cols=cols),
                     f"{m}x{n}x{k} sampled")


def _gpu_problem_sampled_check(m, n, k, a_scale, w_scale, flags=0, seed=5,
                               n_rows=64, n_cols=192):
    data = dg.generate_input(m, n, k, seed=seed, a_scale=a_scale,
                             w_scale=w_scale)
    c = data[9]
    dg.dual_gemm(data[0], data[1], data[2], data[6], data[7], data[8], c,
                 flags=flags | _lib.FLAG_SYNC_CHECK)
    torch.cuda.synchronize()
    rng = np.random.default_rng(seed)
    rows = np.sort(rng.choice(m, n_rows, replace=False))
    cols = np.sort(rng.choice(n, n_cols, replace=False))
    ri = torch.from_numpy(rows).cuda()
    ci = torch.from_numpy(cols).cuda()

    def host(t, idx):
        return t.view(torch.uint8).squeeze(-1).index_select(0, idx).cpu().numpy()

    a, sfa = host(data[0], ri), host(data[3], ri)
    b1, sfb1 = host(data[1], ci), host(data[4], ci)
    b2, sfb2 = host(data[2], ci), host(data[5], ci)
    # the blocked scales the kernel read must hold the same bytes as the plain
    sfa_blk = data[6].view(torch.uint8).cpu().numpy()
    assert np.array_equal(O.from_blocked(sfa_blk, m, k)[rows], sfa)
    ref = O.dual_gemm(a, sfa, b1, sfb1, b2, sfb2)
    got = c.squeeze(-1)[ri][:, ci].cpu().numpy()
    assert_close(got, ref, f"{m}x{n}x{k} sampled")
    return data


def test_config4_prefill_sampled():
    _gpu_problem_sampled_check(4096, 14336, 4096, 0.5, 0.02)


@pytest.mark.parametrize("world", [1, 8])
def test_config5_rank_slice_sampled(world):
    # Each rank of the N-sharded config computes M x (N / world) x K.
    _gpu_problem_sampled_check(8192, 28672 // world, 8192, 0.5, 0.02)


def test_quantizer_bit_exact_against_oracle():
    rng = np.random.default_rng(3)
    rows, k = 300, 1024
    x = rng.standard_normal((rows, k)).astype(np.float32)
    x[0] *= 1e-3          # subnormal e4m3 scales
    x[1] *= 1e4           # saturating scales
    x[2, :16] = 0.0       # all-zero block
    x[3, :16] = 1e-9      # scale rounds to zero
    # exact e2m1 ties: amax = 6 gives scale 1.0, so these land on midpoints
    x[4, :16] = np.array([6, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5,
                          -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5, -0.1],
                         np.float32)
    codes, sf = O.quantize(x)
    blk = O.to_blocked(sf)
    gc, gsf, gblk = dg.quantize_nvfp4(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(gsf.view(torch.uint8).cpu().numpy(), sf)
    assert np.array_equal(gblk.cpu().numpy(), blk)
    gcodes = gc.cpu().numpy()
    if not np.array_equal(gcodes, codes):
        bad = np.argwhere(gcodes != codes)[:8]
        raise AssertionError(f"code mismatch at {bad.tolist()}: gpu "
                             f"{[hex(gcodes[tuple(b)]) for b in bad]} oracle "
                             f"{[hex(codes[tuple(b)]) for b in bad]}")


def test_property_doubling_b2_scales_doubles_output():
    # Adding 1 to the e4m3 exponent of every SFB2 scale multiplies A B2^T by
    # exactly 2, so C must double bit for bit wherever it stays finite.
    p = O.make_problem(256, 4096, 7168, seed=21)
    exps = (p["sfb2"] >> 3) & 0xF
    assert exps.min() >= 1 and exps.max() <= 13
    c1 = run(p)
    q = dict(p)
    q["sfb2"] = (p["sfb2"] + 8).astype(np.uint8)
    q["sfb2_blocked"] = O.to_blocked(q["sfb2"])
    c2 = run(q)
    a1 = np.abs(c1.astype(np.float32))
    # fp16 normal range on both sides: doubling a subnormal is not exact
    fin = np.isfinite(c2) & (a1 < 30000) & (a1 >= 2.0 ** -13)
    assert fin.mean() > 0.4  # silu sends about half the outputs to ~0
    want = (c1[fin].astype(np.float32) * 2).astype(np.float16)
    bad = int((c2[fin] != want).sum())
    assert bad == 0, f"{bad} of {fin.sum()} outputs did not double exactly"


def test_property_row_permutation_equivariance():
    # Whole-tile schedule: every output is summed in the same order, so
    # permuting A's rows permutes C's rows exactly.
    p = O.make_problem(384, 512, 1024, seed=4)
    perm = np.random.default_rng(4).permutation(384)
    q = dict(p)
    q["a"] = p["a"][perm]
    q["sfa"] = p["sfa"][perm]
    q["sfa_blocked"] = O.to_blocked(q["sfa"])
    c = run(p, _lib.FLAG_NO_STREAMK)
    cp = run(q, _lib.FLAG_NO_STREAMK)
    assert np.array_equal(cp, c[perm])


def test_workspace_shared_across_plans(streamk_problem):
    # One library-owned workspace serves calls whose plans differ in tile
    # width and grid; the counters must never alias earlier partials.
    p, ref = streamk_problem
    for flags in (_lib.FLAG_BN64 | 13, _lib.FLAG_BN128 | 3, _lib.FLAG_BN64 | 7,
                  _lib.FLAG_BN128 | 5 | _lib.FLAG_PAIR,
                  _lib.FLAG_BN128 | 3 | _lib.FLAG_NO_PAIR,
                  _lib.FLAG_BN64 | 10 | _lib.FLAG_PAIR):
        got = run(p, flags | _lib.FLAG_FORCE_STREAMK)
        assert_close(got, ref, f"flags={flags:#x}")


def test_caller_owned_workspace_matches_library_workspace(streamk_problem):
    p, ref = streamk_problem
    flags = 7 | _lib.FLAG_FORCE_STREAMK
    need = dg.workspace_size(256, 512, 2048, flags)
    assert need > 0
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    d = to_device(p)
    for _ in range(2):
        dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                     d["sfb1_blocked"], d["sfb2_blocked"], d["c"],
                     flags=flags | _lib.FLAG_SYNC_CHECK, workspace=ws)
        torch.cuda.synchronize()
        assert_close(d["c"].cpu().numpy(), ref, "caller workspace")
    too_small = torch.zeros(max(need // 2, 256), dtype=torch.uint8,
                            device="cuda")
    with pytest.raises(ValueError, match="workspace"):
        dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                     d["sfb1_blocked"], d["sfb2_blocked"], d["c"],
                     flags=flags, workspace=too_small)


def test_empty_k_gives_zeros():
    a = torch.empty((128, 0), dtype=torch.uint8, device="cuda")
    b = torch.empty((128, 0), dtype=torch.uint8, device="cuda")
    sf = torch.empty((0,), dtype=torch.uint8, device="cuda")
    c = torch.full((128, 128), 7.0, dtype=torch.float16, device="cuda")
    dg.dual_gemm(a, b, b, sf, sf, sf, c)
    torch.cuda.synchronize()
    assert not c.any()


def test_invalid_shapes_raise():
    p = O.make_problem(128, 128, 256, seed=0)
    d = to_device(p)
    with pytest.raises(ValueError):
        dg.dual_gemm(d["a"], d["b1"][:100], d["b2"][:100], d["sfa_blocked"],
                     d["sfb1_blocked"], d["sfb2_blocked"], d["c"][:, :100])
    with pytest.raises(ValueError):
        dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"][:10],
                     d["sfb1_blocked"], d["sfb2_blocked"], d["c"])


def test_device_error_word_clean_after_runs():
    word = torch.zeros(1)  # placeholder to keep the CUDA context alive
    import ctypes
    w = ctypes.c_uint(123)
    rc = _lib.load().nvfp4_dual_gemm_device_status(0, ctypes.byref(w))
    assert rc == 0 and w.value == 0
    del word


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_slices_equal_full_product(world):
    """N-sharding through views (nvfp4_dual_gemm_b200.shard): the column
    slices computed from each rank's B rows and blocked-scale byte range
    equal the full product bit for bit under one whole-tile schedule."""
    from nvfp4_dual_gemm_b200 import shard
    m, n, k = 256, 128 * world * 2, 1024
    p = O.make_problem(m, n, k, seed=50 + world)
    d = to_device(p)
    flags = (_lib.FLAG_BN128 | _lib.FLAG_NO_PAIR | _lib.FLAG_NO_STREAMK |
             _lib.FLAG_NO_SPLITK)
    full = torch.empty(m, n, dtype=torch.float16, device="cuda")
    dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                 d["sfb1_blocked"], d["sfb2_blocked"], full, flags=flags)
    parts = []
    for r in range(world):
        spec = shard.shard_spec(n, k, world, r)
        parts.append(shard.sharded_dual_gemm(
            spec, d["a"], d["b1"], d["b2"], d["sfa_blocked"],
            d["sfb1_blocked"], d["sfb2_blocked"], flags=flags))
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(parts, dim=1), full)
    assert_close(full.cpu().numpy(), O.reference_output(p), "full")


@pytest.mark.parametrize("order", ["adjacent", "b2_far_above", "b2_below"])
@pytest.mark.parametrize("flags", [
    0,
    _lib.FLAG_BN64 | _lib.FLAG_NO_PAIR | _lib.FLAG_NO_SPLITK,
    _lib.FLAG_BN128 | _lib.FLAG_NO_PAIR | _lib.FLAG_NO_SPLITK,
    _lib.FLAG_SPLITK,
    7 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_NO_PAIR,
])
def test_weight_placement_and_merged_copy(order, flags):
    # When B2 lies above B1, one copy brings both weight tiles of a K block
    # through a single map over the two matrices; when it lies below, two
    # copies do.  Both must give the same bits.
    m, n, k = 256, 512, 2048
    p = O.make_problem(m, n, k, seed=123)
    d = to_device(p)
    nb = n * k // 2
    big = torch.zeros(4 * nb, dtype=torch.uint8, device="cuda")
    if order == "adjacent":
        b1, b2 = big[:nb], big[nb:2 * nb]
    elif order == "b2_far_above":
        b1, b2 = big[:nb], big[3 * nb - 4096:4 * nb - 4096]
    else:
        b2, b1 = big[:nb], big[2 * nb + 256:3 * nb + 256]
    b1.copy_(d["b1"].reshape(-1))
    b2.copy_(d["b2"].reshape(-1))
    b1 = b1.view(n, k // 2)
    b2 = b2.view(n, k // 2)
    outs = []
    for extra in (0, _lib.FLAG_NO_MERGED_B):
        d["c"].fill_(float("nan"))
        dg.dual_gemm(d["a"], b1, b2, d["sfa_blocked"], d["sfb1_blocked"],
                     d["sfb2_blocked"], d["c"],
                     flags=flags | extra | _lib.FLAG_SYNC_CHECK)
        torch.cuda.synchronize()
        outs.append(d["c"].cpu().numpy())
    assert np.array_equal(outs[0].view(np.uint16), outs[1].view(np.uint16))
    assert_close(outs[0], O.reference_output(p), f"{order} {flags:#x}")


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("rows,k,pitch", [(300, 1024, 0), (1, 64, 0),
                                          (129, 7168, 0), (77, 512, 640),
                                          (130, 576, 0), (5, 960, 1024)])
def test_activation_quantizer_dtypes_and_pitch(dtype, rows, k, pitch):
    # fp32 / fp16 / bf16 rows (optionally inside a wider row pitch) quantised
    # on the GPU: bit-exact against the oracle applied to the same values
    # widened to fp32; the padding rows of the blocked buffer are zero.
    rng = np.random.default_rng(rows + k)
    x = (rng.standard_normal((rows, max(k, pitch))) *
         rng.choice([1e-3, 1.0, 30.0], size=(rows, 1))).astype(np.float32)
    x[0, :16] = 0.0
    tdt = getattr(torch, dtype)
    xt = torch.from_numpy(x).to(tdt).cuda()[:, :k]
    x32 = xt.float().cpu().numpy()
    codes, sf = O.quantize(x32)
    gc, gsf, gblk = dg.quantize_nvfp4(xt)
    torch.cuda.synchronize()
    assert np.array_equal(gc.cpu().numpy(), codes)
    assert np.array_equal(gsf.view(torch.uint8).cpu().numpy(), sf)
    assert np.array_equal(gblk.cpu().numpy(), O.to_blocked(sf))
    # without the plain scales
    gc2, none, gblk2 = dg.quantize_nvfp4(xt, plain=False)
    torch.cuda.synchronize()
    assert none is None
    assert np.array_equal(gblk2.cpu().numpy(), gblk.cpu().numpy())


def _finite_16bit_values(dtype):
    """Every finite value of a 16-bit float type, as float32 (both zeros)."""
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.int16)
    v = torch.from_numpy(bits).view(getattr(torch, dtype)).float().numpy()
    return v[np.isfinite(v)]


def _every_value_under_every_scale(dtype):
    """Blocks of 16 that put every finite 16-bit v with s/16 <= |v| <= amax
    (and +-0, and a few tiny negatives that round to -0) under every
    positive e4m3 scale s: each block opens with an amax whose scale is s,
    the largest 16-bit value with that scale.  Returns [rows, 1024] float32
    values (exact in the 16-bit type); zero blocks pad the last row."""
    vals = _finite_16bit_values(dtype)
    pos = np.sort(vals[vals > 0])
    with np.errstate(invalid="ignore", over="ignore"):
        pos_sc = O.e4m3_encode(pos / np.float32(6.0))
    blocks = []
    for code in range(1, 0x7F):
        amaxes = pos[pos_sc == code]
        assert len(amaxes), f"no {dtype} amax has e4m3 scale {code:#x}"
        amax = amaxes[-1]
        s = O.e4m3_decode(np.uint8(code))
        mag = np.abs(vals)
        sel = vals[((mag >= s / 16) & (mag <= amax)) | (mag == 0)]
        tiny = -pos[(pos < s / 8)][-4:]
        members = np.concatenate([sel, tiny]).astype(np.float32)
        pad = (-len(members)) % 15
        members = np.concatenate([members, np.zeros(pad, np.float32)])
        body = members.reshape(-1, 15)
        head = np.full((body.shape[0], 1), amax, np.float32)
        blocks.append(np.concatenate([head, body], axis=1))
    x = np.concatenate(blocks).reshape(-1)
    x = np.concatenate([x, np.zeros((-len(x)) % 1024, np.float32)])
    return x.reshape(-1, 1024)


def _check_quantised_rows(x, gc, gsf, gblk):
    codes, sf = O.quantize(x)
    gcodes = gc.cpu().numpy()
    if not np.array_equal(gcodes, codes):
        bad = np.argwhere(gcodes != codes)
        first = bad[:8]
        raise AssertionError(
            f"{len(bad)} code bytes differ, first at {first.tolist()}: "
            f"values {[x[r, 2 * c:2 * c + 2].tolist() for r, c in first]} "
            f"gpu {[hex(gcodes[tuple(b)]) for b in first]} oracle "
            f"{[hex(codes[tuple(b)]) for b in first]}")
    assert np.array_equal(gsf.view(torch.uint8).cpu().numpy(), sf)
    assert np.array_equal(gblk.cpu().numpy(), O.to_blocked(sf))


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_activation_quantizer_every_value_under_every_scale(dtype):
    # The 16-bit encoder replaces v / s by a two-term reciprocal product and
    # the hardware e2m1 conversion; over every finite 16-bit v and every
    # e4m3 scale it can meet (all midpoint ties v = t * s, -0, subnormal
    # scales and values, saturation at 6 included) its codes and scales are
    # bit-exact against the oracle's fp32 division.
    x = _every_value_under_every_scale(dtype)
    xt = torch.from_numpy(x).to(getattr(torch, dtype)).cuda()
    assert np.array_equal(xt.float().cpu().numpy(), x)
    gc, gsf, gblk = dg.quantize_nvfp4(xt)
    torch.cuda.synchronize()
    _check_quantised_rows(x, gc, gsf, gblk)


def test_activation_quantizer_fp32_near_every_midpoint():
    # fp32 rows: values on and a few ulps around every e2m1 midpoint, grid
    # point and fp32 rounding boundary times every positive e4m3 scale s,
    # in blocks opened by the largest fp32 amax whose scale is s (quotients
    # up to ~6.4 saturate); plus blocks of huge and tiny values.  Bit-exact
    # against the oracle's fp32 division.
    rng = np.random.default_rng(23)
    blocks = []
    for code in range(1, 0x7F):
        s = O.e4m3_decode(np.uint8(code)).astype(np.float32)
        amax = np.float32(6 * s * 1.0625)
        while O.e4m3_encode(np.float32(amax / np.float32(6))) != code:
            amax = np.nextafter(amax, np.float32(0))
        v = near_midpoint_fp32(s, rng)
        v = v[np.abs(v) <= amax]
        v = np.concatenate([v, np.zeros((-len(v)) % 15, np.float32)])
        body = v.reshape(-1, 15)
        blocks.append(np.concatenate(
            [np.full((len(body), 1), amax, np.float32), body], axis=1))
    blocks.append(np.array([[3e38, -3e38, 1e30, -1e-30, 1e-45, -0.0] +
                            [2e38] * 10], np.float32))
    blocks.append(np.array([[1e-40, -1e-40, 1e-45, -1e-45] + [0.0] * 12],
                           np.float32))
    x = np.concatenate(blocks).reshape(-1)
    x = np.concatenate([x, np.zeros((-len(x)) % 1024, np.float32)])
    x = x.reshape(-1, 1024)
    gc, gsf, gblk = dg.quantize_nvfp4(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    _check_quantised_rows(x, gc, gsf, gblk)


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_activation_quantizer_many_units_per_warp(dtype):
    # 2001 ragged rows of K = 7104 (seven 1024-element runs, the last one
    # partial) inside a wider pitch: 14,336 units for at most 9,472 warps, so
    # warps step through several (row, run) pairs and the run index wraps
    # into the next row; bit-exact against the oracle.
    rng = np.random.default_rng(41)
    rows, k, pitch = 2001, 7104, 7168
    x = (rng.standard_normal((rows, pitch)) *
         rng.choice([1e-3, 1.0, 40.0], size=(rows, 1))).astype(np.float32)
    xt = torch.from_numpy(x).to(getattr(torch, dtype)).cuda()[:, :k]
    x32 = xt.float().cpu().numpy()
    gc, gsf, gblk = dg.quantize_nvfp4(xt)
    torch.cuda.synchronize()
    _check_quantised_rows(x32, gc, gsf, gblk)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
def test_activation_quantizer_nan_elements(dtype):
    # A NaN element takes no part in its block's scale and encodes as a zero
    # carrying the NaN's sign bit; the block's other elements and all other
    # blocks are encoded as if the NaN were 0.
    rng = np.random.default_rng(17)
    x = rng.standard_normal((256, 1024)).astype(np.float32)
    x[::3, 5] = np.nan
    x[1::5, 40:43] = -np.nan
    xt = torch.from_numpy(x).to(getattr(torch, dtype)).cuda()
    ints = torch.int32 if dtype == "float32" else torch.int16
    raw = xt.view(ints).cpu().numpy()
    isnan = torch.isnan(xt).cpu().numpy()
    clean = np.where(isnan, np.float32(0), xt.float().cpu().numpy())
    codes, sf = O.quantize(clean)
    want = O.unpack_codes(codes)
    want[isnan] = np.where(raw[isnan] < 0, 8, 0)
    gc, gsf, gblk = dg.quantize_nvfp4(xt)
    torch.cuda.synchronize()
    assert np.array_equal(O.unpack_codes(gc.cpu().numpy()), want)
    assert np.array_equal(gsf.view(torch.uint8).cpu().numpy(), sf)
    assert np.array_equal(gblk.cpu().numpy(), O.to_blocked(sf))


@pytest.mark.parametrize("rows,k,pitch", [(300, 1024, 0), (1, 64, 0),
                                          (128, 7168, 0), (129, 4160, 0),
                                          (77, 512, 48)])
def test_scale_layout_converter(rows, k, pitch):
    # plain -> blocked and back on the device, against the oracle's layout
    # functions; a pitched plain buffer (a slice of wider rows) included
    rng = np.random.default_rng(rows * 7 + k)
    kb = k // 16
    wide = rng.integers(0, 256, size=(rows, max(kb, pitch)), dtype=np.uint8)
    sf = torch.from_numpy(wide).cuda()[:, :kb]
    blk = dg.scales_to_blocked(sf)
    torch.cuda.synchronize()
    want = O.to_blocked(wide[:, :kb])
    assert np.array_equal(blk.cpu().numpy(), want)
    back = dg.scales_from_blocked(blk, rows, k)
    torch.cuda.synchronize()
    assert np.array_equal(back.cpu().numpy(), wide[:, :kb])


@pytest.mark.parametrize("flags", [
    0,
    _lib.FLAG_SPLITK | _lib.FLAG_PAIR | _lib.FLAG_BN128,
    _lib.FLAG_SPLITK | _lib.FLAG_NO_PAIR | _lib.FLAG_BN64,
    _lib.FLAG_NO_PAIR | _lib.FLAG_NO_STREAMK | _lib.FLAG_BN128,
    5 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_PAIR | _lib.FLAG_BN128,
])
def test_static_weights_back_to_back(flags):
    # Weight copies issued before the dependency wait: several calls with
    # the same weights and different activations, queued back to back with
    # no synchronisation between them, each checked against the oracle.
    base = O.make_problem(256, 512, 2048, seed=31)
    d = to_device(base)
    flags |= _lib.FLAG_STATIC_WEIGHTS
    outs, refs = [], []
    for i in range(3):
        p = O.make_problem(256, 512, 2048, seed=40 + i)
        q = dict(base, a=p["a"], sfa=p["sfa"], sfa_blocked=p["sfa_blocked"])
        a = torch.from_numpy(q["a"]).cuda()
        sfa = torch.from_numpy(q["sfa_blocked"]).cuda()
        c = torch.full((256, 512), float("nan"), dtype=torch.float16,
                       device="cuda")
        dg.dual_gemm(a, d["b1"], d["b2"], sfa, d["sfb1_blocked"],
                     d["sfb2_blocked"], c, flags=flags)
        outs.append(c)
        refs.append(O.reference_output(q))
    torch.cuda.synchronize()
    for i, (c, ref) in enumerate(zip(outs, refs)):
        assert_close(c.cpu().numpy(), ref, f"call {i} flags {flags:#x}")
    import ctypes
    word = ctypes.c_uint(123)
    rc = _lib.load().nvfp4_dual_gemm_device_status(0, ctypes.byref(word))
    assert rc == 0 and word.value == 0  # no bounded wait expired


# Whole 2-SM pair tiles of 128 columns store fp16 C through shared memory
# and TMA by default; NVFP4DG_FLAG_NO_TMA_STORE keeps the row-by-row stores.
# Both against the oracle, with rows past M (the store boxes are clipped by
# the tensor map, or skipped when a CTA's rows all lie past M), several
# tiles per CTA (the boxes reused after their previous store has read them)
# and a forced stream-K grid (tiles split along K keep row stores).
@pytest.mark.parametrize("m,n,k", [(256, 512, 2048), (300, 768, 1024),
                                   (129, 256, 512), (100, 256, 512),
                                   (1024, 1024, 1024)])
@pytest.mark.parametrize("extra", [0, _lib.FLAG_NO_TMA_STORE, 3,
                                   6 | _lib.FLAG_FORCE_STREAMK])
def test_pair_tile_c_store_paths(m, n, k, extra):
    p = O.make_problem(m, n, k, seed=61)
    flags = _lib.FLAG_PAIR | _lib.FLAG_BN128 | _lib.FLAG_NO_SPLITK | extra
    if not extra & _lib.FLAG_FORCE_STREAMK:
        flags |= _lib.FLAG_NO_STREAMK
    got = run(p, flags)
    assert_close(got, O.reference_output(p), f"flags {flags:#x}")
