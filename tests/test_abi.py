"""CPU tests of the C ABI library: it loads without a GPU, exports every
symbol the header declares, validates arguments without touching the GPU,
and its host-side scheduler covers every K block of every tile exactly once."""
import ctypes
import os
import re
from collections import defaultdict

import pytest

import nvfp4_dual_gemm_b200 as dg
from nvfp4_dual_gemm_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "nvfp4_dual_gemm.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"NVFP4DG_API\s+[\w\s\*]*?\b(nvfp4_\w+)\s*\(",
                                 text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 9
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)
    assert lib.nvfp4_dual_gemm_version() == 101


def test_invalid_arguments_rejected_without_gpu():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    # N not a multiple of 64
    rc = lib.nvfp4_dual_gemm_run(p, p, p, p, p, p, p, 128, 100, 256, 1, 0, None)
    assert rc == _lib.ERR_INVALID and "multiple of 64" in _lib.last_error()
    # K not a multiple of 256
    rc = lib.nvfp4_dual_gemm_run(p, p, p, p, p, p, p, 128, 128, 100, 1, 0, None)
    assert rc == _lib.ERR_INVALID
    # L < 1; batched problems (L > 1) only through the main entry points
    rc = lib.nvfp4_dual_gemm_run(p, p, p, p, p, p, p, 128, 128, 256, 0, 0, None)
    assert rc == _lib.ERR_INVALID and "L must be >= 1" in _lib.last_error()
    rc = lib.nvfp4_dual_gemm_run_noalloc(p, p, p, p, p, p, p, 128, 128, 256, 2,
                                         0, None)
    assert rc == _lib.ERR_INVALID and "L must be 1" in _lib.last_error()
    # misaligned pointer
    q = ctypes.c_void_p(24)
    rc = lib.nvfp4_dual_gemm_run(q, p, p, p, p, p, p, 128, 128, 256, 1, 0, None)
    assert rc == _lib.ERR_ALIGN
    # NULL pointer
    rc = lib.nvfp4_dual_gemm_run(None, p, p, p, p, p, p, 128, 128, 256, 1, 0,
                                 None)
    assert rc == _lib.ERR_INVALID and "NULL" in _lib.last_error()
    # empty problems are a no-op that never touches the GPU
    assert lib.nvfp4_dual_gemm_run(None, None, None, None, None, None, None,
                                   0, 128, 256, 1, 0, None) == _lib.OK
    assert lib.nvfp4_dual_gemm_run(None, None, None, None, None, None, None,
                                   128, 0, 256, 1, 0, None) == _lib.OK
    # quantiser argument checks
    assert lib.nvfp4_quantize(None, 4, 100, None, None, None, None) == \
        _lib.ERR_INVALID


def test_status_check_raises_python_errors():
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_INVALID, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_DEVICE, "x")
    _lib.check(_lib.OK, "x")


SHAPES = [
    (128, 256, 256), (256, 4096, 7168), (512, 3072, 7168), (4096, 14336, 4096),
    (8192, 3584, 8192), (1536, 512, 7168), (256, 512, 256), (3072, 1024, 1536),
    (7168, 1024, 256), (7168, 2304, 2048), (4608, 384, 7168),
    (7168, 384, 2304), (512, 768, 7168), (4096, 768, 512), (200, 192, 768),
]


def cover(m, n, k, flags=0, sms=148):
    pl = dg.plan(m, n, k, flags, sms)
    bn = pl["bn"]
    m_tiles = (m + 128 * pl["ctas"] - 1) // (128 * pl["ctas"])
    tiles = m_tiles * (n // bn)
    kb = k // 256
    seen = defaultdict(list)
    slots = set()
    split = pl["split"] == 2
    for cta in range(pl["grid"]):
        recs = dg.plan_work(m, n, k, cta, flags, sms)
        if split:  # one record per CTA: tile cta // 2, K half cta % 2
            assert len(recs) == 1 and recs[0][0] == cta // 2
        for tile, k0, k1, slot in recs:
            assert 0 <= tile < tiles and 0 <= k0 < k1 <= kb
            seen[tile].append((k0, k1, slot, cta))
            if slot >= 0:
                assert slot // 2 == cta and slot not in slots
                slots.add(slot)
            elif not split:
                assert (k0, k1) == (0, kb)
    assert sorted(seen) == list(range(tiles))
    for tile, segs in seen.items():
        segs.sort()
        # segments tile K exactly once, in order
        assert segs[0][0] == 0 and segs[-1][1] == kb
        for a, b in zip(segs, segs[1:]):
            assert a[1] == b[0]
        if split:
            assert len(segs) == 2 and [s[3] % 2 for s in segs] == [0, 1]
        elif len(segs) > 1:
            assert all(s[2] >= 0 for s in segs)
            assert tile >= pl["dp_tiles"]
    return pl, seen


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_schedule_covers_every_block_once(m, n, k):
    cover(m, n, k)


@pytest.mark.parametrize("grid", [1, 2, 3, 5, 6, 7, 10, 13, 14, 148])
@pytest.mark.parametrize("force", [0, dg.FLAG_FORCE_STREAMK])
@pytest.mark.parametrize("pair", [dg.FLAG_PAIR, dg.FLAG_NO_PAIR])
def test_forced_grid_stream_k(grid, force, pair):
    pl, seen = cover(256, 512, 2048, flags=grid | force | pair)
    assert pl["grid"] * pl["ctas"] <= max(grid, 2)
    # 256 x 512 has 8 or 16 single-CTA tiles and 4 or 8 pair tiles, so these
    # grids (in CTAs) cannot cover them in whole tiles
    splits = (3, 5, 7) if pair == dg.FLAG_NO_PAIR else (6, 10, 14)
    if force and grid in splits:
        assert pl["sk_tiles"] > 0
        assert any(len(s) > 1 for s in seen.values())


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("pair", [dg.FLAG_PAIR, dg.FLAG_NO_PAIR])
def test_schedule_forced_stream_k_covers_every_block_once(m, n, k, pair):
    pl, _ = cover(m, n, k, flags=dg.FLAG_FORCE_STREAMK | pair)
    assert pl["ctas"] == (2 if pair == dg.FLAG_PAIR else 1)


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("pair", [dg.FLAG_PAIR, dg.FLAG_NO_PAIR])
def test_schedule_pair_modes_cover_every_block_once(m, n, k, pair):
    cover(m, n, k, flags=pair)


def test_workspace_counters_fit_for_every_plan():
    # counters live in a fixed 64 KiB region: (tiles split along K) x (CTAs
    # per unit) must stay below 16384 for every grid the flags allow
    for grid in (1, 7, 148, 4095):
        for pair in (dg.FLAG_PAIR, dg.FLAG_NO_PAIR):
            pl = dg.plan(8192, 28672, 8192, grid | pair | dg.FLAG_FORCE_STREAMK)
            assert pl["sk_tiles"] * pl["ctas"] <= 16384


def test_no_streamk_flag_gives_whole_tiles():
    pl, seen = cover(512, 3072, 7168, flags=dg.FLAG_NO_STREAMK)
    assert pl["sk_tiles"] == 0
    assert all(len(s) == 1 for s in seen.values())


def test_bn_flags():
    assert dg.plan(256, 4096, 7168, dg.FLAG_BN64)["bn"] == 64
    assert dg.plan(256, 4096, 7168, dg.FLAG_BN128)["bn"] == 128
    assert dg.plan(256, 192, 7168)["bn"] == 64  # N % 128 != 0


def test_decode_shape_uses_every_sm_or_whole_tiles():
    pl = dg.plan(256, 4096, 7168)
    assert pl["grid"] * pl["ctas"] <= 148


@pytest.mark.parametrize("m,n,k", [(256, 4096, 7168), (256, 512, 2048),
                                   (200, 256, 768), (333, 192, 1024),
                                   (128, 64, 512)])
def test_cluster_split_k_covers_every_block_once(m, n, k):
    pl, seen = cover(m, n, k, flags=dg.FLAG_SPLITK)
    assert pl["split"] == 2 and pl["ctas"] == 1 and pl["sk_tiles"] == 0
    assert pl["grid"] == 2 * len(seen) <= 148
    h = (k // 256 + 1) // 2
    for segs in seen.values():
        assert [(a, b) for a, b, _, _ in sorted(segs)] == [(0, h), (h, k // 256)]


@pytest.mark.parametrize("m,n,k", [(256, 4096, 7168), (256, 512, 2048),
                                   (200, 256, 768), (333, 192, 1024),
                                   (128, 64, 512), (512, 2048, 1024)])
def test_pair_cluster_split_k_covers_every_block_once(m, n, k):
    # 2-SM pairs in clusters of four: unit 2t + h is pair h of tile t
    pl, seen = cover(m, n, k, flags=dg.FLAG_SPLITK | dg.FLAG_PAIR)
    assert pl["split"] == 2 and pl["ctas"] == 2 and pl["sk_tiles"] == 0
    assert pl["grid"] == 2 * len(seen) and 2 * pl["grid"] <= 148
    h = (k // 256 + 1) // 2
    for segs in seen.values():
        assert [(a, b) for a, b, _, _ in sorted(segs)] == [(0, h), (h, k // 256)]


def test_cluster_split_k_choice_and_limits():
    # decode shape: 32 pair tiles of 256 x 128 -> 128 CTAs in 32 clusters of
    # four (two 2-SM pairs, one per half of K)
    pl = dg.plan(256, 4096, 7168)
    assert pl["split"] == 2 and pl["bn"] == 128 and pl["ctas"] == 2
    assert pl["grid"] * pl["ctas"] == 128
    assert dg.plan(256, 4096, 7168, dg.FLAG_NO_PAIR)["ctas"] == 1
    assert dg.plan(256, 4096, 7168, dg.FLAG_NO_SPLITK)["split"] == 0
    # too many tiles for 2 CTAs each, or a single K block: not possible
    for shape in ((4096, 14336, 4096), (256, 4096, 256)):
        for extra in (0, dg.FLAG_PAIR):
            with pytest.raises(RuntimeError):
                dg.plan(*shape, dg.FLAG_SPLITK | extra)
        assert dg.plan(*shape)["split"] == 0
    # 384 rows: 3 single-CTA row tiles but 2 pair tiles of 256 (4 SMs each),
    # so 20 column tiles fit single CTAs (120 SMs) but not pairs (160)
    assert dg.plan(384, 2560, 1024, dg.FLAG_SPLITK)["ctas"] == 1
    with pytest.raises(RuntimeError):
        dg.plan(384, 2560, 1024, dg.FLAG_SPLITK | dg.FLAG_PAIR)
    # exclusive flags are rejected before any GPU work
    lib = _lib.load()
    ptr = ctypes.c_void_p(16)
    for bad in (dg.FLAG_NO_SPLITK, dg.FLAG_FORCE_STREAMK):
        rc = lib.nvfp4_dual_gemm_run(ptr, ptr, ptr, ptr, ptr, ptr, ptr, 256,
                                     512, 2048, 1, dg.FLAG_SPLITK | bad, None)
        assert rc == _lib.ERR_INVALID and "SPLITK" in _lib.last_error()


def _blocked(rows, k):
    return ((rows + 127) // 128) * (k // 64) * 512


def _align(x):
    return (x + 255) // 256 * 256


@pytest.mark.parametrize("m,n,k", [(256, 4096, 7168), (200, 320, 512),
                                   (4096, 14336, 4096), (1, 64, 256)])
def test_host_staging_size_holds_every_buffer(m, n, k):
    want = (_align(m * k // 2) + _align(_blocked(m, k)) + 2 * _align(n * k // 2)
            + 2 * _align(_blocked(n, k)) + _align(m * n * 2))
    assert dg.host_staging_size(m, n, k) == want


def test_host_slab_counts():
    lib = _lib.load()
    slabs = lib.nvfp4_dual_gemm_host_slabs
    # automatic: one slab (upload, kernel, download back to back) when C is
    # small next to the weights, several when its download is long enough
    # to hide behind the upload
    assert slabs(256, 4096, 7168, 0) == 1
    assert slabs(128, 7168, 2048, 0) == 1
    assert 3 <= slabs(4096, 14336, 4096, 0) <= 6
    assert 2 <= slabs(1024, 7168, 4096, 0) <= 6
    # requested counts, rounded to whole 128-row groups
    assert slabs(64, 320, 512, 2) == 2    # 256 + 64 rows
    assert slabs(64, 320, 512, 3) == 3
    assert slabs(64, 320, 512, 16) == 3
    assert slabs(64, 1024, 512, 3) == 3   # 384 + 384 + 256
    assert slabs(64, 1024, 512, 17) == 0
    assert slabs(64, 0, 512, 1) == 0


def test_host_entry_rejects_bad_arguments_without_gpu():
    lib = _lib.load()
    h = ctypes.c_void_p(8)  # host buffers may have any alignment
    m, n, k = 256, 512, 1024
    need = lib.nvfp4_dual_gemm_host_staging_size(m, n, k, 1)
    st = ctypes.c_void_p(1 << 20)

    def run(*, m=m, n=n, k=k, slabs=0, staging=st, nbytes=need, a=h):
        return lib.nvfp4_dual_gemm_run_host(a, h, h, h, h, h, h, m, n, k, 1, 0,
                                            slabs, staging, nbytes, None)

    assert run(n=100) == _lib.ERR_INVALID
    assert run(k=100) == _lib.ERR_INVALID
    assert run(slabs=17) == _lib.ERR_INVALID
    assert run(slabs=-1) == _lib.ERR_INVALID
    assert run(a=None) == _lib.ERR_INVALID and "NULL" in _lib.last_error()
    assert run(staging=None) == _lib.ERR_WORKSPACE
    assert run(nbytes=need - 1) == _lib.ERR_WORKSPACE
    assert run(staging=ctypes.c_void_p((1 << 20) + 16)) == _lib.ERR_ALIGN
    assert run(m=0, staging=None, nbytes=0) == _lib.OK
    assert lib.nvfp4_dual_gemm_host_staging_size(m, 100, k, 1) == 0
    with pytest.raises(ValueError):
        dg.host_staging_size(m, 100, k)


def test_host_api_checks_placement():
    import torch
    m, n, k = 128, 128, 256
    a = torch.zeros(m, k // 2, dtype=torch.uint8)
    b = torch.zeros(n, k // 2, dtype=torch.uint8)
    sfa = torch.zeros(_blocked(m, k), dtype=torch.uint8)
    sfb = torch.zeros(_blocked(n, k), dtype=torch.uint8)
    c = torch.zeros(m, n, dtype=torch.float16)
    with pytest.raises(ValueError, match="CPU tensor"):
        dg.dual_gemm_host(a, b, b, sfa, sfb, sfb, c.to("meta"))
    with pytest.raises(ValueError, match="multiple of 64"):
        dg.dual_gemm_host(a, b[:100], b[:100], sfa, sfb, sfb, c)
    with pytest.raises(ValueError, match="CUDA tensor"):
        dg.dual_gemm(a, b, b, sfa, sfb, sfb, c)


SK_CASES = [
    (m, n, k, f)
    for (m, n, k) in [(256, 3072, 4096), (512, 3072, 7168), (1024, 7168, 4096),
                      (4096, 14336, 4096), (384, 1024, 2048), (7168, 384, 2304),
                      (200, 192, 768), (2048, 2048, 2048)]
    for f in (0, _lib.FLAG_FORCE_STREAMK | _lib.FLAG_NO_PAIR,
              _lib.FLAG_FORCE_STREAMK | _lib.FLAG_PAIR,
              _lib.FLAG_FORCE_STREAMK | _lib.FLAG_BN64 | _lib.FLAG_NO_PAIR,
              13 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_NO_PAIR)
]


@pytest.mark.parametrize("m,n,k,flags", SK_CASES)
def test_stream_k_waits_cannot_cycle(m, n, k, flags):
    """The CTA (unit) holding a stream-K tile's first K blocks finishes the
    tile after waiting for the other contributors' partials.  That wait ends
    only if (a) the owner's segment is the owner's last item, (b) every other
    contributor's segment is its first stream-K item (computed before any
    wait of its own), and (c) all units are resident at once."""
    p = dg.plan(m, n, k, flags)
    if p["sk_tiles"] == 0:
        return
    assert p["grid"] * p["ctas"] <= 148
    kblocks = k // 256
    segs = defaultdict(list)
    for u in range(p["grid"]):
        recs = dg.plan_work(m, n, k, u, flags)
        sk = [r for r in recs if r[0] >= p["dp_tiles"]]
        for i, (tile, kb0, kb1, slot) in enumerate(sk):
            segs[tile].append((u, kb0, kb1, i == 0, i == len(sk) - 1, slot))
    for tile, ss in segs.items():
        ss.sort()
        if len(ss) == 1:
            assert ss[0][1:3] == (0, kblocks) and ss[0][5] == -1
            continue
        owner = ss[0]
        assert owner[1] == 0 and owner[4], (tile, ss)       # (a)
        for u, kb0, kb1, first, last, slot in ss[1:]:
            assert first and slot >= 0, (tile, ss)           # (b)
        # the segments tile the K range in unit order
        assert [s[1] for s in ss[1:]] == [s[2] for s in ss[:-1]]
        assert ss[-1][2] == kblocks


@pytest.mark.parametrize("flags", [
    148 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_NO_PAIR | _lib.FLAG_BN128,
    148 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_NO_PAIR | _lib.FLAG_BN64,
    148 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_PAIR | _lib.FLAG_BN128,
])
def test_many_contributor_plans(flags):
    # the plans the GPU test of many stream-K contributors per tile relies on
    m, n, k = 256, 512, 7168
    pl = dg.plan(m, n, k, flags)
    assert pl["grid"] * pl["ctas"] == 148 and pl["dp_tiles"] == 0
    per_tile = defaultdict(int)
    for u in range(pl["grid"]):
        for tile, kb0, kb1, slot in dg.plan_work(m, n, k, u, flags):
            per_tile[tile] += 1
    assert min(per_tile.values()) >= 9, dict(per_tile)


def test_stream_k_small_grid_search():
    # whole-problem stream-K may pick a grid smaller than the SM count
    flags = _lib.FLAG_FORCE_STREAMK | _lib.FLAG_NO_PAIR | _lib.FLAG_BN128
    pl = dg.plan(256, 512, 7168, flags)
    assert pl["sk_tiles"] == 8 and pl["grid"] < 148


def test_tile_division_by_multiply_high():
    # Restatement of set_div / div_by (schedule.h, used by tile_lmn for the
    # row-tile and the column-tile counts): the quotient of every tile index
    # by every divisor the planner can produce.
    import numpy as np
    n = np.arange(1 << 17, dtype=np.uint64)
    for d in list(range(1, 1025)) + [4095, 4096, 8191, 16384]:
        shift = 0
        while (1 << shift) < d:
            shift += 1
        mul = ((1 << 32) * ((1 << shift) - d)) // d + 1
        assert 0 < mul < (1 << 32) or d == 1
        hi = (n * np.uint64(mul)) >> np.uint64(32)
        q = (hi + n) >> np.uint64(shift)
        assert np.array_equal(q, n // np.uint64(d)), d


def test_quantize_rows_rejects_bad_arguments_without_gpu():
    lib = _lib.load()
    p = ctypes.c_void_p(256)
    q = lib.nvfp4_quantize_rows
    assert q(p, 7, 4, 64, 64, p, None, p, None) == _lib.ERR_INVALID   # dtype
    assert q(p, _lib.DTYPE_F16, 4, 100, 100, p, None, p, None) == _lib.ERR_INVALID
    assert q(p, _lib.DTYPE_F16, 4, 64, 32, p, None, p, None) == _lib.ERR_INVALID
    assert q(p, _lib.DTYPE_F16, 4, 64, 68, p, None, p, None) == _lib.ERR_ALIGN
    assert q(ctypes.c_void_p(8), _lib.DTYPE_F32, 4, 64, 64, p, None, p,
             None) == _lib.ERR_ALIGN
    assert q(p, _lib.DTYPE_BF16, 4, 64, 64, None, None, p, None) == \
        _lib.ERR_INVALID
    assert q(None, _lib.DTYPE_F32, 0, 64, 64, None, None, None, None) == _lib.OK


def test_scale_converter_rejects_bad_arguments_without_gpu():
    lib = _lib.load()
    p = ctypes.c_void_p(256)
    to, back = lib.nvfp4_scales_to_blocked, lib.nvfp4_scales_from_blocked
    assert to(p, 4, 100, 8, p, None) == _lib.ERR_INVALID     # K % 64
    assert to(p, 4, 128, 4, p, None) == _lib.ERR_INVALID     # ld < K/16
    assert to(p, 4, 128, 10, p, None) == _lib.ERR_ALIGN      # ld % 4
    assert to(p, 4, 128, 8, ctypes.c_void_p(260), None) == _lib.ERR_ALIGN
    assert back(ctypes.c_void_p(260), 4, 128, p, 8, None) == _lib.ERR_ALIGN
    assert to(None, 4, 128, 8, p, None) == _lib.ERR_INVALID
    assert to(None, 0, 128, 8, None, None) == _lib.OK


def test_grouped_arguments_rejected_without_gpu():
    # nvfp4_dual_gemm_run_grouped validates its group table before any CUDA
    # call: group count, row offsets on 128-row boundaries, no overlap once
    # each group is rounded up to 128 rows, no cluster split-K.
    lib = _lib.load()
    p = ctypes.c_void_p(256)
    run = lib.nvfp4_dual_gemm_run_grouped

    def call(rows, row0, flags=0, n=128, k=256, groups=None):
        g = len(rows) if groups is None else groups
        r = (ctypes.c_int * max(1, len(rows)))(*rows)
        o = (ctypes.c_int * max(1, len(row0)))(*row0)
        return run(p, p, p, p, p, p, p, r, o, g, n, k, flags, None, 0, None)

    assert call([128], [0], groups=0) == _lib.ERR_INVALID
    assert call([1] * 65, [128 * i for i in range(65)]) == _lib.ERR_INVALID
    assert call([128, 64], [0, 100]) == _lib.ERR_INVALID
    assert "multiple of 128" in _lib.last_error()
    assert call([130, 64], [0, 128]) == _lib.ERR_INVALID
    assert "overlaps" in _lib.last_error()
    assert call([-1], [0]) == _lib.ERR_INVALID
    assert call([128], [0], flags=_lib.FLAG_SPLITK) == _lib.ERR_INVALID
    assert "split-K" in _lib.last_error()
    assert call([128], [0], n=100) == _lib.ERR_INVALID
    assert run(p, p, p, p, p, p, p, None, None, 1, 128, 256, 0, None, 0,
               None) == _lib.ERR_INVALID

