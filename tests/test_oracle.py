"""CPU tests of the oracle: format tables, rounding, packing, blocked layout,
known-answer dual GEMMs."""
import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O
from tests.helpers import near_midpoint_fp32


def test_e2m1_table_matches_ocp_values():
    # OCP MX v1.0 e2m1: +-{0, 0.5, 1, 1.5, 2, 3, 4, 6}
    assert list(O.E2M1_VALUES[:8]) == [0, 0.5, 1, 1.5, 2, 3, 4, 6]
    assert list(O.E2M1_VALUES[8:]) == [-0.0, -0.5, -1, -1.5, -2, -3, -4, -6]
    assert np.all(np.signbit(O.E2M1_VALUES[8:]))


def test_e2m1_round_to_nearest_even_and_saturation():
    q = np.array([0.0, 0.25, 0.2501, 0.75, 1.25, 1.2501, 1.75, 2.5, 2.5001,
                  3.5, 5.0, 5.0001, 100.0, -0.1, -6.5], np.float32)
    want = [0.0, 0.0, 0.5, 1.0, 1.0, 1.5, 2.0, 2.0, 3.0, 4.0, 4.0, 6.0, 6.0,
            -0.0, -6.0]
    got = O.E2M1_VALUES[O.e2m1_encode(q)]
    assert list(got) == want
    # every grid value maps to itself
    for code in range(16):
        v = O.E2M1_VALUES[code]
        c = O.e2m1_encode(np.array([v], np.float32))[0]
        assert O.E2M1_VALUES[c] == v and np.signbit(O.E2M1_VALUES[c]) == np.signbit(v)


def test_e4m3_decode_table():
    t = O.E4M3_TABLE
    assert t[0x00] == 0 and t[0x01] == 2.0 ** -9 and t[0x08] == 2.0 ** -6
    assert t[0x38] == 1.0 and t[0x7E] == 448.0 and np.isnan(t[0x7F])
    assert t[0xB8] == -1.0


def test_e4m3_encode_matches_torch_cast_in_range():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(100_000).astype(np.float32) * s
                        for s in (1e-3, 1e-2, 0.1, 1.0, 10.0, 100.0)])
    x = x[np.abs(x) <= 448]
    vals = O.E4M3_TABLE[:0x7F]
    mids = ((vals[1:] + vals[:-1]) / 2).astype(np.float32)  # exact ties
    x = np.concatenate([x, vals, mids, -mids])
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(O.e4m3_encode(x), ref)


def test_e4m3_encode_saturates():
    assert O.e4m3_encode(np.array([500.0, -1e9], np.float32)).tolist() == [0x7E, 0xFE]


def test_pack_unpack_nibble_order():
    codes = np.array([[1, 2, 3, 4]], np.uint8)
    packed = O.pack_codes(codes)
    assert packed.tolist() == [[0x21, 0x43]]  # element 2i in the low nibble
    assert np.array_equal(O.unpack_codes(packed), codes)


def test_blocked_layout_matches_reference_addressing():
    # Reference: atom index = rowblock * (K/64) + k64, 512 B per atom
    # (nvfp4_dual_gemm.cu:226-243); within an atom row r%32 owns 16 bytes,
    # 4 per 32-row quadrant.
    rows, k = 256, 512
    off = O.blocked_offsets(rows, k)
    assert off[0, 0] == 0 and off[0, 3] == 3 and off[0, 4] == 512
    assert off[1, 0] == 16 and off[32, 0] == 4 and off[96, 2] == 14
    assert off[128, 0] == (k // 64) * 512
    assert len(np.unique(off)) == off.size


def test_blocked_roundtrip_with_padding():
    rng = np.random.default_rng(1)
    sf = rng.integers(0, 0x7F, (300, 64)).astype(np.uint8)
    buf = O.to_blocked(sf)
    assert buf.size == 3 * 16 * 512
    assert np.array_equal(O.from_blocked(buf, 300, 1024), sf)
    mask = np.ones(buf.size, bool)
    mask[O.blocked_offsets(300, 1024)] = False
    assert not buf[mask].any()  # padding rows are zero


def test_quantize_dequantize_error_bound():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((64, 256)).astype(np.float32)
    codes, sf = O.quantize(x)
    y = O.dequantize(codes, sf)
    blk = np.abs(x).reshape(64, 16, 16).max(axis=2, keepdims=True)
    err = np.abs(x - y).reshape(64, 16, 16)
    # half a grid step of e2m1 (<= 1.0 at the top of the range) times the
    # scale, plus the e4m3 rounding of the scale itself
    assert np.all(err <= blk / 6 * 1.0625 * 1.0 + 1e-6)


def test_zero_block_gives_zero_codes():
    x = np.zeros((1, 64), np.float32)
    x[0, 16:32] = 1e-6  # amax / 6 rounds to 0 in e4m3
    codes, sf = O.quantize(x)
    assert not codes.any() and not sf.any()


def test_one_hot_known_answer():
    # A row i has a single non-zero code at k = i (value 1.0 with scale 1.0),
    # so (A B^T)[i, n] = B[n, i] exactly: checks nibble order and scales.
    m, n, k = 4, 8, 64
    a = np.zeros((m, k), np.float32)
    for i in range(m):
        a[i, 2 * i + 1] = 6.0  # odd K index -> high nibble
    b1 = np.arange(n * k, dtype=np.float32).reshape(n, k) % 7 - 3
    b2 = np.ones((n, k), np.float32) * 2
    qa, sa = O.quantize(a)
    q1, s1 = O.quantize(b1)
    q2, s2 = O.quantize(b2)
    c = O.dual_gemm(qa, sa, q1, s1, q2, s2).astype(np.float32)
    d1 = O.dequantize(q1, s1)
    d2 = O.dequantize(q2, s2)
    da = O.dequantize(qa, sa)
    for i in range(m):
        x1 = da[i, 2 * i + 1] * d1[:, 2 * i + 1]
        x2 = da[i, 2 * i + 1] * d2[:, 2 * i + 1]
        want = (x1 / (1 + np.exp(-x1)) * x2).astype(np.float16).astype(np.float32)
        assert np.array_equal(c[i], want)


def test_reference_output_fp32_vs_fp64_config1():
    p = O.make_problem(128, 256, 256, seed=0)
    c32 = O.reference_output(p)
    c64 = O.reference_output(p, accumulate=np.float64)
    ok, n_bad, _ = O.check_close(c32, c64)
    assert ok, n_bad


def test_sampled_reference_matches_full():
    p = O.make_problem(128, 256, 512, seed=3)
    full = O.reference_output(p)
    rows = np.array([0, 5, 127])
    cols = np.array([1, 64, 255])
    part = O.reference_output(p, rows=rows, cols=cols)
    assert np.array_equal(part, full[np.ix_(rows, cols)])


def test_make_problem_is_deterministic():
    p1 = O.make_problem(128, 128, 256, seed=7)
    p2 = O.make_problem(128, 128, 256, seed=7)
    for key in ("a", "b1", "b2", "sfa", "sfb1", "sfb2"):
        assert np.array_equal(p1[key], p2[key])


@pytest.mark.parametrize("bad", [np.nan])
def test_check_close_rejects_nan(bad):
    ok, n, _ = O.check_close(np.array([bad], np.float16), np.array([1], np.float16))
    assert not ok and n == 1


def _threshold_codes(v, sd):
    """The division-free e2m1 encoding the CUDA quantiser uses
    (quant_block16 in csrc/dual_gemm.cu): locate |v| among the exact
    products t * sd of the grid midpoints by binary search, ties at
    0.75 / 1.75 / 3.5 going up (> the float just below)."""
    v = np.asarray(v, dtype=np.float32)
    sd = np.float32(sd)
    below = lambda x: (np.float32(x).view(np.uint32) - np.uint32(1)).view(
        np.float32)
    ts = [np.float32(0.25) * sd, below(np.float32(0.75) * sd),
          np.float32(1.25) * sd, below(np.float32(1.75) * sd),
          np.float32(2.5) * sd, below(np.float32(3.5) * sd),
          np.float32(5.0) * sd]
    a = np.abs(v)
    assert all(x < y for x, y in zip(ts, ts[1:]))
    # the kernel's three-level binary search over the increasing midpoints
    b2 = a > ts[3]
    b1 = a > np.where(b2, ts[5], ts[1])
    b0 = a > np.where(b2, np.where(b1, ts[6], ts[4]),
                      np.where(b1, ts[2], ts[0]))
    m = (4 * b2 + 2 * b1 + b0).astype(np.uint8)
    return (m | np.where(np.signbit(v), 8, 0)).astype(np.uint8)


def test_division_free_e2m1_encoding_equals_division():
    # For every positive e4m3 scale: values on and around each midpoint
    # t * sd (a few float32 steps either side), around the grid points, and
    # random fp16-representable values (the fused epilogue quantises fp16
    # results), signed.  The kernel's comparison form must give the code of
    # e2m1(RN(v / sd)) exactly.
    rng = np.random.default_rng(0)
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    grid = O.E2M1_VALUES[:8]
    for b in range(1, 0x7F):
        sd = O.e4m3_decode(np.uint8(b))
        centres = np.concatenate([mids, grid, [6.0, 7.0, 100.0]]) * sd
        steps = np.arange(-4, 5, dtype=np.int64)
        near = (centres.astype(np.float32).view(np.int32)[:, None] +
                steps[None, :]).astype(np.int32).view(np.float32).ravel()
        rand = (rng.standard_normal(512).astype(np.float32) * 3 * sd)
        rand = rand.astype(np.float16).astype(np.float32)
        v = np.concatenate([near, rand, [0.0, np.inf]]).astype(np.float32)
        v = np.concatenate([v, -v])
        with np.errstate(over="ignore", invalid="ignore"):
            want = O.e2m1_encode(v / sd)
        got = _threshold_codes(v, sd)
        bad = np.flatnonzero(got != want)
        assert bad.size == 0, (b, v[bad[:4]], got[bad[:4]], want[bad[:4]])


def _bf16(x):
    """float32 -> the bf16 values (round to nearest even) as float32."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return (u.astype(np.uint32) << 16).view(np.float32)


def test_packed_16bit_e2m1_encoding_equals_division():
    # The compare form for fp16 / bf16 data (quant_block16_x2_cmp: the
    # NVFP4-output epilogue, and blocks holding a NaN in the quantiser):
    # the midpoint products t * s rounded to the 16-bit type (exact: at most
    # 7 significant bits, within range) and compared with |v| as 16-bit
    # values, the >= midpoints as > the 16-bit value just below.  Every fp16
    # value and a spread of bf16 values, for every positive e4m3 scale.
    h16 = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    h16 = h16[~np.isnan(h16)]
    rng = np.random.default_rng(2)
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    for b in range(1, 0x7F):
        sd = O.e4m3_decode(np.uint8(b)).astype(np.float32)
        for kind in ("f16", "bf16"):
            if kind == "f16":
                v = h16.astype(np.float32)
                t = (mids * sd).astype(np.float16)
                assert np.array_equal(t.astype(np.float32), mids * sd)
                below = (t.view(np.uint16) - 1).view(np.float16).astype(
                    np.float32)
                t = t.astype(np.float32)
            else:
                v = _bf16(np.concatenate([
                    rng.standard_normal(20000).astype(np.float32) * 3 * sd,
                    mids * sd, [0.0, np.inf]]).astype(np.float32))
                t = _bf16(mids * sd)
                assert np.array_equal(t, mids * sd)
                below = ((t.view(np.uint32) >> 16) - 1).astype(
                    np.uint32) << 16
                below = below.view(np.float32)
            ts = [t[0], below[1], t[2], below[3], t[4], below[5], t[6]]
            v = np.concatenate([v, -v]).astype(np.float32)
            a = np.abs(v)
            b2 = a > ts[3]
            b1 = a > np.where(b2, ts[5], ts[1])
            b0 = a > np.where(b2, np.where(b1, ts[6], ts[4]),
                              np.where(b1, ts[2], ts[0]))
            got = ((4 * b2 + 2 * b1 + b0) |
                   np.where(np.signbit(v), 8, 0)).astype(np.uint8)
            with np.errstate(over="ignore", invalid="ignore"):
                want = O.e2m1_encode(v / sd)
            bad = np.flatnonzero(got != want)
            assert bad.size == 0, (b, kind, v[bad[:4]])


@pytest.mark.skipif(np.finfo(np.longdouble).nmant < 63,
                    reason="needs an 80-bit long double to model the fma")
def test_reciprocal_product_e2m1_encoding_equals_division():
    # The activation quantiser's form for fp16 / bf16 rows
    # (quant_block16_x2): q = v * rh + RN(v * rl) rounded once (fma), with
    # rh = 1/s rounded toward zero and rl = RN(RN(1 - s * rh) * rh), then
    # e2m1 round-to-nearest-even.  The fma's single rounding is modelled in
    # 80-bit long double (exact: the sum spans fewer than 64 bits).  Every
    # finite fp16 and bf16 value, signed zeros included, under every
    # positive e4m3 scale.
    L = np.longdouble
    bits = np.arange(65536, dtype=np.uint32)
    bf16 = (bits << 16).view(np.float32)
    f16 = bits.astype(np.uint16).view(np.float16).astype(np.float32)
    for kind, vals in (("bf16", bf16), ("f16", f16)):
        v = vals[np.isfinite(vals)]
        vl = v.astype(L)
        for b in range(1, 0x7F):
            s = O.e4m3_decode(np.uint8(b)).astype(np.float32)
            rh = np.float32(np.float32(1) / s)
            if L(rh) * L(s) > 1:  # round toward zero
                rh = np.nextafter(rh, np.float32(0))
            rl = np.float32(np.float32(L(1) - L(s) * L(rh)) * rh)
            assert rl >= 0
            with np.errstate(over="ignore"):
                p = (v * rl).astype(np.float32)
                q = (vl * L(rh) + p.astype(L)).astype(np.float32)
                want = O.e2m1_encode((v / s).astype(np.float32))
            got = O.e2m1_encode(q)
            bad = np.flatnonzero(got != want)
            assert bad.size == 0, (kind, b, v[bad[:4]], q[bad[:4]])


def _rn_f32(fr):
    """A Fraction rounded once to the nearest float32 (ties to even),
    overflowing to +-inf; returns a Python float holding that value."""
    from fractions import Fraction
    if fr == 0:
        return 0.0
    sign = -1.0 if fr < 0 else 1.0
    a = abs(fr)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if Fraction(2) ** e > a:
        e -= 1
    e = max(e, -126) - 23          # ulp exponent (subnormals: 2^-149)
    scaled = a / Fraction(2) ** e
    m, rem = divmod(scaled.numerator, scaled.denominator)
    if 2 * rem > scaled.denominator or (2 * rem == scaled.denominator and
                                        m & 1):
        m += 1
    if m * 2.0 ** e > 3.4028234663852886e38:
        return sign * float("inf")
    return sign * m * 2.0 ** e


def test_reciprocal_product_e2m1_encoding_fp32():
    # The same form for fp32 rows (quant_block16_rcp), with the fma's single
    # rounding modelled exactly (fractions): values on and around every
    # midpoint, grid point and fp32 rounding boundary times s, under every
    # positive e4m3 scale, give the codes of e2m1(RN(v / s)).
    from fractions import Fraction
    rng = np.random.default_rng(9)
    for b in range(1, 0x7F):
        s = O.e4m3_decode(np.uint8(b)).astype(np.float32)
        rh = np.float32(np.float32(1) / s)
        if Fraction(float(rh)) * Fraction(float(s)) > 1:
            rh = np.nextafter(rh, np.float32(0))
        e = np.float32(_rn_f32(1 - Fraction(float(s)) * Fraction(float(rh))))
        rl = np.float32(_rn_f32(Fraction(float(e)) * Fraction(float(rh))))
        v = near_midpoint_fp32(s, rng)
        q = np.array([_rn_f32(Fraction(float(x)) * Fraction(float(rh)) +
                              Fraction(_rn_f32(Fraction(float(x)) *
                                               Fraction(float(rl)))))
                      for x in v], np.float32)
        # v = +-0: v * rh has v's sign, RN(v * rl) v's sign times rl's, and
        # their sum is -0 only when both are -0 (IEEE round to nearest)
        neg0 = np.signbit(v) & ~np.signbit(rl)
        q = np.where(v == 0, np.where(neg0, np.float32(-0.0), 0), q)
        with np.errstate(over="ignore"):
            want = O.e2m1_encode((v / s).astype(np.float32))
        got = O.e2m1_encode(q)
        bad = np.flatnonzero(got != want)
        assert bad.size == 0, (b, v[bad[:4]], q[bad[:4]])
