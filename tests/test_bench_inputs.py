"""The benchmark's input generator (plain torch, bench.py) against the
oracle's quantiser and blocked layout, on CPU: both arms of bench.py time
the bytes this generator makes, so they must be the BASELINE recipe's."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import bench
from oracle import nvfp4_oracle as O


def _tie_blocks() -> np.ndarray:
    """Blocks whose scale is exact and whose values sit on every e2m1
    midpoint (ties), on grid points, at +-0 and past the saturation point."""
    rows = []
    for s in (1.0, 0.5, 2.0 ** -6, 0.015625 * 1.125, 3.5):
        amax = 6.0 * s
        mids = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0]
        grid = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0]
        v = [amax] + [m * s for m in mids] + [g * s for g in grid] + [-amax]
        rows.append(np.array(v, np.float32))
        rows.append(-np.array(v, np.float32))
    rows.append(np.zeros(16, np.float32))
    rows.append(np.array([-0.0] * 8 + [1e-12] * 8, np.float32))
    return np.stack(rows).reshape(-1, 32)  # 12 blocks: 6 rows of 2 blocks


@pytest.mark.parametrize("seed", [0, 1])
def test_torch_quantiser_equals_oracle(seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((96, 512)) *
         rng.choice([1e-4, 0.02, 0.5, 1.0, 300.0], size=(96, 1))
         ).astype(np.float32)
    x[:6, :32] = _tie_blocks()
    codes_t, sf_t = bench.nvfp4_quantize_torch(torch.from_numpy(x))
    codes_o, sf_o = O.quantize(x)
    assert np.array_equal(sf_t.numpy(), sf_o)
    assert np.array_equal(codes_t.numpy(), codes_o)


def test_torch_quantiser_ties_and_signs():
    x = _tie_blocks()
    codes_t, sf_t = bench.nvfp4_quantize_torch(torch.from_numpy(x))
    codes_o, sf_o = O.quantize(x)
    assert np.array_equal(sf_t.numpy(), sf_o)
    assert np.array_equal(codes_t.numpy(), codes_o)


@pytest.mark.parametrize("rows,k", [(128, 256), (300, 1024), (5, 64)])
def test_blocked_layout_equals_oracle(rows, k):
    rng = np.random.default_rng(rows)
    sf = rng.integers(0, 127, size=(rows, k // 16), dtype=np.uint8)
    got = bench.blocked_torch(torch.from_numpy(sf)).numpy()
    assert np.array_equal(got, O.to_blocked(sf))


def test_make_data_tuple_and_shard_slices():
    m, n, k = 128, 512, 256
    d = bench.make_data(m, n, k, seed=3, a_scale=0.5, w_scale=0.02,
                        device="cpu")
    assert d[0].dtype == torch.float4_e2m1fn_x2 and d[0].shape == (m, k // 2, 1)
    assert d[3].dtype == torch.float8_e4m3fn and d[4].shape == (n, k // 16, 1)
    assert d[9].dtype == torch.float16 and d[9].shape == (m, n, 1)
    for plain, blk in ((d[3], d[6]), (d[4], d[7]), (d[5], d[8])):
        sf = plain.view(torch.uint8).squeeze(-1).numpy()
        assert np.array_equal(blk.view(torch.uint8).numpy(), O.to_blocked(sf))
    world = 4
    for r in range(world):
        s = bench.shard_data(d, n, k, world, r)
        rows = n // world
        b1 = s[1].view(torch.uint8).squeeze(-1).numpy()
        assert np.array_equal(
            b1, d[1].view(torch.uint8).squeeze(-1).numpy()[r * rows:
                                                           (r + 1) * rows])
        sf1 = d[4].view(torch.uint8).squeeze(-1).numpy()[r * rows:
                                                          (r + 1) * rows]
        assert np.array_equal(s[7].view(torch.uint8).numpy(),
                              O.to_blocked(sf1))
        assert s[9].shape == (m, rows, 1)


def test_geomean_and_roofline_arithmetic():
    assert bench.geomean([2.0, 8.0]) == pytest.approx(4.0)
    peaks = {"hbm_gbs": 6000.0, "bf16_tflops": 1500.0,
             "bf16_tflops_sustained": 1400.0, "source": "test"}
    r = bench.roofline(256, 4096, 7168, 10.0, peaks, "c2")
    assert r["bound"] == "hbm"
    assert r["frac"] == pytest.approx(
        bench.algo_bytes(256, 4096, 7168) / 10e-6 / 6000e9, rel=1e-3)
    r = bench.roofline(4096, 14336, 4096, 200.0, peaks, "c4")
    assert r["bound"] == "tensor"
    assert r["peak"] == 6000.0
