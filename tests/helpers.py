"""Shared helpers for the tests: move oracle problems to the GPU and compare."""
from __future__ import annotations

import numpy as np
import torch

from oracle import nvfp4_oracle as O

RTOL = 1e-3  # tolerance on the fp16 output stated by the task definition
ATOL = 1e-3


def to_device(p: dict, device="cuda") -> dict:
    """Upload an oracle problem as the reference's data layout (uint8 views)."""
    d = {}
    for k in ("a", "b1", "b2", "sfa_blocked", "sfb1_blocked", "sfb2_blocked"):
        d[k] = torch.from_numpy(np.ascontiguousarray(p[k])).to(device)
    for k in ("sfa", "sfb1", "sfb2"):
        d[k] = torch.from_numpy(np.ascontiguousarray(p[k])).to(device)
    d["c"] = torch.full((p["M"], p["N"]), float("nan"), dtype=torch.float16,
                        device=device)
    return d


def data_tuple(d: dict):
    """The reference's 10-tuple (submission.py:1154) from device tensors."""
    fp4 = torch.float4_e2m1fn_x2
    f8 = torch.float8_e4m3fn
    return (d["a"].view(fp4).unsqueeze(-1), d["b1"].view(fp4).unsqueeze(-1),
            d["b2"].view(fp4).unsqueeze(-1), d["sfa"].view(f8).unsqueeze(-1),
            d["sfb1"].view(f8).unsqueeze(-1), d["sfb2"].view(f8).unsqueeze(-1),
            d["sfa_blocked"].view(f8), d["sfb1_blocked"].view(f8),
            d["sfb2_blocked"].view(f8), d["c"].unsqueeze(-1))


def assert_close(got: np.ndarray, ref: np.ndarray, what: str = "") -> None:
    ok, n_bad, worst = O.check_close(got, ref, RTOL, ATOL)
    if not ok:
        g = got[worst]
        r = ref[worst]
        raise AssertionError(
            f"{what}: {n_bad} of {got.size} outputs outside rtol=atol=1e-3; "
            f"worst at {worst}: got {g} ref {r}")


def near_midpoint_fp32(s, rng):
    """fp32 values on, and a few ulps around, every e2m1 midpoint and grid
    point times s, around every fp32 rounding boundary (t +- ulp(t)/2) * s,
    and random ones up to 6.4 s, with both signs; plus zeros and tiny and
    huge values."""
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    grid = np.array([0.5, 1, 1.5, 2, 3, 4, 6], np.float32)
    t = np.concatenate([mids, grid])
    ulp = np.spacing(t)
    centres = np.concatenate([t, t + ulp / 2, t - ulp / 2]).astype(
        np.float64) * float(s)
    centres = centres.astype(np.float32)
    steps = np.arange(-3, 4, dtype=np.int64)
    near = (centres.view(np.int32)[:, None] + steps[None, :]).astype(
        np.int32).view(np.float32).ravel()
    rand = (rng.random(64) * 6.4 * s).astype(np.float32)
    v = np.concatenate([near, rand, [0.0, 1e-40, 1e-30, 3e38]]).astype(
        np.float32)
    return np.concatenate([v, -v])
