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
