"""GPU tests of grouped problems (``nvfp4_dual_gemm_run_grouped``): experts
of a mixture-of-experts FFN with their own token counts in one launch.

Group g's rows of C are compared with the oracle's product of the same rows
of A and expert g's weights within rtol = atol = 1e-3; rows outside every
group must stay untouched.  Covered: empty groups, groups shorter than a
tile, groups spanning several tiles, 2-SM pair and single-CTA tiles, whole
tiles and stream-K, and the argument checks.
"""
import numpy as np
import pytest
import torch

import nvfp4_dual_gemm_b200 as dg
from nvfp4_dual_gemm_b200 import _lib
from oracle import nvfp4_oracle as O
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu

PATHS = {
    "auto": 0,
    "pair_bn128": _lib.FLAG_PAIR | _lib.FLAG_BN128 | _lib.FLAG_NO_STREAMK,
    "1sm_bn64": _lib.FLAG_NO_PAIR | _lib.FLAG_BN64 | _lib.FLAG_NO_STREAMK,
    "streamk_pair": 5 | _lib.FLAG_PAIR | _lib.FLAG_BN64 |
    _lib.FLAG_FORCE_STREAMK,
    "streamk_1sm": 7 | _lib.FLAG_NO_PAIR | _lib.FLAG_BN128 |
    _lib.FLAG_FORCE_STREAMK,
    "static_weights": _lib.FLAG_STATIC_WEIGHTS,
}


def grouped_problem(rows, n, k, seed):
    row0 = dg.group_offsets(rows)
    R = max([r + m for r, m in zip(row0, rows) if m > 0])
    pa = O.make_problem(R, 64, k, seed=seed)  # A rows (its B is unused)
    experts = [O.make_problem(64, n, k, seed=seed + 1 + g)
               for g in range(len(rows))]

    def stack(key):
        return torch.from_numpy(np.stack([e[key] for e in experts])).cuda() \
            .permute(1, 2, 0)

    def cat(key):
        return torch.from_numpy(np.concatenate(
            [e[key] for e in experts])).cuda()

    d = {"a": torch.from_numpy(pa["a"]).cuda(),
         "sfa": torch.from_numpy(pa["sfa_blocked"]).cuda(),
         "b1": stack("b1"), "b2": stack("b2"),
         "sfb1": cat("sfb1_blocked"), "sfb2": cat("sfb2_blocked"),
         "c": torch.full((R, n), float("nan"), dtype=torch.float16,
                         device="cuda")}
    refs = []
    for g, (r0, m) in enumerate(zip(row0, rows)):
        e = experts[g]
        rs = slice(r0, r0 + m)
        refs.append(O.dual_gemm(pa["a"][rs], pa["sfa"][rs], e["b1"],
                                e["sfb1"], e["b2"], e["sfb2"]) if m else None)
    return d, row0, refs


@pytest.mark.parametrize("path", list(PATHS))
@pytest.mark.parametrize("rows,n,k", [([0, 37, 128, 300, 5], 256, 1024),
                                      ([256, 1, 0, 200], 384, 512)])
def test_grouped_matches_each_group(path, rows, n, k):
    flags = PATHS[path]
    if flags & _lib.FLAG_BN128 and n % 128:
        pytest.skip("BN = 128 needs N % 128 == 0")
    d, row0, refs = grouped_problem(rows, n, k, seed=sum(rows) + n)
    dg.dual_gemm_grouped(d["a"], d["b1"], d["b2"], d["sfa"], d["sfb1"],
                         d["sfb2"], d["c"], rows,
                         flags=flags | _lib.FLAG_SYNC_CHECK)
    torch.cuda.synchronize()
    c = d["c"].cpu().numpy()
    covered = np.zeros(c.shape[0], bool)
    for g, (r0, m) in enumerate(zip(row0, rows)):
        if m:
            assert_close(c[r0:r0 + m], refs[g], f"{path} group {g}")
            covered[r0:r0 + m] = True
    assert np.isnan(c[~covered]).all(), "rows outside the groups were written"


@pytest.mark.parametrize("flags", [
    0, 5 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_PAIR | _lib.FLAG_BN64])
def test_grouped_twice_and_custom_offsets(flags):
    # explicit offsets with gaps between groups; two calls in a row, the
    # second with a caller-owned workspace
    rows = [130, 64]
    row0 = [128, 512]
    R = 576
    pa = O.make_problem(R, 64, 768, seed=3)
    experts = [O.make_problem(64, 128, 768, seed=4 + g) for g in range(2)]
    a = torch.from_numpy(pa["a"]).cuda()
    sfa = torch.from_numpy(pa["sfa_blocked"]).cuda()
    b1 = torch.from_numpy(np.stack([e["b1"] for e in experts])).cuda() \
        .permute(1, 2, 0)
    b2 = torch.from_numpy(np.stack([e["b2"] for e in experts])).cuda() \
        .permute(1, 2, 0)
    sfb1 = torch.from_numpy(np.concatenate(
        [e["sfb1_blocked"] for e in experts])).cuda()
    sfb2 = torch.from_numpy(np.concatenate(
        [e["sfb2_blocked"] for e in experts])).cuda()
    ws = torch.zeros(max(dg.grouped_workspace_size(rows, 128, 768, flags),
                         256), dtype=torch.uint8, device="cuda")
    for call in range(2):
        c = torch.full((R, 128), float("nan"), dtype=torch.float16,
                       device="cuda")
        dg.dual_gemm_grouped(a, b1, b2, sfa, sfb1, sfb2, c, rows, row0,
                             flags=flags | _lib.FLAG_SYNC_CHECK,
                             workspace=ws if call else None)
        torch.cuda.synchronize()
        h = c.cpu().numpy()
        for g in range(2):
            rs = slice(row0[g], row0[g] + rows[g])
            e = experts[g]
            ref = O.dual_gemm(pa["a"][rs], pa["sfa"][rs], e["b1"], e["sfb1"],
                              e["b2"], e["sfb2"])
            assert_close(h[rs], ref, f"group {g}")
        assert np.isnan(h[:128]).all() and np.isnan(h[258:512]).all()


def test_grouped_argument_errors():
    d, row0, _ = grouped_problem([128, 64], 128, 256, seed=9)
    args = (d["a"], d["b1"], d["b2"], d["sfa"], d["sfb1"], d["sfb2"],
            d["c"])
    with pytest.raises(ValueError):   # first row not a multiple of 128
        dg.dual_gemm_grouped(*args, [128, 64], [0, 100])
    with pytest.raises(ValueError):   # overlapping groups
        dg.dual_gemm_grouped(*args, [130, 64], [0, 128])
    with pytest.raises(ValueError):   # cluster split-K is not offered
        dg.dual_gemm_grouped(*args, [128, 64], flags=_lib.FLAG_SPLITK)
    with pytest.raises(ValueError):   # weights of one expert only
        dg.dual_gemm_grouped(d["a"], d["b1"][..., :1], d["b2"][..., :1],
                             d["sfa"], d["sfb1"], d["sfb2"], d["c"],
                             [128, 64])
