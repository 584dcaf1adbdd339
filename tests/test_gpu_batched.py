"""GPU tests of batched problems (L > 1): L independent dual GEMMs of one
shape in one launch, tiles of all batches scheduled together.

The reference's tensors carry an L dimension ([rows, K/2, L], batch after
batch in memory) that its kernel ignores (nvfp4_dual_gemm.cu:381-446 reads
batch 0 only); here every batch is computed.  Each batch is compared with
the oracle's product of that batch within rtol = atol = 1e-3, over every
schedule (whole tiles, stream-K, cluster split-K, 1-SM and 2-SM pair tiles)
and for the NVFP4 output.
"""
import numpy as np
import pytest
import torch

import nvfp4_dual_gemm_b200 as dg
from nvfp4_dual_gemm_b200 import _lib
from oracle import nvfp4_oracle as O
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu

BN64, BN128 = _lib.FLAG_BN64, _lib.FLAG_BN128
PATHS = {
    "auto": 0,
    "1sm_bn64": BN64 | _lib.FLAG_NO_PAIR | _lib.FLAG_NO_STREAMK,
    "1sm_bn128": BN128 | _lib.FLAG_NO_PAIR | _lib.FLAG_NO_STREAMK,
    "pair_bn128": BN128 | _lib.FLAG_PAIR | _lib.FLAG_NO_STREAMK,
    "streamk_1sm": 7 | BN64 | _lib.FLAG_NO_PAIR | _lib.FLAG_FORCE_STREAMK,
    "streamk_pair": 5 | BN128 | _lib.FLAG_PAIR | _lib.FLAG_FORCE_STREAMK,
    "splitk_1sm": BN128 | _lib.FLAG_NO_PAIR | _lib.FLAG_SPLITK,
    "splitk_pair": BN64 | _lib.FLAG_PAIR | _lib.FLAG_SPLITK,
}


def batched(problems, device="cuda"):
    """Stack oracle problems into the batch-after-batch tensors the API
    takes: [rows, cols, L] views of [L, rows, cols] tensors, blocked scales
    one layout after another, C [M, N, L]."""
    def stack(key):
        return torch.from_numpy(np.stack([p[key] for p in problems])).to(
            device).permute(1, 2, 0)

    def cat(key):
        return torch.from_numpy(np.concatenate(
            [p[key] for p in problems])).to(device)

    m, n = problems[0]["M"], problems[0]["N"]
    d = {k: stack(k) for k in ("a", "b1", "b2")}
    for k in ("sfa_blocked", "sfb1_blocked", "sfb2_blocked"):
        d[k] = cat(k)
    d["c"] = torch.full((len(problems), m, n), float("nan"),
                        dtype=torch.float16, device=device).permute(1, 2, 0)
    return d


def run_batched(problems, flags):
    d = batched(problems)
    dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                 d["sfb1_blocked"], d["sfb2_blocked"], d["c"],
                 flags=flags | _lib.FLAG_SYNC_CHECK)
    torch.cuda.synchronize()
    return d, d["c"].permute(2, 0, 1).cpu().numpy()


@pytest.mark.parametrize("path", list(PATHS))
@pytest.mark.parametrize("m,n,k,L", [(128, 256, 512, 3), (200, 384, 768, 2),
                                     (300, 128, 1024, 4)])
def test_batched_matches_each_batch(path, m, n, k, L):
    flags = PATHS[path]
    if flags & BN128 and n % 128:
        pytest.skip("BN = 128 needs N % 128 == 0")
    problems = [O.make_problem(m, n, k, seed=100 * b + m + n)
                for b in range(L)]
    pl = dg.plan(m, n, k, flags)
    if flags & _lib.FLAG_SPLITK and 2 * pl["ctas"] * pl["dp_tiles"] * L > 148:
        pytest.skip("cluster split-K needs 2 x tiles x CTAs <= SMs")
    _, got = run_batched(problems, flags)
    for b, p in enumerate(problems):
        assert_close(got[b], O.reference_output(p),
                     f"{path} {m}x{n}x{k} batch {b} of {L}")


def test_batched_nvfp4_output():
    problems = [O.make_problem(256, 512, 1024, seed=7 + b) for b in range(3)]
    d, c16 = run_batched(problems, 0)
    cq, sfc = dg.dual_gemm_nvfp4(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                                 d["sfb1_blocked"], d["sfb2_blocked"])
    torch.cuda.synchronize()
    assert cq.shape == (256, 256, 3)
    cq = cq.permute(2, 0, 1).cpu().numpy()
    blk = sfc.cpu().numpy().reshape(3, -1)
    for b in range(3):
        codes, sf = O.quantize(c16[b].astype(np.float32))
        assert np.array_equal(cq[b], codes), f"codes of batch {b}"
        assert np.array_equal(blk[b], O.to_blocked(sf)), f"scales of batch {b}"


def test_batched_custom_kernel_entry():
    # generate_input's batch-after-batch tensors through the reference's
    # entry point; batch 0 holds the inputs of the unbatched problem of the
    # same seed (the schedules differ, so outputs agree to the tolerance)
    data = dg.generate_input(128, 256, 512, l=2, seed=3)
    out = dg.custom_kernel(data)
    torch.cuda.synchronize()
    assert out.shape == (128, 256, 2)
    single = dg.generate_input(128, 256, 512, l=1, seed=3)
    assert torch.equal(single[0].view(torch.uint8)[..., 0],
                       data[0].view(torch.uint8)[..., 0])
    out1 = dg.custom_kernel(single)
    torch.cuda.synchronize()
    assert_close(out[:, :, 0].cpu().numpy(), out1[:, :, 0].cpu().numpy(),
                 "batch 0 vs unbatched")
    for b in range(2):
        def host(t, rows):
            return t.view(torch.uint8)[..., b].cpu().numpy()
        a = host(data[0], 128)
        b1, b2 = host(data[1], 256), host(data[2], 256)
        sfa, sfb1, sfb2 = (host(data[3], 128), host(data[4], 256),
                           host(data[5], 256))
        ref = O.dual_gemm(a, sfa, b1, sfb1, b2, sfb2)
        assert_close(out[:, :, b].cpu().numpy(), ref, f"batch {b}")


def test_batched_argument_errors():
    problems = [O.make_problem(128, 128, 256, seed=b) for b in range(2)]
    d = batched(problems)
    # C with the wrong batch count
    c1 = torch.empty((128, 128, 1), dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError):
        dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                     d["sfb1_blocked"], d["sfb2_blocked"], c1)
    # blocked scales of one batch only
    with pytest.raises(ValueError):
        dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"][:512 * 4],
                     d["sfb1_blocked"], d["sfb2_blocked"], d["c"])
    # the host-buffer entry point takes unbatched problems only
    with pytest.raises(ValueError):
        dg.dual_gemm_host(*(d[k].cpu() for k in ("a", "b1", "b2",
                                                 "sfa_blocked",
                                                 "sfb1_blocked",
                                                 "sfb2_blocked", "c")))
