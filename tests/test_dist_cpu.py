"""N-sharding host logic on CPU: shard views, gather of the column slices and
the max-over-ranks timing reduction, run as world_size-2 gloo ranks.

Each rank takes its slice of B1/B2 and of the blocked scales through
``shard_weights`` (views, no copies), computes its C slice with the oracle,
and the gathered result must equal the oracle's full output."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nvfp4_dual_gemm_b200 import shard
from oracle import nvfp4_oracle as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, shape, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        m, n, k = shape
        p = O.make_problem(m, n, k, seed=21)
        spec = shard.shard_spec(n, k, world, rank)
        B1 = torch.from_numpy(p["b1"])
        B2 = torch.from_numpy(p["b2"])
        S1 = torch.from_numpy(p["sfb1_blocked"])
        S2 = torch.from_numpy(p["sfb2_blocked"])
        b1, b2, s1, s2 = shard.shard_weights(spec, B1, B2, S1, S2)
        # Views of the caller's storage, and the right bytes.
        assert b1.data_ptr() == B1[spec.n0].data_ptr()
        assert s1.data_ptr() == S1.reshape(-1)[spec.scale_bytes[0]:].data_ptr()
        want1 = O.to_blocked(p["sfb1"][spec.n0:spec.n1])
        assert np.array_equal(s1.numpy().reshape(-1), want1.reshape(-1))
        sf1 = O.from_blocked(s1.numpy(), spec.rows, k)
        sf2 = O.from_blocked(s2.numpy(), spec.rows, k)
        c_r = O.dual_gemm(p["a"], p["sfa"], b1.numpy(), sf1, b2.numpy(), sf2)
        full = shard.gather_columns(torch.from_numpy(c_r), spec)
        # Column placement, exactly: every rank contributes its rank id.
        tag = torch.full((m, spec.rows), float(rank), dtype=torch.float16)
        tags = shard.gather_columns(tag, spec)
        t_max = shard.max_over_ranks(1.5 + rank)
        np.savez(os.path.join(result_dir, f"r{rank}.npz"), full=full.numpy(),
                 tags=tags.numpy(), t_max=t_max)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shape", [(64, 512, 512), (130, 768, 256)])
def test_two_rank_shard_gather(tmp_path, shape):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), shape,
                                         str(tmp_path)),
                       nprocs=world, start_method="spawn", join=True)
    m, n, k = shape
    ref = O.reference_output(O.make_problem(m, n, k, seed=21))
    for r in range(world):
        got = np.load(tmp_path / f"r{r}.npz")
        ok, n_bad, worst = O.check_close(got["full"], ref)
        assert ok, f"rank {r}: {n_bad} outputs differ (worst {worst})"
        cols = np.repeat(np.arange(world), n // world)
        assert np.array_equal(got["tags"], np.broadcast_to(cols, (m, n)))
        assert float(got["t_max"]) == 1.5 + world - 1


def test_shard_spec_ranges_and_errors():
    s = shard.shard_spec(28672, 8192, 8, 3)
    assert (s.n0, s.n1, s.rows) == (10752, 14336, 3584)
    per_block = 8192 // 64 * 512
    assert s.scale_bytes == (10752 // 128 * per_block, 14336 // 128 * per_block)
    spans = [shard.shard_spec(1024, 256, 4, r) for r in range(4)]
    assert [x.n0 for x in spans] == [0, 256, 512, 768]
    assert spans[-1].n1 == 1024
    with pytest.raises(ValueError):
        shard.shard_spec(28672 + 64, 8192, 8, 0)   # slice not 128-row aligned
    with pytest.raises(ValueError):
        shard.shard_spec(1024, 300, 2, 0)          # K not a multiple of 256
    with pytest.raises(ValueError):
        shard.shard_spec(1024, 256, 2, 2)          # rank outside the world


def test_shard_weights_rejects_wrong_sizes():
    spec = shard.shard_spec(256, 256, 2, 1)
    b = torch.zeros(256, 128, dtype=torch.uint8)
    sf = torch.zeros(256 * 256 // 16, dtype=torch.uint8)
    with pytest.raises(ValueError):
        shard.shard_weights(spec, b[:128], b, sf, sf)
    with pytest.raises(ValueError):
        shard.shard_weights(spec, b, b, sf[:-1], sf)
    out = shard.shard_weights(spec, b, b, sf, sf)
    assert out[0].shape == (128, 128) and out[2].numel() == 128 * 256 // 16


def test_max_over_ranks_single_process():
    assert shard.max_over_ranks(2.5) == 2.5
