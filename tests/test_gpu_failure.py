"""Failure detection on the GPU without a GPU fault: a bounded wait is made to
run out and the error is read on the host.

The reference spins on its mbarriers without a limit
(tma-interface.cuh:64-75), so a scheduling error there hangs the GPU.  Here
every wait is bounded; the test hook NVFP4DG_FLAG_TEST_SK_TIMEOUT makes the
owner of each tile split along K (stream-K) wait for one contribution more
than exist, with a short limit.  That wait is a spin on a global counter
with no copy or MMA of the waiting thread outstanding.  It must end with
the owner's error bit in the device error word (NVFP4DG_ERR_DEVICE), and the
same device must then run a clean, oracle-checked call.
"""
import ctypes

import pytest
import torch

import nvfp4_dual_gemm_b200 as dg
from nvfp4_dual_gemm_b200 import _lib
from oracle import nvfp4_oracle as O
from tests.helpers import assert_close, to_device

pytestmark = pytest.mark.gpu

KERR_EPILOGUE = 1 << 2  # device error word bit of an epilogue-side wait


def _call(d, flags, ws):
    dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                 d["sfb1_blocked"], d["sfb2_blocked"], d["c"],
                 flags=flags | _lib.FLAG_SYNC_CHECK, workspace=ws)
    torch.cuda.synchronize()


@pytest.mark.parametrize("flags", [
    5 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_BN64 | _lib.FLAG_NO_PAIR,
    6 | _lib.FLAG_FORCE_STREAMK | _lib.FLAG_BN128 | _lib.FLAG_PAIR,
])
def test_stream_k_owner_wait_runs_out_and_device_recovers(flags):
    m, n, k = 256, 512, 2048
    assert dg.plan(m, n, k, flags)["sk_tiles"] > 0
    p = O.make_problem(m, n, k, seed=51)
    d = to_device(p)
    ws = torch.zeros(dg.workspace_size(m, n, k, flags), dtype=torch.uint8,
                     device="cuda")
    with pytest.raises(RuntimeError) as exc:
        _call(d, flags | _lib.FLAG_TEST_SK_TIMEOUT, ws)
    msg = str(exc.value)
    assert f"status {_lib.ERR_DEVICE}" in msg
    word = int(msg.rsplit("device error word ", 1)[1].split(")")[0])
    assert word & KERR_EPILOGUE
    # the error word was read and cleared by the failing call
    w = ctypes.c_uint(123)
    rc = _lib.load().nvfp4_dual_gemm_device_status(
        torch.cuda.current_device(), ctypes.byref(w))
    assert rc == _lib.OK and w.value == 0, (rc, w.value)
    # the owners that gave up left their tile counters behind: a caller-owned
    # workspace is zero-filled again, then the same device computes cleanly
    ws.zero_()
    d["c"].fill_(float("nan"))
    _call(d, flags, ws)
    assert_close(d["c"].cpu().numpy(), O.reference_output(p),
                 "clean call after the expired wait")
    # and the library-owned workspace path too
    d["c"].fill_(float("nan"))
    dg.dual_gemm(d["a"], d["b1"], d["b2"], d["sfa_blocked"],
                 d["sfb1_blocked"], d["sfb2_blocked"], d["c"],
                 flags=flags | _lib.FLAG_SYNC_CHECK)
    torch.cuda.synchronize()
    assert_close(d["c"].cpu().numpy(), O.reference_output(p),
                 "clean call, library workspace")
