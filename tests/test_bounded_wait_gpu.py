"""Failure detection on the GPU without a GPU fault: every wait inside the
GEMM kernel is bounded, and a wait that runs out makes the kernel record
MG_ERR_TIMEOUT and the wait site in its device status word, stop every role,
drain its in-flight copies and MMAs, free its tensor memory and exit -- where
the reference prints and aborts the process (macrograd_error.h:79).

The failure is made on the host: MG_GEMM_TEST_STALL=1 has each CTA's TMA
producer withhold its second K-block, and MG_GEMM_WAIT_LIMIT_MS=50 shortens
every wait's limit, so a wait for that stage (or for the accumulator it
never completes) runs out after 50 ms. The test checks that the call returns, that mg_device_status reports
the timeout and a wait site that the withheld stage can trip, and that the next ordinary call on the same
context succeeds and matches the oracle. Both kernels are exercised: the
single-SM one and the SM pair (a cluster of two CTAs)."""
import ctypes

import numpy as np
import pytest

import oracle_bridge as ob

torch = pytest.importorskip("torch")
import macrograd_b200 as mg  # noqa: E402
from macrograd_b200 import _lib, functional as F  # noqa: E402

pytestmark = pytest.mark.gpu

# wait sites a withheld stage can run out (mg_gemm_kernel.cuh): the split
# warps waiting for it to land (2), the MMA issuer waiting for the split (4),
# the epilogue waiting for the accumulator (5) -- the epilogue's wait starts
# first, at the kernel's start, so it is usually the one that runs out
STALL_SITES = {2, 4, 5}


def _status(reset):
    detail = ctypes.c_int32(0)
    st = mg.load().mg_device_status(ctypes.byref(detail), int(reset))
    return st, detail.value


@pytest.mark.parametrize("pair,M", [("0", 64), ("1", 256)], ids=["single_sm", "sm_pair"])
def test_a_wait_that_runs_out_is_reported_and_the_next_call_works(monkeypatch, pair, M):
    assert mg.load().mg_set_mode(_lib.MG_MODE_TF32X3) == 0
    assert _status(True)[0] == _lib.MG_OK, "device status not clean before the test"
    A = ob.seeded_uniform((M, 64), 960)   # K = 64: two K-blocks, the second withheld
    B = ob.seeded_uniform((64, 96), 961)
    Ag, Bg = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    monkeypatch.setenv("MG_GEMM_PAIR", pair)
    monkeypatch.setenv("MG_GEMM_WAIT_LIMIT_MS", "50")
    monkeypatch.setenv("MG_GEMM_TEST_STALL", "1")
    F.matmul(Ag, Bg)                      # the launch itself succeeds
    st, where = _status(True)             # synchronises: the kernel has exited
    assert st == _lib.MG_ERR_TIMEOUT, f"device status {st}"
    assert where in STALL_SITES, f"wait site {where}"
    monkeypatch.delenv("MG_GEMM_TEST_STALL")
    monkeypatch.delenv("MG_GEMM_WAIT_LIMIT_MS")
    C = F.matmul(Ag, Bg).cpu().numpy()     # the context is still usable
    assert _status(False)[0] == _lib.MG_OK
    assert ob.frob_rel_err(C, ob.oracle_matmul(A, B)) <= 1e-5
