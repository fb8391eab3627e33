"""Failure detection without a GPU fault.

Every wait of the pipelined kernels (TMA -> MMA -> softmax/epilogue hand-offs
on mbarriers) is bounded in time: a wait that runs out raises the CTA's abort
flag, records NT_B200_ERR_DEVICE_TIMEOUT in the library's device error word
and returns, so a broken pipeline ends with an error status instead of a hung
GPU.  `nt_b200_wait_timeout_selftest` drives that same wait on an mbarrier
that nothing ever arrives on, with a short limit; the tests check the status
the host reads and that the context keeps working afterwards."""

import time

import pytest
import torch

from ninetoothed_b200 import _lib


def test_selftest_rejects_limits_outside_its_range_without_launching():
    lib = _lib.library()
    assert lib.nt_b200_wait_timeout_selftest(10, None) == 10001
    assert lib.nt_b200_wait_timeout_selftest(2_000_000_000, None) == 10001


@pytest.mark.gpu
def test_a_wait_that_runs_out_is_reported_and_the_context_survives():
    from ninetoothed_b200 import programs
    from ninetoothed_b200.runtime import device_status

    lib = _lib.library()
    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream().cuda_stream
    assert device_status() == 0  # start from a clear error word
    start = time.perf_counter()
    assert lib.nt_b200_wait_timeout_selftest(20_000_000, stream) == 0  # 20 ms limit
    assert device_status() == 10005  # NT_B200_ERR_DEVICE_TIMEOUT
    assert time.perf_counter() - start < 5.0
    assert device_status() == 0  # reading the word clears it
    # the context is intact: a real kernel still runs and is still right
    x = torch.randn(64, 300, device="cuda")
    torch.testing.assert_close(programs.softmax(x), torch.softmax(x, dim=-1), rtol=1e-5, atol=1e-6)
    assert device_status() == 0
