"""Failure detection on the GPU without a fault: a bounded wait gives up.

A one-thread kernel waits on a barrier that nothing completes.  After its spin
limit it records a timeout in the device error word and returns, as every wait
of the tensor-core GEMM does.  The host reads the status, the word is cleared,
and the context keeps working.
"""
import numpy as np
import pytest

from minitensor_cpp_b200 import abi

pytestmark = pytest.mark.gpu


def test_a_bounded_wait_that_runs_out_reports_an_error_and_the_gpu_keeps_working(cuda):
    import torch

    s = torch.cuda.current_stream().cuda_stream
    abi.check_device_errors(0, s)  # start from a clear word
    abi.check(abi.lib().mtc_selftest_bounded_wait(20000, s), "self-test launch")
    with pytest.raises(abi.MtcError, match="gave up waiting"):
        abi.check_device_errors(0, s)
    abi.check_device_errors(0, s)  # cleared by the read above
    # the context is intact: a GEMM on the same stream still matches the oracle
    a = torch.randn(256, 128, device="cuda")
    b = torch.randn(128, 512, device="cuda")
    c = torch.empty(256, 512, device="cuda")
    abi.matmul(abi.View.of(a), abi.View.of(b), abi.View.of(c), abi.GEMM_3XTF32)
    torch.cuda.synchronize()
    ref = (a.double() @ b.double()).float()
    assert torch.allclose(c, ref, rtol=1e-4, atol=1e-4)


def test_the_spin_limit_is_validated(cuda):
    with pytest.raises(ValueError):
        abi.check(abi.lib().mtc_selftest_bounded_wait(0, None), "self-test")
