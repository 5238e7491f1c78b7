"""Bounded-wait failure path on the GPU, without a fault: a kernel waits on an
mbarrier nothing completes, gives up after a short bound, records its code in
the device status word, and the context stays usable."""

from __future__ import annotations

import pytest
import torch

import trnblas_b200 as tb
from trnblas_b200 import _native as N

pytestmark = pytest.mark.gpu


def test_wait_selftest_records_status_and_context_survives():
    assert tb.device_status(0) == 0
    N.check(N.lib().trnblas_wait_selftest(2_000_000, N.stream_ptr(torch.device("cuda", 0))), "selftest")
    assert tb.device_status(0) == 6
    assert tb.device_status(0) == 0  # read-and-clear
    x = torch.randn(256, 256, device="cuda")
    assert float((tb.gemm(1.0, x, x) - x.double() @ x.double()).norm()) < 1e-2
    assert tb.device_status(0) == 0


def test_bad_arguments_fail_before_launch():
    with pytest.raises(ValueError):
        N.check(N.lib().trnblas_gemm(9, 1, 4, 4, 4, 1.0, None, 4, 0, 0, None, 4, 0, 0, 0.0, None, 0, 0, None, 4, 0, None, 0, None), "gemm")
    with pytest.raises(ValueError):
        N.check(N.lib().trnblas_wait_selftest(0, None), "selftest")
