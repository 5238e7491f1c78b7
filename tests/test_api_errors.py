"""Argument errors of the public API, checked before any device work (CPU
tensors, no GPU needed), with the reference's exception types: ValueError for
shapes and flags, TypeError for a non-int slice count or a non-float
gemm_fp64 operand (trnblas/level3.py:137-193, 196-240, 243-295, 332-417;
trnblas/_flags.py:18-51)."""

from __future__ import annotations

import pytest
import torch

import trnblas_b200 as tb

f64 = torch.float64


@pytest.mark.parametrize(
    "call,exc",
    [
        (lambda: tb.syrk(1.0, torch.randn(2, 3, 4)), ValueError),
        (lambda: tb.gemm_fp64(torch.randn(3, 3, dtype=f64), torch.randn(3, 3, dtype=f64), slices=2.0), TypeError),
        (lambda: tb.gemm_fp64(torch.randn(3, 3, dtype=f64), torch.randn(3, 3, dtype=f64), slices=True), TypeError),
        (lambda: tb.gemm_fp64(torch.randn(3, 3, dtype=f64), torch.randn(3, 3, dtype=f64), slices=13), ValueError),
        (lambda: tb.gemm_fp64(torch.randn(3, 3, dtype=f64), torch.randn(3, 3, dtype=f64), slices=0), ValueError),
        (lambda: tb.gemm_fp64(torch.randn(3, dtype=f64), torch.randn(3, 3, dtype=f64)), ValueError),
        (lambda: tb.gemm_fp64(torch.ones(3, 3, dtype=torch.int64), torch.ones(3, 3, dtype=torch.int64)), TypeError),
        (lambda: tb.gemm_fp64(torch.randn(3, 4, dtype=f64), torch.randn(3, 3, dtype=f64)), ValueError),
        (lambda: tb.trsm(1.0, torch.randn(3, 4), torch.randn(3, 2)), ValueError),
        (lambda: tb.trsm(1.0, torch.randn(3, 3), torch.randn(2, 3, 2)), ValueError),
        (lambda: tb.trsm(1.0, torch.randn(3, 3), torch.randn(4, 2)), ValueError),
        (lambda: tb.trsm(1.0, torch.randn(3, 3), torch.randn(3, 2), side="middle"), ValueError),
        (lambda: tb.trsm(1.0, torch.randn(3, 3), torch.randn(3, 2), diag="sometimes"), ValueError),
        (lambda: tb.metric_inv_half(torch.randn(3, 4)), ValueError),
        (lambda: tb.symm(1.0, torch.randn(3, 4), torch.randn(4, 2)), ValueError),
        (lambda: tb.trmm(1.0, torch.randn(3, 4), torch.randn(4, 2)), ValueError),
        (lambda: tb.gemm(1.0, torch.randn(3, 3), torch.randn(3, 3), transA="C"), ValueError),
        (lambda: tb.syrk(1.0, torch.randn(3, 3), uplo="middle"), ValueError),
    ],
)
def test_argument_errors_before_device_work(call, exc):
    with pytest.raises(exc):
        call()
