"""The C-ABI library loads and exports every entry point include/trnblas_b200.h
declares; host-side argument checks and workspace queries need no GPU."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from trnblas_b200 import _native as N

HEADER = Path(__file__).resolve().parent.parent / "include" / "trnblas_b200.h"


def header_symbols() -> list[str]:
    return sorted(set(re.findall(r"TRNBLAS_API\s+[\w\s\*]+?\b(trnblas_\w+)\s*\(", HEADER.read_text())))


def test_header_symbols_exported():
    syms = header_symbols()
    assert len(syms) >= 12
    handle = ctypes.CDLL(str(N.LIB_PATH))
    for s in syms:
        assert hasattr(handle, s), s
    assert sorted(N.exported_symbols()) == syms  # the binding declares exactly the header's API


def test_version_and_no_error():
    assert N.lib().trnblas_version() == 100


def test_workspace_queries():
    L = N.lib()
    assert L.trnblas_gemm_workspace_size(N.BF16, 1, 128, 128, 128, 0, 0) == 0
    w = L.trnblas_gemm_workspace_size(N.F32, 1, 100, 50, 30, 0, 0)
    assert w >= 2 * 100 * 32 * 4 + 2 * 50 * 32 * 4
    assert L.trnblas_gemm_workspace_size(N.F32, 4, 100, 50, 30, 100 * 30, 0) > w
    assert L.trnblas_syrk_workspace_size(N.F32, 64, 64) >= 2 * 64 * 64 * 4
    assert L.trnblas_gemm_fp64_workspace_size(64, 64, 64, 8) >= 8 * 2 * 64 * 64
    assert L.trnblas_gemm_fp64_workspace_size(64, 64, 64, 13) == 0
    assert L.trnblas_pair_energy_workspace_size(4, 10, 32, 0, 10) >= 5 * 40 * 32


def test_argument_errors_without_gpu():
    L = N.lib()
    rc = L.trnblas_gemm(7, 1, 4, 4, 4, 1.0, None, 4, 0, 0, None, 4, 0, 0, 0.0, None, 0, 0, None, 4, 0, None, 0, None)
    assert rc == N.ERR_ARG and "dtype" in N.last_error()
    rc = L.trnblas_gemm(N.F32, 1, -1, 4, 4, 1.0, None, 4, 0, 0, None, 4, 0, 0, 0.0, None, 0, 0, None, 4, 0, None, 0, None)
    assert rc == N.ERR_ARG
    rc = L.trnblas_syrk(N.F32, 4, 4, 1.0, None, 4, 0, 0.0, None, 0, 3, None, 4, None, 0, None)
    assert rc == N.ERR_ARG and "c_uplo" in N.last_error()
    rc = L.trnblas_gemm_fp64(4, 4, 4, None, 4, 0, None, 4, 0, 0, None, 4, None, 0, None)
    assert rc == N.ERR_ARG
    rc = L.trnblas_pair_energy(4, 10, 32, None, None, None, 0, 11, None, None, 0, None)
    assert rc == N.ERR_ARG
    with pytest.raises(ValueError):
        N.check(rc, "pair")
    # empty problems are no-ops
    assert L.trnblas_gemm(N.F32, 1, 0, 4, 4, 1.0, None, 4, 0, 0, None, 4, 0, 0, 0.0, None, 0, 0, None, 4, 0, None, 0, None) == 0


def test_dtype_codes():
    import torch

    assert N.dtype_code(torch.float32) == N.F32 and N.dtype_code(torch.bfloat16) == N.BF16
    with pytest.raises(TypeError):
        N.dtype_code(torch.int32)
