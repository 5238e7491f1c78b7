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


FAKE = 1 << 20  # a non-NULL address that the argument checks reject before any use


@pytest.mark.parametrize("dtype", [N.F32, N.BF16, N.F16])
@pytest.mark.parametrize("lda,ldb,ta,tb", [(3, 8, 0, 0), (8, 3, 0, 0), (-8, 8, 0, 0), (8, 4, 1, 0), (8, 7, 0, 1)])
def test_gemm_leading_dimensions_checked_for_every_dtype(dtype, lda, ldb, ta, tb):
    """lda / ldb below the stored row length (A: K, or M when transposed; B: N,
    or K when transposed) or negative are refused before any device work, for
    the fp32 split path as well as the 16-bit TMA path. M = 8, N = 8, K = 4,
    except the transposed cases, where the short leading dimension is set
    against M = 8 (A) or K = 8 (B)."""
    L = N.lib()
    M, Nn, K = (8, 8, 4) if not ta and not tb else ((8, 8, 8))
    rc = L.trnblas_gemm(dtype, 1, M, Nn, K, 1.0, FAKE, lda, 0, ta, FAKE, ldb, 0, tb, 0.0, None, 0, 0,
                        FAKE, Nn, 0, FAKE, 1 << 20, None)
    assert rc == N.ERR_ARG and "lda/ldb" in N.last_error()


def test_syrk_lda_checked_for_fp32():
    L = N.lib()
    rc = L.trnblas_syrk(N.F32, 8, 16, 1.0, FAKE, 8, 0, 0.0, None, 0, 0, FAKE, 8, FAKE, 1 << 20, None)
    assert rc == N.ERR_ARG and "lda" in N.last_error()


def test_gemm_k_limit():
    L = N.lib()
    rc = L.trnblas_gemm(N.F32, 1, 8, 8, (1 << 31) - 2, 1.0, FAKE, 1 << 31, 0, 0, FAKE, 8, 0, 0, 0.0, None, 0, 0,
                        FAKE, 8, 0, FAKE, 1 << 20, None)
    assert rc == N.ERR_ARG and "limit" in N.last_error()


def test_noalloc_argument_checks_without_gpu():
    """The allocation-free fp32 GEMM checks sizes before it touches the device:
    leading dimensions as trnblas_gemm, dimensions at the limits (whose scratch
    size would overflow a 64-bit product) and a problem too large for the
    built-in scratch are refused."""
    L = N.lib()
    fn = L.trnblas_gemm_f32_noalloc
    # lda below K (fp32 path checks it too)
    assert fn(64, 64, 64, 1.0, FAKE, 32, 0, FAKE, 64, 0, 0.0, None, 0, FAKE, 64, None) == N.ERR_ARG
    assert "lda/ldb" in N.last_error()
    big = (1 << 31) - 1
    assert fn(big, big, big - 3, 1.0, FAKE, big, 0, FAKE, big, 0, 0.0, None, 0, FAKE, big, None) == N.ERR_WORKSPACE
    assert "scratch" in N.last_error()
    assert fn(1 << 31, 8, 8, 1.0, FAKE, 8, 0, FAKE, 8, 0, 0.0, None, 0, FAKE, 8, None) == N.ERR_ARG
    assert fn(4096, 4096, 4096, 1.0, FAKE, 4096, 0, FAKE, 4096, 0, 0.0, None, 0, FAKE, 4096, None) == N.ERR_WORKSPACE


def test_symm_argument_checks_without_gpu():
    """trnblas_symm takes the kernel dtypes, and a leading dimension of the
    symmetric operand below n is refused before any device work; the 16-bit
    form needs the full symmetric operand's bytes of workspace."""
    fn = N.lib().trnblas_symm
    assert fn(99, 0, 1, 64, 32, 1.0, FAKE, 64, FAKE, 32, 0.0, None, 0, FAKE, 32, None, 0, None) == N.ERR_ARG
    assert "dtype" in N.last_error()
    assert fn(N.BF16, 0, 1, 64, 32, 1.0, FAKE, 32, FAKE, 32, 0.0, None, 0, FAKE, 32, None, 0, None) == N.ERR_ARG
    assert fn(N.BF16, 0, 1, 64, 32, 1.0, FAKE, 64, FAKE, 32, 0.0, None, 0, FAKE, 32, None, 0, None) == N.ERR_WORKSPACE
    assert N.lib().trnblas_symm_workspace_size(N.BF16, 0, 100, 7) >= 100 * 104 * 2
    assert N.lib().trnblas_symm_workspace_size(N.F32, 1, 7, 100) == N.lib().trnblas_gemm_workspace_size(N.F32, 1, 7, 100, 100, 0, 0)
    # side left: S is op(A) (64 x 64), lda 32 < 64
    assert fn(N.F32, 0, 1, 64, 32, 1.0, FAKE, 32, FAKE, 32, 0.0, None, 0, FAKE, 32, None, 0, None) == N.ERR_ARG
    # side right: S is op(B) (32 x 32), lda 16 < 32
    assert fn(N.F32, 1, 0, 64, 32, 1.0, FAKE, 16, FAKE, 32, 0.0, None, 0, FAKE, 32, None, 0, None) == N.ERR_ARG
    assert "lda/ldb" in N.last_error()


def test_dtype_codes():
    import torch

    assert N.dtype_code(torch.float32) == N.F32 and N.dtype_code(torch.bfloat16) == N.BF16
    with pytest.raises(TypeError):
        N.dtype_code(torch.int32)
