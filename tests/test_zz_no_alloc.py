"""The allocation-free fp32 GEMM entry point, called through the C ABI.

It is for callers that cannot allocate device memory when they multiply (a
plugin whose host application owns all device memory, or a loop in which
cudaMalloc's device synchronisation is not allowed): its split scratch is an
array built into the library. The test compares it with the ordinary
trnblas_gemm (caller-provided workspace) on two calls in a row, so the second
call runs on scratch that still holds the first call's contents, and checks
that an over-size problem is refused. With a second GPU it repeats the
comparison with that GPU current, where the library looks up the array's
address on that device for the first time.

The file name sorts last so that pytest collects it after every other test:
a run that stops at the first failure (-x) has then already run the rest of
the suite, and a failure here cannot hide another. It also runs alone in a
fresh process.
"""

from __future__ import annotations

import pytest
import torch

from trnblas_b200 import _native as N

pytestmark = pytest.mark.gpu
TOL = 1e-5  # the fp32 (3xTF32) tolerance of the GEMM tests


def _relf(x, ref):
    return float((x.double() - ref.double()).norm() / ref.double().norm())


def _noalloc(A, B, C, alpha, beta, transA, transB, M, N_, K):
    D = torch.empty((M, N_), dtype=torch.float32, device=A.device)
    lda, ldb = A.stride(0), B.stride(0)
    rc = N.lib().trnblas_gemm_f32_noalloc(
        M, N_, K, alpha, A.data_ptr(), lda, int(transA), B.data_ptr(), ldb, int(transB),
        beta, C.data_ptr(), C.stride(0), D.data_ptr(), D.stride(0), N.stream_ptr(A.device))
    return rc, D


def _with_workspace(A, B, C, alpha, beta, transA, transB, M, N_, K):
    D = torch.empty((M, N_), dtype=torch.float32, device=A.device)
    ws_n = N.lib().trnblas_gemm_workspace_size(N.F32, 1, M, N_, K, 0, 0)
    ws = torch.empty(ws_n, dtype=torch.uint8, device=A.device)
    rc = N.lib().trnblas_gemm(
        N.F32, 1, M, N_, K, alpha, A.data_ptr(), A.stride(0), 0, int(transA), B.data_ptr(),
        B.stride(0), 0, int(transB), beta, C.data_ptr(), C.stride(0), 0, D.data_ptr(),
        D.stride(0), 0, ws.data_ptr(), ws_n, N.stream_ptr(A.device))
    return rc, D


def _two_calls(dev: torch.device):
    g = torch.Generator(device=dev).manual_seed(11)
    # odd leading dimensions (517, then 257) send the first two calls through
    # the split into the built-in scratch, the second on the first's leftover
    # contents; the third has TMA-aligned operands (split inside the kernel)
    cases = [(300, 200, 517, False, False), (257, 129, 333, True, False), (1024, 768, 1536, True, True)]
    for M, N_, K, ta, tb in cases:
        A = torch.randn(*((K, M) if ta else (M, K)), device=dev, generator=g)
        B = torch.randn(*((N_, K) if tb else (K, N_)), device=dev, generator=g)
        C = torch.randn(M, N_, device=dev, generator=g)
        rc1, D1 = _noalloc(A, B, C, 0.75, -0.5, ta, tb, M, N_, K)
        rc2, D2 = _with_workspace(A, B, C, 0.75, -0.5, ta, tb, M, N_, K)
        assert rc1 == 0, N.last_error()
        assert rc2 == 0, N.last_error()
        torch.cuda.synchronize(dev)
        assert _relf(D1, D2) <= TOL
        a = A.double().T if ta else A.double()
        b = B.double().T if tb else B.double()
        assert _relf(D1, 0.75 * a @ b - 0.5 * C.double()) <= TOL
    assert N.device_status(dev.index) == 0


def test_noalloc_matches_trnblas_gemm_on_two_calls():
    _two_calls(torch.device("cuda", 0))


def test_noalloc_on_second_device():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs a second GPU")
    with torch.cuda.device(1):
        _two_calls(torch.device("cuda", 1))


def test_noalloc_rejects_oversize_problem():
    A = torch.empty(1, device="cuda")
    # 2 * (M + N) * K * 4 bytes = 2 * 8192 * 4096 * 4 = 256 MiB of split planes
    rc = N.lib().trnblas_gemm_f32_noalloc(4096, 4096, 4096, 1.0, A.data_ptr(), 4096, 0, A.data_ptr(),
                                          4096, 0, 0.0, None, 0, A.data_ptr(), 4096,
                                          N.stream_ptr(A.device))
    assert rc == N.ERR_WORKSPACE
    assert "scratch" in N.last_error()
