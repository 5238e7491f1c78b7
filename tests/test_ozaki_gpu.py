"""gemm_fp64 (Ozaki on the int8 tensor cores) against the oracle: digits bit
for bit against the reference's split, results bit for bit against the
oracle's restatement of the kernel arithmetic, accuracy against host fp64
BLAS (gate: relative Frobenius error <= 1e-14 at k = 8)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import trnblas_b200 as tb
from oracle import ozaki as OZ
from trnblas_b200 import _native as N

pytestmark = pytest.mark.gpu
DEV = "cuda"
Z = np.load("tests/golden/ozaki.npz")


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert tb.device_status(0) == 0


def _split(X: np.ndarray, k: int):
    Xd = torch.from_numpy(np.ascontiguousarray(X)).to(DEV)
    R, K = Xd.shape
    dig = torch.empty((k, R, K), dtype=torch.int8, device=DEV)
    ex = torch.empty(R, dtype=torch.int32, device=DEV)
    ws = torch.empty(8 * R + 256, dtype=torch.uint8, device=DEV)
    N.check(N.lib().trnblas_ozaki_split(R, K, Xd.data_ptr(), K, 1, k, dig.data_ptr(), K, ex.data_ptr(),
                                        ws.data_ptr(), ws.numel(), N.stream_ptr(Xd.device)), "split")
    return dig.cpu().numpy(), ex.cpu().numpy().astype(np.int64)


@pytest.mark.parametrize("k", [1, 3, 8, 12])
def test_split_bitwise_vs_reference(k):
    d, e = _split(Z["X"], k)
    assert np.array_equal(d, Z[f"split_row_{k}_d"]) and np.array_equal(e, Z[f"split_row_{k}_e"])
    d, e = _split(Z["X"].T, k)  # per column of X = per row of X^T
    assert np.array_equal(d.transpose(0, 2, 1), Z[f"split_col_{k}_d"]) and np.array_equal(e, Z[f"split_col_{k}_e"])


@pytest.mark.parametrize("k", [5, 8])
def test_split_any_strides_bitwise(k):
    """Element (r, c) at X[r * rs + c * ks] with neither stride 1 (every other
    column of a wider matrix): the generic row-max pass and the digit pass
    give the digits of the same matrix made contiguous, bit for bit."""
    X = Z["X"]
    R, K = X.shape
    wide = np.zeros((R, 2 * K))
    wide[:, ::2] = X
    Wd = torch.from_numpy(wide).to(DEV)
    dig = torch.empty((k, R, K), dtype=torch.int8, device=DEV)
    ex = torch.empty(R, dtype=torch.int32, device=DEV)
    ws = torch.empty(8 * R + 256, dtype=torch.uint8, device=DEV)
    N.check(N.lib().trnblas_ozaki_split(R, K, Wd.data_ptr(), 2 * K, 2, k, dig.data_ptr(), K, ex.data_ptr(),
                                        ws.data_ptr(), ws.numel(), N.stream_ptr(Wd.device)), "split")
    d, e = _split(X, k)
    assert np.array_equal(dig.cpu().numpy(), d) and np.array_equal(ex.cpu().numpy().astype(np.int64), e)


def test_split_extreme_rows_bitwise():
    d, e = _split(Z["Xe"], 8)
    assert np.array_equal(d, Z["split_extreme_d"]) and np.array_equal(e, Z["split_extreme_e"])


@pytest.mark.parametrize("name,k", [("r0", 4), ("r0", 8), ("r1", 8), ("r2", 8), ("k1", 1)])
def test_gemm_fp64_bitwise_vs_oracle(name, k):
    A, B = Z[f"{name}_A"], Z[f"{name}_B"]
    C = tb.gemm_fp64(torch.from_numpy(A).to(DEV), torch.from_numpy(B).to(DEV), slices=k).cpu().numpy()
    assert np.array_equal(C, OZ.gemm_diag(A, B, k))
    ref = Z["k1_ref"] if name == "k1" else Z[f"{name}_ref{k}"]
    assert float(np.linalg.norm(C - ref) / np.linalg.norm(ref)) <= (1e-14 if k >= 8 or name == "k1" else 1e-9)


@pytest.mark.parametrize("k", [6, 9, 10, 12])
@pytest.mark.parametrize("ta,tbb", [(False, False), (True, True), (True, False)])
def test_gemm_fp64_slices_and_layouts(k, ta, tbb):
    rng = np.random.default_rng(k)
    A = rng.standard_normal((130, 257)) * np.exp2(rng.integers(-10, 11, (130, 257)))
    B = rng.standard_normal((257, 70)) * np.exp2(rng.integers(-10, 11, (257, 70)))
    At = torch.from_numpy(np.ascontiguousarray(A.T)).to(DEV) if ta else torch.from_numpy(A).to(DEV)
    Bt = torch.from_numpy(np.ascontiguousarray(B.T)).to(DEV) if tbb else torch.from_numpy(B).to(DEV)
    C = tb.gemm_fp64(At, Bt, slices=k, transA=ta, transB=tbb).cpu().numpy()
    assert np.array_equal(C, OZ.gemm_diag(A, B, k))


def test_gemm_fp64_config4_accuracy():
    """Benchmark case 4 at full size: 4096^3, m * 2^e entries (seed 4), k = 8,
    against fp64 BLAS (cuBLAS DGEMM) on the same inputs."""
    rng = np.random.default_rng(4)
    A = rng.standard_normal((4096, 4096)) * np.exp2(rng.integers(-10, 11, (4096, 4096)))
    B = rng.standard_normal((4096, 4096)) * np.exp2(rng.integers(-10, 11, (4096, 4096)))
    Ad, Bd = torch.from_numpy(A).to(DEV), torch.from_numpy(B).to(DEV)
    C = tb.gemm_fp64(Ad, Bd)
    H = Ad @ Bd
    assert float((C - H).norm() / H.norm()) <= 1e-14
    # oracle bitwise on a corner block (full product restricted to rows/cols)
    sub = OZ.gemm_diag(A[:64], B[:, :48], 8)
    # the per-row / per-column scales of the block are those of the full split
    assert float(np.abs(C[:64, :48].cpu().numpy() - sub).max()) == 0.0


def test_gemm_fp64_api_errors_and_nonfinite():
    with pytest.raises(TypeError):
        tb.gemm_fp64(torch.randn(3, 3, device=DEV), torch.randn(3, 3, device=DEV), slices=2.0)
    with pytest.raises(ValueError):
        tb.gemm_fp64(torch.randn(3, 3, device=DEV), torch.randn(3, 3, device=DEV), slices=13)
    with pytest.raises(ValueError):
        tb.gemm_fp64(torch.randn(3, 4, device=DEV), torch.randn(3, 3, device=DEV))
    with pytest.raises(TypeError):
        tb.gemm_fp64(torch.ones(3, 3, dtype=torch.int64), torch.ones(3, 3, dtype=torch.int64))
    A = torch.randn(8, 8, device=DEV, dtype=torch.float64)
    A[0, 0] = float("inf")
    out = tb.gemm_fp64(A, torch.randn(8, 8, device=DEV, dtype=torch.float64))
    assert torch.isinf(out[0]).any()
    z = tb.gemm_fp64(torch.randn(4, 0, device=DEV), torch.randn(0, 5, device=DEV))
    assert z.shape == (4, 5) and z.dtype == torch.float64 and not z.any()
