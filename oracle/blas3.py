"""Oracle: level-3 BLAS semantics of the reference, in numpy -- TEST INFRASTRUCTURE.

Restates trnblas/level3.py (reference 0.13.0):
- gemm            level3.py:69-109 with _scale_add :42-66 (op = .mT when trans);
- batched_gemm    level3.py:112-134 / dispatch.py:1385-1427 (matmul broadcasting);
- syrk            level3.py:243-295, _sym_from_triangle :298-302,
                  _symmetrize dispatch.py:3178-3199 (0.5 * (C + C^T)).
Computed in the requested numpy dtype (float64 for error attribution).
"""

from __future__ import annotations

import numpy as np


def _op(X: np.ndarray, trans: bool) -> np.ndarray:
    return np.swapaxes(X, -1, -2) if trans and X.ndim >= 2 else X


def gemm(alpha, A, B, beta=0.0, C=None, transA=False, transB=False, dtype=np.float64):
    """alpha * op(A) @ op(B) + beta * C (C ignored when beta == 0)."""
    a = _op(np.asarray(A, dtype=dtype), transA)
    b = _op(np.asarray(B, dtype=dtype), transB)
    r = dtype(alpha) * np.matmul(a, b)
    if C is not None and beta != 0.0:
        r = r + dtype(beta) * np.asarray(C, dtype=dtype)
    return r


def batched_gemm(alpha, A, B, beta=0.0, C=None, transA=False, transB=False, dtype=np.float64):
    """Batched GEMM with numpy/torch matmul batch broadcasting."""
    return gemm(alpha, A, B, beta, C, transA, transB, dtype)


def sym_from_triangle(C: np.ndarray, uplo: str) -> np.ndarray:
    """The symmetric matrix stored in the `uplo` triangle of C (level3.py:298-302)."""
    if uplo == "upper":
        return np.triu(C) + np.triu(C, 1).T
    return np.tril(C) + np.tril(C, -1).T


def symmetrize(C: np.ndarray) -> np.ndarray:
    return 0.5 * (C + C.T)


def syrk(alpha, A, beta=0.0, C=None, trans=False, uplo="upper", dtype=np.float64):
    """alpha * op(A) op(A)^T + beta * sym_uplo(C), full symmetric (level3.py:243-295)."""
    a = np.asarray(A, dtype=dtype)
    a = a.T if trans else a
    S = symmetrize(a @ a.T)
    n = a.shape[0]
    add = C is not None and beta != 0.0
    if add and np.ndim(C) == 2 and np.shape(C) == (n, n):
        return dtype(alpha) * S + dtype(beta) * sym_from_triangle(np.asarray(C, dtype=dtype), uplo)
    R = dtype(alpha) * S
    return symmetrize(R + dtype(beta) * np.asarray(C, dtype=dtype)) if add else R


def relf(x, ref) -> float:
    """Relative Frobenius error ||x - ref|| / ||ref||."""
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(x - ref) / (den if den > 0 else 1.0))


def symm(alpha, A, B, beta=0.0, C=None, side="left", uplo="upper", dtype=np.float64):
    """trnblas/level3.py:196-240: alpha * sym(A) @ B (+ beta C), or B @ sym(A);
    sym(A) built from A's `uplo` triangle."""
    A = np.asarray(A, dtype=dtype)
    S = np.triu(A) + np.triu(A, 1).T if uplo == "upper" else np.tril(A) + np.tril(A, -1).T
    B = np.asarray(B, dtype=dtype)
    R = alpha * (S @ B if side == "left" else B @ S)
    return R + beta * np.asarray(C, dtype=dtype) if (C is not None and beta != 0.0) else R


def trmm(alpha, A, B, side="left", uplo="upper", trans=False, diag="nonunit", dtype=np.float64):
    """trnblas/level3.py:383-417: alpha * op(tri(A)) @ B or alpha * B @ op(tri(A))."""
    A = np.asarray(A, dtype=dtype)
    T = np.triu(A) if uplo == "upper" else np.tril(A)
    if diag == "unit":
        T = T - np.diag(np.diag(T)) + np.eye(A.shape[0], dtype=dtype)
    M = T.T if trans else T
    B = np.asarray(B, dtype=dtype)
    return alpha * (M @ B if side == "left" else B @ M)
