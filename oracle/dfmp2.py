"""Oracle: DF-MP2 energy end to end and the triangular solve, in numpy --
TEST INFRASTRUCTURE (imported only by tests/, smoke() and bench.py's CPU
baseline; never by the product path).

Restates the reference (trnsci/trnblas 0.13.0):
- trsm                 trnblas/level3.py:332-362 with the torch route of
                       trnblas/nki/dispatch.py:1707-1738 (only the `uplo`
                       triangle of A is read; 'unit' replaces its diagonal);
- metric_inv_half      trnblas/level3.py:365-380, dispatch.py:1877-1882:
                       X = L^-T with J = L L^T;
- df_mp2_energy        examples/df_mp2.py:147-228 (half transform
                       (i nu|P) = C_occ^T (mu nu|P), (ia|P) = C_vir^T (i nu|P),
                       B = (ia|P) X, then the pair energy of
                       oracle/pair_energy.py), which is also what
                       trnblas/parallel.py:258-353 computes with the work split
                       over ranks;
- pack_tril            trnblas/parallel.py:188-197 (row mu (mu + 1) / 2 + nu).
Pinned against the reference's own outputs in tests/golden/dfmp2.npz.
"""

from __future__ import annotations

import numpy as np

from . import pair_energy as _pe


def trsm(alpha, A, B, side="left", uplo="upper", trans=False, diag="nonunit", dtype=np.float64):
    """op(A) X = alpha B (left) or X op(A) = alpha B (right), by dense solve."""
    A = np.asarray(A, dtype=dtype)
    B = np.asarray(B, dtype=dtype)
    tri = np.triu(A) if uplo == "upper" else np.tril(A)
    if diag == "unit":
        tri = tri - np.diag(np.diag(tri)) + np.eye(A.shape[0], dtype=dtype)
    mat = tri.T if trans else tri
    if side == "left":
        return alpha * np.linalg.solve(mat, B)
    return alpha * np.linalg.solve(mat.T, B.T).T


def metric_inv_half(J, dtype=np.float64):
    L = np.linalg.cholesky(np.asarray(J, dtype=dtype))
    return trsm(1.0, L, np.eye(L.shape[0], dtype=dtype), uplo="lower", trans=True, dtype=dtype)


def df_mp2_B(C_occ, C_vir, eri_3c, J_metric, dtype=np.float64):
    """B[i, a, P] = sum_Q (ia|Q) X[Q, P] with (ia|Q) from the two half transforms."""
    C_occ = np.asarray(C_occ, dtype=dtype)
    C_vir = np.asarray(C_vir, dtype=dtype)
    eri = np.asarray(eri_3c, dtype=dtype)
    nbasis, nocc = C_occ.shape
    naux = eri.shape[-1]
    X = metric_inv_half(J_metric, dtype)
    iv = (C_occ.T @ eri.reshape(nbasis, nbasis * naux)).reshape(nocc, nbasis, naux)
    ia = np.einsum("va,ivp->iap", C_vir, iv)
    return ia @ X


def df_mp2_energy(C_occ, C_vir, eri_3c, J_metric, eps_occ, eps_vir, dtype=np.float64) -> float:
    return _pe.chunked_energy(df_mp2_B(C_occ, C_vir, eri_3c, J_metric, dtype), eps_occ, eps_vir, dtype)


def pack_tril(eri_3c) -> np.ndarray:
    eri = np.asarray(eri_3c)
    r, c = np.tril_indices(eri.shape[0])
    return eri[r, c]


def make_inputs(nbasis: int, nocc: int, naux: int, seed: int):
    """Synthetic DF-MP2 inputs with the distributions of the reference's
    example driver (examples/df_mp2.py:245-266): C ~ N(0, 0.1^2), integrals
    ~ N(0, 0.01^2), J = R R^T + naux I with R ~ N(0, 0.01^2), sorted orbital
    energies in [-1.5, -0.5) and [0.1, 1.1). numpy generator (not the
    reference's torch stream), for sizes the fixtures do not store."""
    g = np.random.default_rng(seed)
    C_occ = (g.standard_normal((nbasis, nocc)) * 0.1).astype(np.float32)
    C_vir = (g.standard_normal((nbasis, nbasis - nocc)) * 0.1).astype(np.float32)
    eri = (g.standard_normal((nbasis, nbasis, naux)) * 0.01).astype(np.float32)
    R = (g.standard_normal((naux, naux)) * 0.01).astype(np.float32)
    J = (R @ R.T + naux * np.eye(naux, dtype=np.float32)).astype(np.float32)
    eo = (-np.sort(g.random(nocc)) - 0.5).astype(np.float32)
    ev = (np.sort(g.random(nbasis - nocc)) + 0.1).astype(np.float32)
    return C_occ, C_vir, eri, J, eo, ev
