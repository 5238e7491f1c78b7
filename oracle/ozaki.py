"""Oracle: Ozaki fp64-class GEMM, in numpy -- TEST INFRASTRUCTURE.

Restates the reference trnblas/ozaki.py (0.13.0):
- constants            ozaki.py:42-48 (7-bit digits, TILE_K 128, GROUP_TERMS 4096);
- split                ozaki.py:123-219: per row (or column) exponent e from
                       frexp of the max magnitude, digit 0 = rint(X 2^(6-e)),
                       each next digit rint(128 * remainder), |digit| <= 64;
- diag_groups/schedule ozaki.py:337-365 and exponent_offset :373-375;
- reference_from_digits ozaki.py:389-415 with _two_sum32 :378-386 (the
                       reference's fp32 TwoSum group walk, for pinning);
- combine              ozaki.py:418-455.

`gemm_diag` is the arithmetic of the B200 kernel (trnblas_b200 csrc/ozaki.cu),
restated so its output can be checked bit for bit: every diagonal
d = s + t of slice products is an exact integer sum (int64 here, int32 on the
tensor cores), and the fp64 result is
    acc = sum over d = k-1 .. 0 (smallest first) of fl(acc + S_d * 2^(7 (k-1-d)))
    C   = acc * 2^(eA_i + eB_j + exponent_offset(k)).
"""

from __future__ import annotations

import numpy as np

SLICE_BITS = 7
TILE_K = 128
GROUP_TERMS = 4096
GROUP_TILES = GROUP_TERMS // TILE_K
MIN_SLICES, MAX_SLICES, DEFAULT_SLICES = 1, 12, 8


def check_slices(slices) -> int:
    """ozaki.py:51-58."""
    if isinstance(slices, bool) or not isinstance(slices, (int, np.integer)):
        raise TypeError(f"slices must be an int, got {type(slices).__name__}")
    k = int(slices)
    if not MIN_SLICES <= k <= MAX_SLICES:
        raise ValueError(f"slices must be in [{MIN_SLICES}, {MAX_SLICES}], got {k}")
    return k


def n_products(k: int) -> int:
    return k * (k + 1) // 2


def exponent_offset(k: int) -> int:
    """ozaki.py:373-375."""
    return -2 * (SLICE_BITS - 1) - SLICE_BITS * (k - 1)


def split_rows(X: np.ndarray, k: int):
    """Digits (k, R, C) float64 (integers, |d| <= 64) and exponents (R,) int64
    of a per-row split of X (R, C) (ozaki.py:123-219 with per="row")."""
    k = check_slices(k)
    X = np.ascontiguousarray(X, dtype=np.float64)
    R, C = X.shape
    if R == 0 or C == 0:
        return np.zeros((k, R, C)), np.zeros(R, dtype=np.int64)
    amax = np.maximum(X.max(axis=1), -X.min(axis=1))
    e = np.frexp(amax)[1].astype(np.int64)  # amax < 2^e; amax == 0 -> 0
    shift = (SLICE_BITS - 1) - e
    if shift.max() <= 1023 and shift.min() >= -1022:
        scales = [np.ldexp(1.0, shift)]
    else:
        scales = [np.ldexp(1.0, shift // 2), np.ldexp(1.0, shift - shift // 2)]
    Rb = X * scales[0][:, None]
    for f in scales[1:]:
        Rb = Rb * f[:, None]
    D = np.empty((k, R, C))
    for s in range(k):
        if s:
            Rb = Rb * float(1 << SLICE_BITS)
        d = np.rint(Rb)
        if s + 1 < k:
            Rb = Rb - d
        D[s] = d
    return D, e


def split_cols(X: np.ndarray, k: int):
    """Digits (k, R, C) and exponents (C,) of a per-column split (per="col")."""
    D, e = split_rows(np.ascontiguousarray(np.asarray(X, dtype=np.float64).T), k)
    return np.ascontiguousarray(D.transpose(0, 2, 1)), e


def diag_sums(DA: np.ndarray, DB: np.ndarray) -> np.ndarray:
    """Exact S_d = sum_{s+t=d} A_s @ B_t for d = 0..k-1, int64 (k, M, N).
    DA (k, M, K) row digits of A, DB (k, K, N) column digits of B."""
    k, M, K = DA.shape
    N = DB.shape[2]
    A = DA.astype(np.int64)
    B = DB.astype(np.int64)
    S = np.zeros((k, M, N), dtype=np.int64)
    for d in range(k):
        for s in range(d + 1):
            S[d] += A[s] @ B[d - s]
    return S


def combine_diag(S: np.ndarray, eA: np.ndarray, eB: np.ndarray, k: int) -> np.ndarray:
    """fp64 recombination of exact diagonal sums (the B200 kernel's order)."""
    acc = np.zeros(S.shape[1:], dtype=np.float64)
    for d in range(k - 1, -1, -1):
        acc = acc + S[d].astype(np.float64) * float(2 ** (SLICE_BITS * (k - 1 - d)))
    ea = eA.astype(np.int64) + exponent_offset(k)
    eb = eB.astype(np.int64)
    return _scale2(acc, ea[:, None] + eb[None, :])


def _scale2(v: np.ndarray, ex: np.ndarray) -> np.ndarray:
    """v * 2^ex exactly (two ldexp steps, so no intermediate over/underflows)."""
    h = ex // 2
    return np.ldexp(np.ldexp(v, h), ex - h)


def gemm_diag(A: np.ndarray, B: np.ndarray, k: int = DEFAULT_SLICES) -> np.ndarray:
    """fp64 A @ B by the B200 kernel's arithmetic (exact diagonal sums)."""
    k = check_slices(k)
    A = np.asarray(A, dtype=np.float64)
    B = np.asarray(B, dtype=np.float64)
    M, K = A.shape
    N = B.shape[1]
    if M == 0 or N == 0 or K == 0:
        return np.zeros((M, N))
    DA, eA = split_rows(A, k)
    DB, eB = split_cols(B, k)
    return combine_diag(diag_sums(DA, DB), eA, eB, k)


# ── the reference's own TwoSum walk (for pinning against reference_gemm) ─────


def diag_groups(kt: int, d: int) -> list:
    """ozaki.py:337-355."""
    if kt >= GROUP_TILES:
        return [
            [(s, d - s, k0, min(GROUP_TILES, kt - k0))]
            for s in range(d + 1)
            for k0 in range(0, kt, GROUP_TILES)
        ]
    per = GROUP_TILES // kt
    pairs = [(s, d - s) for s in range(d + 1)]
    return [[(s, t, 0, kt) for s, t in pairs[i : i + per]] for i in range(0, d + 1, per)]


def schedule(k: int, kt: int) -> list:
    """ozaki.py:358-365: diagonals smallest first."""
    return [(d, float(2 ** (SLICE_BITS * (k - 1 - d))), diag_groups(kt, d)) for d in range(k - 1, -1, -1)]


def _two_sum32(hi, lo, p):
    """ozaki.py:378-386, fp32, the kernel's op order."""
    s = hi + p
    bb = s - hi
    t = s - bb
    e1 = hi - t
    e2 = p - bb
    return s, lo + (e1 + e2)


def gemm_twosum(A: np.ndarray, B: np.ndarray, k: int = DEFAULT_SLICES) -> np.ndarray:
    """fp64 A @ B by the reference's group / fp32-TwoSum arithmetic
    (reference_from_digits ozaki.py:389-415 + combine :418-455), unblocked
    (the reference's result does not depend on the M/N blocking)."""
    k = check_slices(k)
    A = np.asarray(A, dtype=np.float64)
    B = np.asarray(B, dtype=np.float64)
    M, K = A.shape
    N = B.shape[1]
    if M == 0 or N == 0 or K == 0:
        return np.zeros((M, N))
    Kp = -(-K // TILE_K) * TILE_K
    DA, eA = split_rows(A, k)
    DB, eB = split_cols(B, k)
    At = np.zeros((k, Kp, M))
    Bp = np.zeros((k, Kp, N))
    At[:, :K] = DA.transpose(0, 2, 1)
    Bp[:, :K] = DB
    hi = lo = None
    for _d, scale, groups in schedule(k, Kp // TILE_K):
        for grp in groups:
            G = None
            for s, t, k0, n in grp:
                r0, r1 = k0 * TILE_K, (k0 + n) * TILE_K
                P = At[s, r0:r1].T @ Bp[t, r0:r1]
                G = P if G is None else G + P
            p = (G * scale).astype(np.float32)
            if hi is None:
                hi, lo = np.zeros_like(p), np.zeros_like(p)
            hi, lo = _two_sum32(hi, lo, p)
    v = hi.astype(np.float64) + lo.astype(np.float64)
    ea = eA.astype(np.int64) + exponent_offset(k)
    return _scale2(v, ea[:, None] + eB.astype(np.int64)[None, :])
