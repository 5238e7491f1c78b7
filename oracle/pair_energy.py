"""Oracle: DF-MP2 pair energy, in numpy -- TEST INFRASTRUCTURE.

Restates the reference (trnsci/trnblas 0.13.0):
- _torch_chunked_pair_energy  trnblas/nki/dispatch.py:2706-2728 (the aten path:
  T_chunk = B_flat[i-chunk] @ B_flat^T, sum T (2T - T^T) / denom);
- _torch_batched_pair_energy  dispatch.py:2514-2533 (the explicit i, j loop);
- the symmetric pair walk     dispatch.py:2648-2677 (_pair_sym_dims weights:
  e_ij = e_ji, so E = sum_i e_ii + 2 sum_{i<j} e_ij);
- aten_rows / occ_chunks      trnblas/nki/multicore.py:116-125, 263-289 (row
  ranges for the SPMD split, parallel.py:126-162).
The trnblas_b200 kernel takes a contiguous range of the linearised i <= j pair
list (p = j (j + 1) / 2 + i); `pair_range_energy` is its oracle.
"""

from __future__ import annotations

import numpy as np


def chunked_energy(B, eps_occ, eps_vir, dtype=np.float64, mem_budget_bytes=1_500_000_000) -> float:
    """dispatch.py:2706-2728 in numpy (all ordered pairs, chunks of occupied rows)."""
    B = np.asarray(B, dtype=dtype)
    eo = np.asarray(eps_occ, dtype=dtype)
    ev = np.asarray(eps_vir, dtype=dtype)
    nocc, nvir, naux = B.shape
    i_block = max(1, min(nocc, int(mem_budget_bytes // (4 * nvir * nocc * nvir))))
    Bf = B.reshape(nocc * nvir, naux)
    eo_pair = eo.reshape(nocc, 1, 1, 1) + eo.reshape(1, nocc, 1, 1)
    ev_pair = ev.reshape(1, 1, nvir, 1) + ev.reshape(1, 1, 1, nvir)
    e = dtype(0.0)
    for i0 in range(0, nocc, i_block):
        i1 = min(i0 + i_block, nocc)
        T = (Bf[i0 * nvir : i1 * nvir] @ Bf.T).reshape(i1 - i0, nvir, nocc, nvir)
        T = T.transpose(0, 2, 1, 3)
        e = e + (T * (2.0 * T - np.swapaxes(T, -1, -2)) / (eo_pair[i0:i1] - ev_pair)).sum()
    return float(e)


def pair_energy_ij(B, eps_occ, eps_vir, i: int, j: int, dtype=np.float64) -> float:
    """e_ij = sum_ab T_ab (2 T_ab - T_ba) / (e_i + e_j - e_a - e_b), T = B_i B_j^T."""
    B = np.asarray(B, dtype=dtype)
    ev = np.asarray(eps_vir, dtype=dtype)
    eo = np.asarray(eps_occ, dtype=dtype)
    T = B[i] @ B[j].T
    den = eo[i] + eo[j] - ev[:, None] - ev[None, :]
    return float((T * (2.0 * T - T.T) / den).sum())


def pair_index(p: int) -> tuple[int, int]:
    """(i, j), i <= j, of linear pair index p = j (j + 1) / 2 + i."""
    j = int((np.sqrt(8.0 * p + 1.0) - 1.0) / 2.0)
    while j * (j + 1) // 2 > p:
        j -= 1
    while (j + 1) * (j + 2) // 2 <= p:
        j += 1
    return p - j * (j + 1) // 2, j


def n_pairs(nocc: int) -> int:
    return nocc * (nocc + 1) // 2


def pair_range_energy(B, eps_occ, eps_vir, pair_begin: int, pair_end: int, dtype=np.float64) -> float:
    """sum over p in [pair_begin, pair_end) of w_p e_ij (w = 1 for i == j, else 2).
    Over the whole range this equals `chunked_energy` (e_ij = e_ji)."""
    B = np.asarray(B, dtype=dtype)
    tot = 0.0
    # group by j so each block is one GEMM: rows i of pair j
    p = pair_begin
    while p < pair_end:
        i, j = pair_index(p)
        i_end = min(j + 1, i + (pair_end - p))  # pairs (i..i_end-1, j)
        Bi = B[i:i_end]  # (ni, nvir, naux)
        T = np.einsum("iap,bp->iab", Bi, B[j])
        eo = np.asarray(eps_occ, dtype=dtype)
        ev = np.asarray(eps_vir, dtype=dtype)
        den = (eo[i:i_end, None, None] + eo[j]) - ev[None, :, None] - ev[None, None, :]
        e = (T * (2.0 * T - np.swapaxes(T, -1, -2)) / den).sum(axis=(1, 2))
        w = np.where(np.arange(i, i_end) == j, 1.0, 2.0)
        tot += float((w * e).sum())
        p += i_end - i
    return tot


def occ_chunks(nocc: int, parts: int) -> list[tuple[int, int]]:
    """multicore.py:116-125: contiguous near-even ranges of occupied rows."""
    parts = max(1, min(parts, nocc))
    base, extra = divmod(nocc, parts)
    out, start = [], 0
    for c in range(parts):
        stop = start + base + (1 if c < extra else 0)
        out.append((start, stop))
        start = stop
    return out


def pair_ranges(nocc: int, parts: int) -> list[tuple[int, int]]:
    """Contiguous ranges of the i <= j pair list, balanced by pair count
    (every pair costs the same 2 nvir^2 naux)."""
    total = n_pairs(nocc)
    parts = max(1, parts)
    return [(total * r // parts, total * (r + 1) // parts) for r in range(parts)]


def make_inputs(nocc: int, nvir: int, naux: int, seed: int, sigma: float = 0.05):
    """Synthetic DF-MP2 inputs of the benchmark recipe: B ~ N(0, sigma^2)
    (nocc, nvir, naux) fp32, eps_occ sorted U[-20, -0.3], eps_vir sorted U[0.1, 5],
    drawn with torch.Generator(seed) in this order."""
    import torch

    g = torch.Generator().manual_seed(seed)
    B = (sigma * torch.randn(nocc * nvir, naux, generator=g)).reshape(nocc, nvir, naux)
    eo = torch.sort(-20.0 + 19.7 * torch.rand(nocc, generator=g)).values
    ev = torch.sort(0.1 + 4.9 * torch.rand(nvir, generator=g)).values
    return B, eo, ev


# ── the same arithmetic in torch, on any device (fp64 references at sizes
#    the numpy loops cannot reach in seconds; still test infrastructure) ──


def aten_rows_torch(B, eps_occ, eps_vir, rows, dtype=None, mem_budget_bytes: int = 1_500_000_000):
    """trnblas/nki/multicore.py:263-289 (`aten_rows`, the chunked aten energy
    of `_torch_chunked_pair_energy`, dispatch.py:2706-2728, restricted to
    occupied rows [i0, i1)): sum over i in rows and every j of e_ij, in
    `dtype` (default B's) on B's device. Same op order: T chunk = B_flat[rows]
    @ B_flat^T, permuted to (i, j, a, b), sum T (2T - T^T) / (eps_o_pair -
    eps_v_pair)."""
    import torch

    dtype = dtype or B.dtype
    B = B.to(dtype)
    eo, ev = eps_occ.to(B.device, dtype), eps_vir.to(B.device, dtype)
    nocc, nvir, naux = B.shape
    i0, i1 = rows
    i_block = max(1, min(nocc, int(mem_budget_bytes // (4 * nvir * nocc * nvir))))
    B_flat = B.reshape(nocc * nvir, naux)
    eps_o_pair = eo.view(nocc, 1, 1, 1) + eo.view(1, nocc, 1, 1)
    eps_v_pair = ev.view(1, 1, nvir, 1) + ev.view(1, 1, 1, nvir)
    e = torch.zeros((), dtype=dtype, device=B.device)
    for a in range(i0, i1, i_block):
        b = min(a + i_block, i1)
        T = (B_flat[a * nvir : b * nvir] @ B_flat.T).reshape(b - a, nvir, nocc, nvir)
        T = T.permute(0, 2, 1, 3)
        e = e + (T * (2.0 * T - T.transpose(-2, -1)) / (eps_o_pair[a:b] - eps_v_pair)).sum()
    return float(e)


def pair_range_energy_torch(B, eps_occ, eps_vir, pair_begin: int, pair_end: int, dtype=None) -> float:
    """`pair_range_energy` (sum of w_p e_ij over a range of the i <= j pair
    list) with the per-pair arithmetic of `_torch_chunked_pair_energy`
    (T = B_i B_j^T, T (2T - T^T) / (e_i + e_j - e_a - e_b)), in `dtype`
    (default B's) on B's device; one GEMM per pair row j."""
    import torch

    dtype = dtype or B.dtype
    eo, ev = eps_occ.to(B.device, dtype), eps_vir.to(B.device, dtype)
    tot = 0.0
    p = pair_begin
    while p < pair_end:
        i, j = pair_index(p)
        i_end = min(j + 1, i + (pair_end - p))
        Bi = B[i:i_end].to(dtype)
        Bj = B[j].to(dtype)
        T = (Bi.reshape(-1, Bi.shape[-1]) @ Bj.T).reshape(i_end - i, Bj.shape[0], Bj.shape[0])
        den = (eo[i:i_end].view(-1, 1, 1) + eo[j]) - ev.view(1, -1, 1) - ev.view(1, 1, -1)
        e = (T * (2.0 * T - T.transpose(-2, -1)) / den).sum(dim=(1, 2))
        w = torch.where(torch.arange(i, i_end, device=B.device) == j, 1.0, 2.0).to(dtype)
        tot += float((w * e).sum())
        p += i_end - i
    return tot
