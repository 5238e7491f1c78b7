"""DF-MP2 pair energy on B200: the fused int8 tensor-core kernel.

Replaces the reference's energy entry points
(`trnblas.nki.dispatch.nki_batched_pair_energy`, trnblas/nki/dispatch.py:
2537-2569, and the per-row kernels behind `multicore.sym_rows` / `aten_rows`,
trnblas/nki/multicore.py:212-289). One launch computes a contiguous range of
the linearised occupied-pair list (i <= j, p = j (j + 1) / 2 + i), so an SPMD
rank takes any balanced slice of it.
"""

from __future__ import annotations

import torch

from . import _native as N
from .level3 import _cuda_device, _to


def n_pairs(nocc: int) -> int:
    """Occupied pairs i <= j."""
    return nocc * (nocc + 1) // 2


def pair_ranges(nocc: int, parts: int) -> list[tuple[int, int]]:
    """`parts` contiguous ranges of the pair list, balanced by pair count
    (every pair costs the same 2 nvir^2 naux)."""
    total = n_pairs(nocc)
    parts = max(1, int(parts))
    return [(total * r // parts, total * (r + 1) // parts) for r in range(parts)]


def _energy_operands(B: torch.Tensor, eps_occ: torch.Tensor, eps_vir: torch.Tensor):
    if B.dim() != 3:
        raise ValueError(f"pair energy expects B of shape (nocc, nvir, naux), got {tuple(B.shape)}")
    nocc, nvir, _ = B.shape
    if eps_occ.numel() != nocc or eps_vir.numel() != nvir:
        raise ValueError(
            f"eps_occ / eps_vir must have nocc={nocc} / nvir={nvir} entries, "
            f"got {eps_occ.numel()} / {eps_vir.numel()}"
        )
    for name, t in (("B", B), ("eps_occ", eps_occ), ("eps_vir", eps_vir)):
        if not t.is_floating_point():
            raise TypeError(f"pair energy: {name} must be a real floating tensor, got {t.dtype}")
    dev = _cuda_device(B, eps_occ, eps_vir)
    Bd = _to(B.detach(), dev).to(torch.float32).contiguous()
    eo = _to(eps_occ.detach(), dev).to(torch.float32).reshape(-1).contiguous()
    ev = _to(eps_vir.detach(), dev).to(torch.float32).reshape(-1).contiguous()
    return Bd, eo, ev, dev


def pair_range_energy(
    B: torch.Tensor,
    eps_occ: torch.Tensor,
    eps_vir: torch.Tensor,
    pair_begin: int = 0,
    pair_end: int | None = None,
) -> torch.Tensor:
    """sum over pairs p in [pair_begin, pair_end) of w_p e_ij, as a 0-d float64
    tensor on the CUDA device (asynchronous; no host sync).

    e_ij = sum_ab T_ab (2 T_ab - T_ba) / (e_i + e_j - e_a - e_b), T = B_i B_j^T,
    w = 1 for i == j and 2 otherwise. B (nocc, nvir, naux) is computed as fp32.
    """
    Bd, eo, ev, dev = _energy_operands(B, eps_occ, eps_vir)
    nocc, nvir, naux = Bd.shape
    total = n_pairs(nocc)
    pair_end = total if pair_end is None else int(pair_end)
    pair_begin = int(pair_begin)
    if not 0 <= pair_begin <= pair_end <= total:
        raise ValueError(f"pair range [{pair_begin}, {pair_end}) outside [0, {total}]")
    out = torch.empty((), dtype=torch.float64, device=dev)
    ws_bytes = N.lib().trnblas_pair_energy_workspace_size(nocc, nvir, naux, pair_begin, pair_end)
    ws = N.workspace(ws_bytes, dev)
    rc = N.lib().trnblas_pair_energy(
        nocc, nvir, naux, N.ptr(Bd), N.ptr(eo), N.ptr(ev), pair_begin, pair_end,
        N.ptr(out), N.ptr(ws), ws_bytes, N.stream_ptr(dev),
    )
    N.check(rc, "trnblas_pair_energy")
    N.count_launches(7)  # 4 split kernels, the pair order, the fused energy kernel, the final sum
    return out


def batched_pair_energy(B: torch.Tensor, eps_occ: torch.Tensor, eps_vir: torch.Tensor) -> torch.Tensor:
    """Total MP2 pair energy over all occupied pairs, as a 0-d tensor on B's device.

    Same inputs and sign convention as the reference's `nki_batched_pair_energy`
    (trnblas/nki/dispatch.py:2537). The result is float64: the kernel
    accumulates in fp64 and an fp32 result would round away the 1e-9
    relative accuracy it holds.
    """
    home = B.device
    e = pair_range_energy(B, eps_occ, eps_vir)
    return e.to(home) if home != e.device else e  # a 0-d result: nothing to stream


def nki_batched_pair_energy(B: torch.Tensor, eps_occ: torch.Tensor, eps_vir: torch.Tensor) -> torch.Tensor:
    """The reference's entry point (trnblas/nki/dispatch.py:2537-2569): the
    total pair energy as a 0-d tensor on B's device in the dtype the
    reference returns, torch.promote_types(B.dtype, eps_vir.dtype)
    (`_pair_result_dtype`, dispatch.py:1334-1340; float32 for float32
    inputs). The kernel's fp64 sum is rounded to that dtype at the end;
    `batched_pair_energy` returns it unrounded."""
    e = batched_pair_energy(B, eps_occ, eps_vir)
    dt = torch.promote_types(B.dtype, eps_vir.dtype)
    return e.to(dt) if (dt.is_floating_point and e.dtype != dt) else e
