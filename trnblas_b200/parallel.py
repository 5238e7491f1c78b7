"""SPMD GEMM and DF-MP2 pair energy across GPUs, one process per GPU.

Drop-in for the reference's `trnblas.parallel` (trnblas/parallel.py:81-162):
`all_gather_rows`, `gemm_row_parallel`, `gemm_col_parallel`,
`gemm_k_parallel`, `pair_energy`, `device`. Run under
`torchrun --nproc-per-node=<gpus>` with `torch.distributed` on the NCCL
backend (NVLink 5 / NVSwitch on a B200 node). Every function is collective:
each rank of `group` calls it with the same shapes. Local products run on the
sm_100a kernels (`trnblas_b200.gemm`); data crosses GPUs only through NCCL.

Additions for B200:
- `gemm_2d`: the 2-D output-block sharded GEMM. Ranks form a pr x pc grid
  (rank = r * pc + c). A is row-sharded 1/w per rank in rank order; B is
  column-sharded 1/w per rank in grid-column-major order (shard index
  c * pr + r), so the shards a grid row / column gathers are contiguous
  blocks. NCCL all-gathers of the non-resident operand blocks run within row /
  column groups, K-chunked on a side stream so the local GEMM of chunk k
  overlaps the gather of chunk k+1. `shard_2d` slices full operands.
- `pair_energy` shards the linearised i <= j pair list by pair count (every
  pair costs the same) and sums one fp64 scalar with a single all-reduce.
The routines also run on gloo with CPU tensors when the local products are
given a CPU implementation (`_local_mm`, `_local_energy`), which is how they
are unit-tested.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import energy as _energy
from .level3 import gemm as _gemm

# Local products: the B200 kernels. CPU/gloo tests replace them.
_local_mm = None
_local_energy = None


def _mm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if _local_mm is not None:
        return _local_mm(a, b)
    return _gemm(1.0, a, b)


def device() -> torch.device:
    """This rank's device: its current GPU when CUDA is available, else the CPU."""
    if torch.cuda.is_available():
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def _rank_world(group) -> tuple[int, int]:
    return dist.get_rank(group), dist.get_world_size(group)


def _reduce_scatter(out: torch.Tensor, inp: torch.Tensor, group) -> None:
    """reduce_scatter_tensor (sum) along dim 0; all-reduce + slice on gloo
    (trnblas/parallel.py:59-68)."""
    if dist.get_backend(group) != "gloo":
        dist.reduce_scatter_tensor(out, inp, group=group)
        return
    r, w = _rank_world(group)
    full = inp.clone()
    dist.all_reduce(full, group=group)
    out.copy_(full.reshape(w, *out.shape)[r])


# ── tensor-parallel GEMM primitives (reference semantics) ────────────────────


def all_gather_rows(x: torch.Tensor, group=None) -> torch.Tensor:
    """Concatenate every rank's `x` (same shape) along dim 0, on every rank."""
    _, w = _rank_world(group)
    out = torch.empty((w * x.shape[0], *x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


def gemm_row_parallel(A_rows: torch.Tensor, B: torch.Tensor, gather: bool = False, group=None):
    """C rows = A rows @ B (A sharded along M, B replicated). With `gather`,
    every rank gets the full C (equal row counts)."""
    C = _mm(A_rows, B)
    return all_gather_rows(C, group) if gather else C


def gemm_col_parallel(A: torch.Tensor, B_cols: torch.Tensor, gather: bool = False, group=None):
    """C cols = A @ B cols (B sharded along N, A replicated). With `gather`,
    every rank gets the full C (equal shard widths)."""
    C = _mm(A, B_cols)
    if not gather:
        return C
    parts = all_gather_rows(C.T.contiguous(), group)
    return parts.T.contiguous()


def gemm_k_parallel(A_k: torch.Tensor, B_k: torch.Tensor, scatter: bool = False, group=None):
    """C = sum over ranks of A_k @ B_k (K sharded). Full C on every rank
    (all-reduce), or with `scatter` this rank's block of rows
    (reduce-scatter; M must divide by the world size)."""
    P = _mm(A_k, B_k)
    if scatter:
        _, w = _rank_world(group)
        out = torch.empty((P.shape[0] // w, P.shape[1]), dtype=P.dtype, device=P.device)
        _reduce_scatter(out, P, group)
        return out
    dist.all_reduce(P, group=group)
    return P


# ── 2-D output-block sharded GEMM ────────────────────────────────────────────


def grid_shape(world: int) -> tuple[int, int]:
    """(pr, pc) with pr * pc == world, pr <= pc, as square as possible:
    1 -> 1x1, 2 -> 1x2, 4 -> 2x2, 8 -> 2x4."""
    pr = int(math.isqrt(world))
    while world % pr:
        pr -= 1
    return pr, world // pr


class Grid2D:
    """Row / column subgroups of a pr x pc rank grid (rank = r * pc + c)."""

    def __init__(self, group=None):
        self.group = group
        self.rank, self.world = _rank_world(group)
        self.pr, self.pc = grid_shape(self.world)
        self.r, self.c = divmod(self.rank, self.pc)
        ranks = dist.get_process_group_ranks(group) if group is not None else list(range(self.world))
        self.row_group = self.col_group = None
        # every rank creates every subgroup, in the same order
        for r in range(self.pr):
            g = dist.new_group([ranks[r * self.pc + c] for c in range(self.pc)])
            if r == self.r:
                self.row_group = g
        for c in range(self.pc):
            g = dist.new_group([ranks[r * self.pc + c] for r in range(self.pr)])
            if c == self.c:
                self.col_group = g

    def block_rows(self, M: int) -> tuple[int, int]:
        """Row range of C this rank's block covers."""
        mb = M // self.pr
        return self.r * mb, (self.r + 1) * mb

    def block_cols(self, N: int) -> tuple[int, int]:
        nb = N // self.pc
        return self.c * nb, (self.c + 1) * nb


def shard_2d(A: torch.Tensor, B: torch.Tensor, grid: Grid2D):
    """This rank's (A_shard, B_shard) for `gemm_2d` from full A (M, K), B (K, N)."""
    w = grid.world
    M, N = A.shape[0], B.shape[1]
    if M % w or N % w:
        raise ValueError(f"gemm_2d needs M and N divisible by the world size {w}")
    mw, nw = M // w, N // w
    s = grid.c * grid.pr + grid.r
    return A[grid.rank * mw : (grid.rank + 1) * mw], B[:, s * nw : (s + 1) * nw]


def gemm_2d(
    A_shard: torch.Tensor,
    B_shard: torch.Tensor,
    grid: Grid2D,
    k_chunks: int = 4,
    kernel_events: list | None = None,
) -> torch.Tensor:
    """This rank's (M/pr) x (N/pc) block of C = A @ B on a pr x pc grid.

    A_shard (M/w, K): rows [rank * M/w, (rank+1) * M/w) of A.
    B_shard (K, N/w): columns of B shard index c * pr + r.
    Grid row r gathers the A shards of its pc ranks (rows of block r) and grid
    column c the B shards of its pr ranks (columns of block c), both over NCCL
    in `k_chunks` K-chunks on a side stream while the local GEMM of the
    previous chunk runs; chunk products accumulate through the fused beta = 1
    epilogue. Returns the C block (rows `grid.block_rows(M)`, columns
    `grid.block_cols(N)`). A grid row / column of one rank needs no gather.
    `kernel_events`, when given, receives a (start, end) CUDA event pair
    around each local GEMM launch on the launching stream.
    """
    pr, pc = grid.pr, grid.pc
    mw, K = A_shard.shape
    K2, nw = B_shard.shape
    if K != K2:
        raise ValueError(f"gemm_2d: A shard has K={K}, B shard K={K2}")
    k_chunks = max(1, min(int(k_chunks), max(K, 1)))
    bounds = [K * i // k_chunks for i in range(k_chunks + 1)]
    dev = A_shard.device
    cuda = dev.type == "cuda"
    comm = torch.cuda.Stream(dev) if cuda else None
    main = torch.cuda.current_stream(dev) if cuda else None

    def gather_chunk(k0, k1):
        if pc == 1:
            a_full = A_shard[:, k0:k1]
        else:
            a_part = A_shard[:, k0:k1].contiguous()
            a_full = torch.empty((pc * mw, k1 - k0), dtype=A_shard.dtype, device=dev)
            dist.all_gather_into_tensor(a_full, a_part, group=grid.row_group)
        if pr == 1:
            b_full = B_shard[k0:k1].T  # a transposed view: the kernel reads it as is
        else:
            b_part = B_shard[k0:k1].T.contiguous()  # (nw, kc)
            b_full = torch.empty((pr * nw, k1 - k0), dtype=B_shard.dtype, device=dev)
            dist.all_gather_into_tensor(b_full, b_part, group=grid.col_group)
        return a_full, b_full  # b_full holds the B block transposed (N_blk, kc)

    C = None
    pending, events = [], []
    if cuda:
        comm.wait_stream(main)
    for i in range(k_chunks):
        # issue the gather of chunk i (chunk 0 before the loop body's GEMM)
        while len(pending) <= min(i + 1, k_chunks - 1):
            j = len(pending)
            if cuda:
                with torch.cuda.stream(comm):
                    pending.append(gather_chunk(bounds[j], bounds[j + 1]))
                e = torch.cuda.Event()
                e.record(comm)
                events.append(e)
            else:
                pending.append(gather_chunk(bounds[j], bounds[j + 1]))
        if cuda:
            main.wait_event(events[i])
        a_full, b_full_t = pending[i]
        if cuda:
            a_full.record_stream(main)
            b_full_t.record_stream(main)
        if _local_mm is not None:
            part = _local_mm(a_full, b_full_t.T)
            C = part if C is None else C + part
        else:
            if kernel_events is not None:
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                ev0.record(main)
            C = _gemm(1.0, a_full, b_full_t, 1.0 if C is not None else 0.0, C, transB=True)
            if kernel_events is not None:
                ev1.record(main)
                kernel_events.append((ev0, ev1))
        pending[i] = None
    if C is None:
        C = torch.zeros((pc * mw, pr * nw), dtype=A_shard.dtype, device=dev)
    return C


# ── DF-MP2 pair energy ───────────────────────────────────────────────────────


def pair_energy(
    B_full: torch.Tensor, eps_occ: torch.Tensor, eps_vir: torch.Tensor, group=None
) -> float:
    """MP2 pair energy with the occupied pairs split over the ranks.

    `B_full` (nocc, nvir, naux) is on this rank's device on every rank, as in
    the reference (trnblas/parallel.py:126-162). Rank r computes the r-th
    pair-count-balanced range of the i <= j pair list on the fused kernel;
    one all-reduce of an fp64 scalar sums them (fp64: the kernel's 1e-9
    relative accuracy would not survive an fp32 sum). Returns a float on
    every rank.
    """
    r, w = _rank_world(group)
    nocc = B_full.shape[0]
    p0, p1 = _energy.pair_ranges(nocc, w)[r]
    if _local_energy is not None:
        e = torch.as_tensor(_local_energy(B_full, eps_occ, eps_vir, p0, p1), dtype=torch.float64).reshape(1)
    else:
        e = _energy.pair_range_energy(B_full, eps_occ, eps_vir, p0, p1).reshape(1)
    dist.all_reduce(e, group=group)
    return float(e.cpu())


__all__ = [
    "Grid2D",
    "all_gather_rows",
    "device",
    "gemm_2d",
    "gemm_col_parallel",
    "gemm_k_parallel",
    "gemm_row_parallel",
    "grid_shape",
    "pair_energy",
    "shard_2d",
]
