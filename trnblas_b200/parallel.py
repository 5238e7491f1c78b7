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
- `df_mp2_energy` is the whole DF-MP2 energy from MO coefficients, 3-centre
  integrals and the metric (trnblas/parallel.py:258-353): every rank uploads
  its rows of the integrals and half-transforms them, a reduce-scatter sums
  the partials over occupied rows, the metric factor is broadcast, each rank
  forms its rows of B, B is all-gathered and the pair energy split as above.
The routines also run on gloo with CPU tensors when the local products are
given a CPU implementation (`_local_mm`, `_local_energy`), which is how they
are unit-tested.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

import time

from . import energy as _energy
from .level3 import batched_gemm as _batched_gemm
from .level3 import gemm as _gemm
from .level3 import metric_inv_half as _metric_inv_half

# Local products: the B200 kernels. CPU/gloo tests replace them.
_local_mm = None
_local_bmm = None
_local_metric = None
_local_energy = None


def _mm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if _local_mm is not None:
        return _local_mm(a, b)
    return _gemm(1.0, a, b)


def _bmm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if _local_bmm is not None:
        return _local_bmm(a, b)
    return _batched_gemm(1.0, a, b)


def device() -> torch.device:
    """This rank's device: its current GPU when CUDA is available, else the CPU."""
    if torch.cuda.is_available():
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def _rank_world(group) -> tuple[int, int]:
    return dist.get_rank(group), dist.get_world_size(group)


def _distributed() -> bool:
    return dist.is_available() and dist.is_initialized()


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


def _panel_gemm(a: torch.Tensor, b_stack: torch.Tensor, pieces: int, C: torch.Tensor, beta: float) -> None:
    """C[:, r*nw:(r+1)*nw] = a @ b_stack[r] + beta * (same), r < pieces, in
    place: one batched launch of the GEMM kernel with A broadcast (batch
    stride 0), B pieces kc x nw stacked along dim 0 and D / C the column slices
    of C (batch stride nw, leading dimension pieces * nw). Each output element
    is read (beta = 1) and written by the same epilogue thread, so C may be
    its own accumulator."""
    from . import _native as N

    M, kc = a.shape
    nw = b_stack.shape[1]
    if _local_mm is not None:
        for r in range(pieces):
            blk = C[:, r * nw : (r + 1) * nw]
            part = _local_mm(a, b_stack[r * kc : (r + 1) * kc])
            blk.copy_(part if beta == 0.0 else blk + part)
        return
    code = N.dtype_code(a.dtype)
    if a.stride(1) != 1:
        a = a.contiguous()
    b_stack = b_stack.contiguous()
    lda, ldc = a.stride(0), C.stride(0)
    es = a.element_size()
    tma_ok = all(v % 16 == 0 for v in (lda * es, nw * es, kc * nw * es, a.data_ptr(), b_stack.data_ptr()))
    if code != N.F32 and not tma_ok:
        # ragged 16-bit shapes (strides off the 16-byte TMA grid): per slab
        # through the public GEMM, which pads such operands
        for r in range(pieces):
            blk = C[:, r * nw : (r + 1) * nw]
            part = _gemm(1.0, a, b_stack[r * kc : (r + 1) * kc])
            if beta == 0.0:
                blk.copy_(part)
            else:
                blk.add_(part)
        return
    dev = a.device
    ws_bytes = N.lib().trnblas_gemm_workspace_size(code, pieces, M, nw, kc, 0, kc * nw)
    ws = N.workspace(ws_bytes, dev)
    rc = N.lib().trnblas_gemm(
        code, pieces, M, nw, kc, 1.0,
        N.ptr(a), lda, 0, 0,
        N.ptr(b_stack), nw, kc * nw, 0,
        float(beta), N.ptr(C) if beta != 0.0 else None, ldc, nw,
        N.ptr(C), ldc, nw,
        N.ptr(ws), ws_bytes, N.stream_ptr(dev),
    )
    N.check(rc, "trnblas_gemm")
    N.count_launches(3 if code == N.F32 else 1)


# ── operand exchange over NVLink by the copy engines (gemm_2d "p2p") ──────────

_READY = {}      # device index -> (int32 flags tensor, last epoch)
_COPY_STREAMS = {}  # device index -> copy streams
_N_COPY_STREAMS = 4


def _ready_flags(dev: torch.device, n: int):
    """This device's readiness flags (at least n) and a fresh epoch."""
    flags, epoch = _READY.get(dev.index, (None, 0))
    if flags is None or flags.numel() < n:
        flags = torch.zeros(max(64, n), dtype=torch.int32, device=dev)
    epoch = (epoch + 1) & 0x7FFFFFFF or 1
    _READY[dev.index] = (flags, epoch)
    return flags, epoch


def _copy_streams(dev: torch.device):
    if dev.index not in _COPY_STREAMS:
        _COPY_STREAMS[dev.index] = [torch.cuda.Stream(dev) for _ in range(_N_COPY_STREAMS)]
    return _COPY_STREAMS[dev.index]


def _rendezvous(dev: torch.device, group) -> None:
    """A one-element all-reduce on the current stream: every rank's earlier
    stream work is done before any rank's later work runs."""
    t = torch.zeros(1, dtype=torch.int32, device=dev)
    dist.all_reduce(t, group=group)


def _exchange_shards(A_shard: torch.Tensor, B_shard: torch.Tensor, grid: Grid2D):
    """Every rank's (A shard, B shard) pointers, mapped into this process
    (CUDA IPC), or None on every rank when any rank cannot export (the
    decision is collective, so all ranks then take the NCCL path)."""
    import ctypes

    from . import _native as N

    rec = torch.zeros(2 * 72 + 1, dtype=torch.uint8)
    ok = True
    for k, t in enumerate((A_shard, B_shard)):
        h = (ctypes.c_char * 64)()
        off = ctypes.c_int64()
        if N.lib().trnblas_ipc_export(t.data_ptr(), h, ctypes.byref(off)) != 0:
            ok = False
            break
        rec[72 * k : 72 * k + 64] = torch.frombuffer(bytearray(h.raw), dtype=torch.uint8)
        rec[72 * k + 64 : 72 * k + 72] = torch.frombuffer(bytearray(off.value.to_bytes(8, "little", signed=True)),
                                                          dtype=torch.uint8)
    rec[-1] = 1 if ok else 0
    allrec = torch.empty((grid.world, rec.numel()), dtype=torch.uint8, device=A_shard.device)
    dist.all_gather_into_tensor(allrec, rec.to(A_shard.device), group=grid.group)
    allrec = allrec.cpu()
    if not bool(allrec[:, -1].all()):
        return None
    ptrs = []
    for r in range(grid.world):
        if r == grid.rank:
            ptrs.append((A_shard.data_ptr(), B_shard.data_ptr()))
            continue
        pair = []
        for k in range(2):
            hb = bytes(allrec[r, 72 * k : 72 * k + 64].tolist())
            off = int.from_bytes(bytes(allrec[r, 72 * k + 64 : 72 * k + 72].tolist()), "little", signed=True)
            p = ctypes.c_void_p()
            N.check(N.lib().trnblas_ipc_open(hb, off, ctypes.byref(p)), "trnblas_ipc_open")
            pair.append(p.value)
        ptrs.append(tuple(pair))
    return ptrs


def _gemm_2d_p2p(A_shard, B_shard, grid: Grid2D, kernel_events=None):
    """gemm_2d with the operand exchange overlapped with the GEMM: the shards
    of this rank's grid row (A) and grid column (B) are copied into local
    buffers by the copy engines (peer shards pulled over NVLink; no SM, so
    nothing competes with the GEMM's persistent CTAs), each copy raising a
    ready flag, while ONE GEMM launch (trnblas_gemm_ready) multiplies: its
    producer waits for the flags of a tile's A rows and B slab before loading
    them, and the tile walk starts on this rank's own shards. Returns None
    (nothing launched) when the shards cannot be shared; the caller then
    gathers with NCCL."""
    from . import _native as N

    dev = A_shard.device
    pr, pc = grid.pr, grid.pc
    mw, K = A_shard.shape
    nw = B_shard.shape[1]
    main = torch.cuda.current_stream(dev)
    # every rank's shards are written before any peer reads them
    _rendezvous(dev, grid.group)
    ptrs = _exchange_shards(A_shard, B_shard, grid)
    if ptrs is None:
        return None
    es = A_shard.element_size()
    a_full = torch.empty((pc * mw, K), dtype=A_shard.dtype, device=dev)
    b_full = torch.empty((pr * K, nw), dtype=B_shard.dtype, device=dev)
    C = torch.empty((pc * mw, pr * nw), dtype=A_shard.dtype, device=dev)
    flags, epoch = _ready_flags(dev, pc + pr)
    streams = _copy_streams(dev)
    for st in streams:
        st.wait_stream(main)
    row_ranks = [grid.r * pc + c for c in range(pc)]  # A shard c' of block row r
    col_ranks = [r * pc + grid.c for r in range(pr)]  # B slab r' of block column c
    jobs = [("a", grid.c), ("b", grid.r)]
    jobs += [("b", (grid.r + d) % pr) for d in range(1, pr)]
    jobs += [("a", (grid.c + d) % pc) for d in range(1, pc)]
    a_bytes, b_bytes = mw * K * es, K * nw * es
    for n, (kind, idx) in enumerate(jobs):
        st = streams[n % len(streams)]
        if kind == "a":
            dst, src, nbytes, flag = a_full.data_ptr() + idx * a_bytes, ptrs[row_ranks[idx]][0], a_bytes, idx
        else:
            dst, src, nbytes, flag = b_full.data_ptr() + idx * b_bytes, ptrs[col_ranks[idx]][1], b_bytes, pc + idx
        N.check(N.lib().trnblas_copy_async(dst, src, nbytes, st.cuda_stream), "trnblas_copy_async")
        N.check(N.lib().trnblas_stream_signal(flags.data_ptr() + 4 * flag, epoch, st.cuda_stream),
                "trnblas_stream_signal")
    for t in (a_full, b_full, flags):
        for st in streams:
            t.record_stream(st)
    if kernel_events is not None:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(main)
    code = N.dtype_code(A_shard.dtype)
    rc = N.lib().trnblas_gemm_ready(
        code, pr, pc * mw, nw, K, 1.0,
        a_full.data_ptr(), K, 0, 0,
        b_full.data_ptr(), nw, K * nw, 0,
        0.0, None, 0, 0,
        C.data_ptr(), pr * nw, nw,
        flags.data_ptr(), epoch, mw, pc, grid.c * mw, grid.r, main.cuda_stream,
    )
    N.check(rc, "trnblas_gemm_ready")
    N.count_launches(1)
    if kernel_events is not None:
        ev1.record(main)
        kernel_events.append((ev0, ev1))
    for st in streams:
        main.wait_stream(st)
    # every peer has finished pulling from this rank's shards before the
    # caller may release or overwrite them
    _rendezvous(dev, grid.group)
    return C


def _p2p_eligible(A_shard, B_shard, grid: Grid2D, k_chunks: int) -> bool:
    import os

    return (
        os.environ.get("TRNBLAS_B200_P2P", "1") != "0"
        and A_shard.device.type == "cuda"
        and A_shard.dtype in (torch.bfloat16, torch.float16)
        and B_shard.dtype == A_shard.dtype
        and grid.world > 1
        and k_chunks == 1
        and _local_mm is None
        and dist.get_backend(grid.group) == "nccl"
        and A_shard.shape[0] % 256 == 0
        and A_shard.shape[1] % 8 == 0
        and B_shard.shape[1] % 8 == 0
    )


def gemm_2d(
    A_shard: torch.Tensor,
    B_shard: torch.Tensor,
    grid: Grid2D,
    k_chunks: int = 1,
    kernel_events: list | None = None,
    transport: str = "auto",
) -> torch.Tensor:
    """This rank's (M/pr) x (N/pc) block of C = A @ B on a pr x pc grid.

    A_shard (M/w, K): rows [rank * M/w, (rank+1) * M/w) of A.
    B_shard (K, N/w): columns of B shard index c * pr + r.
    Grid row r gathers the A shards of its pc ranks (rows of block r) and grid
    column c the B shards of its pr ranks (columns of block c) over NCCL, in
    `k_chunks` K-chunks on a side stream, each chunk's gather issued before the
    previous chunk's GEMM. B shards are gathered as they lie (kc x N/w row
    slabs, stacked along dim 0: no transposed copies) and multiplied by one
    batched launch that writes each slab's columns of the C block in place;
    later chunks accumulate through the fused beta = 1 epilogue. Returns the C
    block (rows `grid.block_rows(M)`, columns `grid.block_cols(N)`). A grid
    row / column of one rank needs no gather. `kernel_events`, when given,
    receives a (start, end) CUDA event pair around each local GEMM launch on
    the launching stream.

    transport "auto" (default) exchanges the shards of 16-bit operands on
    GPUs by copy-engine pulls over NVLink overlapped with one GEMM launch
    (`_gemm_2d_p2p`) and otherwise with NCCL all-gathers; "nccl" forces the
    latter (TRNBLAS_B200_P2P=0 disables the former).
    """
    pr, pc = grid.pr, grid.pc
    mw, K = A_shard.shape
    K2, nw = B_shard.shape
    if K != K2:
        raise ValueError(f"gemm_2d: A shard has K={K}, B shard K={K2}")
    k_chunks = max(1, min(int(k_chunks), max(K // 16, 1)))
    # chunk bounds on multiples of 16 elements, so gathered chunks keep
    # 16-byte aligned rows for the TMA loads
    bounds = [min(K, (K * i // k_chunks) // 16 * 16) for i in range(k_chunks)] + [K]
    dev = A_shard.device
    cuda = dev.type == "cuda"
    comm = torch.cuda.Stream(dev) if cuda else None
    main = torch.cuda.current_stream(dev) if cuda else None
    A_shard = A_shard if A_shard.stride(1) == 1 else A_shard.contiguous()
    B_shard = B_shard.contiguous()
    if transport == "auto" and K > 0 and _p2p_eligible(A_shard.contiguous(), B_shard, grid, k_chunks):
        C = _gemm_2d_p2p(A_shard.contiguous(), B_shard, grid, kernel_events)
        if C is not None:
            return C

    def gather_chunk(k0, k1):
        whole = k0 == 0 and k1 == K
        if pc == 1:
            a_full = A_shard[:, k0:k1]
        else:
            a_part = A_shard if whole else A_shard[:, k0:k1].contiguous()
            a_full = torch.empty((pc * mw, k1 - k0), dtype=A_shard.dtype, device=dev)
            dist.all_gather_into_tensor(a_full, a_part, group=grid.row_group)
        if pr == 1:
            b_full = B_shard[k0:k1]
        else:
            b_full = torch.empty((pr * (k1 - k0), nw), dtype=B_shard.dtype, device=dev)
            dist.all_gather_into_tensor(b_full, B_shard[k0:k1], group=grid.col_group)
        return a_full, b_full  # b_full: pr slabs (kc x nw) of the column block

    C = torch.empty((pc * mw, pr * nw), dtype=A_shard.dtype, device=dev)
    if K == 0:
        return C.zero_()
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
        a_full, b_full = pending[i]
        if cuda:
            a_full.record_stream(main)
            b_full.record_stream(main)
        if kernel_events is not None:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(main)
        _panel_gemm(a_full, b_full, pr, C, 0.0 if i == 0 else 1.0)
        if kernel_events is not None:
            ev1.record(main)
            kernel_events.append((ev0, ev1))
        pending[i] = None
    return C


# ── DF-MP2 pair energy ───────────────────────────────────────────────────────


def _replicate_host_rows(x: torch.Tensor, group=None) -> torch.Tensor:
    """A host tensor that every rank needs whole on its device: rank r copies
    rows [r q, (r + 1) q) (q = ceil(rows / w)) to its device and one
    all-gather assembles all rows on every rank, so the host links carry the
    tensor once in all instead of once per rank (the ranks' uploads share the
    host's memory bandwidth; NVLink carries the rest)."""
    r, w = _rank_world(group)
    n = x.shape[0]
    q = -(-n // w)
    part = torch.zeros((q, *x.shape[1:]), dtype=x.dtype, device=device())
    r0, r1 = min(r * q, n), min((r + 1) * q, n)
    if r1 > r0:
        part[: r1 - r0].copy_(x[r0:r1], non_blocking=True)
    return all_gather_rows(part, group)[:n]


def pair_energy(
    B_full: torch.Tensor, eps_occ: torch.Tensor, eps_vir: torch.Tensor, group=None
) -> float:
    """MP2 pair energy with the occupied pairs split over the ranks.

    `B_full` (nocc, nvir, naux) is on this rank's device on every rank, as in
    the reference (trnblas/parallel.py:126-162); a host `B_full` (the same
    on every rank) is uploaded a 1/w slice per rank and all-gathered. Rank r computes the r-th
    pair-count-balanced range of the i <= j pair list on the fused kernel;
    one all-reduce of an fp64 scalar sums them (fp64: the kernel's 1e-9
    relative accuracy would not survive an fp32 sum). Returns a float on
    every rank.
    """
    r, w = _rank_world(group) if _distributed() else (0, 1)
    if w > 1 and B_full.device.type == "cpu":
        B_full = _replicate_host_rows(B_full, group)
    nocc = B_full.shape[0]
    p0, p1 = _energy.pair_ranges(nocc, w)[r]
    if _local_energy is not None:
        e = torch.as_tensor(_local_energy(B_full, eps_occ, eps_vir, p0, p1), dtype=torch.float64).reshape(1)
    else:
        e = _energy.pair_range_energy(B_full, eps_occ, eps_vir, p0, p1).reshape(1)
    if w > 1:
        dist.all_reduce(e, group=group)
    return float(e.cpu())


# ── DF-MP2 energy end to end ─────────────────────────────────────────────────


def pack_tril(eri_3c: torch.Tensor) -> torch.Tensor:
    """(nbasis, nbasis, naux) integrals symmetric in the first two indices ->
    their packed lower triangle (npair, naux), pair (mu, nu <= mu) at row
    mu (mu + 1) / 2 + nu (PySCF's pack_tril order; its `_cderi` is this
    transposed), as trnblas/parallel.py:188-197."""
    n = eri_3c.shape[0]
    r, c = torch.tril_indices(n, n, device=eri_3c.device)
    return eri_3c[r, c]


def _eri_rows(nbasis: int, parts: int, symmetric: bool) -> list[tuple[int, int]]:
    """`parts` contiguous ranges of mu balanced by the bytes each uploads: a
    full row weighs nbasis, a packed lower-triangle row mu + 1."""
    weights = [mu + 1 if symmetric else 1 for mu in range(nbasis)]
    total = sum(weights)
    bounds, acc, start = [], 0, 0
    for mu, wt in enumerate(weights):
        acc += wt
        if len(bounds) < parts - 1 and acc * parts >= total * (len(bounds) + 1):
            bounds.append((start, mu + 1))
            start = mu + 1
    bounds.append((start, nbasis))
    while len(bounds) < parts:
        bounds.append((nbasis, nbasis))
    return bounds


def _rows_lower_triangle(eri_3c: torch.Tensor, m0: int, m1: int, nbasis: int, dev) -> torch.Tensor:
    """Rows mu in [m0, m1) as (n_r, nbasis, naux) on `dev` with (mu nu|P) for
    nu <= mu and zeros above the diagonal, uploading only the lower triangle
    (`eri_3c` full (nbasis, nbasis, naux) or packed (npair, naux))."""
    p0, p1 = m0 * (m0 + 1) // 2, m1 * (m1 + 1) // 2
    if eri_3c.dim() == 2:
        packed = eri_3c[p0:p1]
    else:
        packed = torch.cat([eri_3c[mu, : mu + 1] for mu in range(m0, m1)])
    naux = packed.shape[-1]
    buf = torch.zeros((p1 - p0 + 1, naux), dtype=torch.float32, device=dev)  # last row stays zero
    buf[: p1 - p0].copy_(packed)
    mu = torch.arange(m0, m1, device=dev)
    nu = torch.arange(nbasis, device=dev)
    src = (mu * (mu + 1) // 2 - p0)[:, None] + nu[None, :]
    src = torch.where(nu[None, :] <= mu[:, None], src, torch.full_like(src, p1 - p0))
    return buf.index_select(0, src.reshape(-1)).reshape(m1 - m0, nbasis, naux)


def _half_transform_part(Cp: torch.Tensor, eri_3c: torch.Tensor, rows, dev, symmetric: bool, nbasis: int):
    """This rank's share of (i nu|P) = sum_mu C[mu, i] (mu nu|P), summed over
    its rows mu of the integrals: (nocc_pad, nbasis * naux) on `dev`.

    With `symmetric`, (mu nu|P) = (nu mu|P) and only the lower triangle of
    the rows is uploaded; the mirrored entries (nu < mu) contribute through the
    same data: sum_{nu < mu} C[nu, i] (mu nu|P) is added to (i mu|P)."""
    naux = eri_3c.shape[-1]
    m0, m1 = rows
    n_r = m1 - m0
    nocc_pad = Cp.shape[1]
    if n_r == 0:
        return torch.zeros((nocc_pad, nbasis * naux), dtype=torch.float32, device=dev)
    Cr = Cp[m0:m1].to(dev)  # (n_r, nocc_pad)
    if not symmetric:
        eri_r = eri_3c[m0:m1].reshape(n_r, nbasis * naux).to(dev, torch.float32)
        return _mm(Cr.T, eri_r)
    L = _rows_lower_triangle(eri_3c, m0, m1, nbasis, dev)  # (n_r, nbasis, naux)
    part = _mm(Cr.T, L.reshape(n_r, nbasis * naux))  # the nu <= mu terms
    # mirrored terms for every mu of the range: C^T (nocc_pad, nbasis) @ L[mu]
    # counts nu <= mu; the diagonal nu == mu is already in `part`
    CT = Cp.T.contiguous().to(dev)
    Mr = _bmm(CT.unsqueeze(0).expand(n_r, nocc_pad, nbasis), L)  # (n_r, nocc_pad, naux)
    diag = L[torch.arange(n_r, device=dev), torch.arange(m0, m1, device=dev)]  # (n_r, naux)
    Mr = Mr - Cr.unsqueeze(2) * diag.unsqueeze(1)
    part.view(nocc_pad, nbasis, naux)[:, m0:m1, :] += Mr.permute(1, 0, 2)
    return part


def df_mp2_energy(
    C_occ: torch.Tensor,
    C_vir: torch.Tensor,
    eri_3c: torch.Tensor,
    J_metric: torch.Tensor,
    eps_occ: torch.Tensor,
    eps_vir: torch.Tensor,
    group=None,
    timings: dict | None = None,
    eri_symmetric: bool = False,
) -> float:
    """DF-MP2 correlation energy, split over the ranks of `group`
    (trnblas/parallel.py:258-353; examples/df_mp2.py:147-228 on one GPU).

    C_occ (nbasis, nocc), C_vir (nbasis, nvir), eri_3c (nbasis, nbasis,
    naux) three-centre integrals (mu nu|P), J_metric (naux, naux) SPD, the
    orbital energies; host or device tensors, the same on every rank (each
    rank reads only its rows of eri_3c). `eri_symmetric=True` declares
    (mu nu|P) = (nu mu|P): only lower triangles are read and uploaded, and
    eri_3c may then be the packed (npair, naux) triangle of `pack_tril`.
    Without an initialised process group it runs on this process's GPU.
    Returns the energy (a float) on every rank; `timings` receives seconds
    per stage under the reference's keys.

    Dataflow (r = rank, w = world size):
    1+2a. rank 0 forms X = J^-1/2 (`metric_inv_half`, Cholesky + blocked
          trsm); every rank uploads its byte-balanced rows mu_r of the
          integrals and forms its partial (i nu|P) = C_occ[mu_r]^T (mu_r nu|P)
          on the GEMM kernel (each GPU has its own host link, so unlike the
          reference no rank is kept off the upload);
    2b.   a reduce-scatter over occupied rows (padded to a multiple of w)
          leaves rank r its occ_r rows of (i nu|P); X is broadcast;
    3.    (ia|P) = C_vir^T (i nu|P) (batched GEMM, C_vir^T broadcast) and
          B = (ia|P) X for those rows;
    4.    B is all-gathered and the fused pair-energy kernel sums the rank's
          pair range; one fp64 all-reduce.
    All products are fp32 on the tensor cores (3xTF32), as the reference's
    fp32 pipeline.
    """
    if eri_3c.dim() == 2 and not eri_symmetric:
        raise ValueError("a packed (npair, naux) eri_3c needs eri_symmetric=True")
    multi = _distributed()
    r, w = _rank_world(group) if multi else (0, 1)
    dev = device()
    nbasis, nocc = C_occ.shape
    nvir = C_vir.shape[1]
    naux = J_metric.shape[0]
    occ_r = -(-nocc // w)
    nocc_pad = occ_r * w
    t = {}
    clock = [time.perf_counter()]

    def mark(name):
        if timings is not None:
            if dev.type == "cuda":
                torch.cuda.synchronize(dev)
            now = time.perf_counter()
            t[name] = now - clock[0]
            clock[0] = now

    X = torch.empty((naux, naux), dtype=torch.float32, device=dev)
    if r == 0:
        Jd = J_metric.to(dev, torch.float32)
        X.copy_(_local_metric(Jd) if _local_metric is not None else _metric_inv_half(Jd))
    Cp = torch.zeros((nbasis, nocc_pad), dtype=torch.float32)
    Cp[:, :nocc] = C_occ.detach().to("cpu", torch.float32)
    rows = _eri_rows(nbasis, w, eri_symmetric)[r]
    part = _half_transform_part(Cp, eri_3c, rows, dev, eri_symmetric, nbasis)
    mark("chol_upload_2a")
    if w > 1:
        iv_r = torch.empty((occ_r, nbasis * naux), dtype=torch.float32, device=dev)
        _reduce_scatter(iv_r, part, group)
        del part
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast(X, src, group=group)
    else:
        iv_r = part
    mark("rs_iv_bcast_X")

    CvT = C_vir.detach().T.to(dev, torch.float32).contiguous()  # (nvir, nbasis)
    ia_r = _bmm(CvT.unsqueeze(0).expand(occ_r, nvir, nbasis), iv_r.reshape(occ_r, nbasis, naux))
    del iv_r
    B_r = _mm(ia_r.reshape(occ_r * nvir, naux), X).reshape(occ_r, nvir, naux)
    del ia_r
    mark("local_2b_3")

    B_full = (all_gather_rows(B_r, group) if w > 1 else B_r)[:nocc].contiguous()
    del B_r
    mark("ag_B")
    eo = eps_occ.detach().to(dev, torch.float32)
    ev = eps_vir.detach().to(dev, torch.float32)
    e = pair_energy(B_full, eo, ev, group)
    mark("energy")
    if timings is not None:
        timings.update(t)
    return e


__all__ = [
    "Grid2D",
    "all_gather_rows",
    "device",
    "df_mp2_energy",
    "gemm_2d",
    "gemm_col_parallel",
    "gemm_k_parallel",
    "gemm_row_parallel",
    "grid_shape",
    "pack_tril",
    "pair_energy",
    "shard_2d",
]
