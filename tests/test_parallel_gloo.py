"""SPMD host logic on 2 gloo CPU ranks (no GPU): the reference's GEMM
primitives, the 2-D output-block GEMM and the pair-range energy split, with
the local products replaced by CPU stand-ins (torch.matmul / the oracle)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fn_name, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        import trnblas_b200.parallel as tp
        from oracle import pair_energy as PE

        tp._local_mm = torch.matmul
        tp._local_energy = lambda B, eo, ev, a, b: PE.pair_range_energy(B.numpy(), eo.numpy(), ev.numpy(), a, b)
        out = globals()[fn_name](rank, world, tp)
        q.put((rank, out))
    except Exception as e:  # report to the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _run(fn_name, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn_name, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    return [res[r] for r in range(world)]


def _primitives(rank, world, tp):
    g = torch.Generator().manual_seed(5)
    A = torch.randn(8, 6, generator=g)
    B = torch.randn(6, 10, generator=g)
    full = A @ B
    Ar = A[rank * 4 : (rank + 1) * 4]
    rows = tp.gemm_row_parallel(Ar, B, gather=True)
    Bc = B[:, rank * 5 : (rank + 1) * 5]
    cols = tp.gemm_col_parallel(A, Bc, gather=True)
    Ak, Bk = A[:, rank * 3 : (rank + 1) * 3], B[rank * 3 : (rank + 1) * 3]
    ksum = tp.gemm_k_parallel(Ak, Bk)
    kscat = tp.gemm_k_parallel(Ak, Bk, scatter=True)
    return [float((x - y).abs().max()) for x, y in ((rows, full), (cols, full), (ksum, full), (kscat, full[rank * 4 : (rank + 1) * 4]))]


def _gemm2d(rank, world, tp):
    g = torch.Generator().manual_seed(6)
    A = torch.randn(16, 12, generator=g)
    B = torch.randn(12, 20, generator=g)
    grid = tp.Grid2D()
    As, Bs = tp.shard_2d(A, B, grid)
    C = tp.gemm_2d(As, Bs, grid, k_chunks=3)
    r0, r1 = grid.block_rows(16)
    c0, c1 = grid.block_cols(20)
    return float((C - (A @ B)[r0:r1, c0:c1]).abs().max())


def _energy(rank, world, tp):
    from oracle import pair_energy as PE

    B, eo, ev = PE.make_inputs(5, 9, 12, 3)
    return tp.pair_energy(B, eo, ev)


def test_gemm_primitives_two_ranks():
    for errs in _run("_primitives"):
        assert isinstance(errs, list), errs
        assert max(errs) < 1e-5


def test_gemm_2d_two_ranks():
    for err in _run("_gemm2d"):
        assert isinstance(err, float), err
        assert err < 1e-5


def test_pair_energy_two_ranks_matches_single():
    from oracle import pair_energy as PE

    B, eo, ev = PE.make_inputs(5, 9, 12, 3)
    ref = PE.chunked_energy(B.numpy(), eo.numpy(), ev.numpy())
    es = _run("_energy")
    for e in es:
        assert isinstance(e, float), e
        assert abs(e - ref) <= 1e-12 * abs(ref)
    assert es[0] == es[1]


def test_grid_shapes():
    from trnblas_b200.parallel import grid_shape

    assert [grid_shape(w) for w in (1, 2, 4, 8, 6)] == [(1, 1), (1, 2), (2, 2), (2, 4), (2, 3)]
