"""BLAS level 3 on B200: gemm, batched_gemm, syrk, gemm_fp64, trsm,
metric_inv_half, symm, trmm.

Same signatures, argument meanings, return dtypes and exceptions as the
reference's trnblas/level3.py (gemm :69-109, batched_gemm :112-134, gemm_fp64
:137-193, syrk :243-295). Every float32 / bfloat16 / float16 product runs on
the sm_100a tcgen05 kernels through the C ABI (`_native`); there is no routing
table and no torch.matmul fallback for those dtypes. Host (CPU) tensors are
uploaded to the current CUDA device, computed there, and the result comes back
to the host, so a call keeps the reference's "result on the input's device"
contract. Other dtypes (float64, complex, integer) have no kernel in the
reference either; they run torch.matmul on the operands' device, as the
reference's pytorch route does (trnblas/nki/dispatch.py:321-338).
"""

from __future__ import annotations

import math
import os
import warnings

import torch

from . import _native as N
from ._flags import diag_flag, side_flag, trans_flag, uplo_flag

# ── device placement ─────────────────────────────────────────────────────────


def _cuda_device(*tensors: torch.Tensor) -> torch.device:
    """The CUDA device the kernels run on for these operands."""
    devs = {t.device for t in tensors if isinstance(t, torch.Tensor) and t.device.type == "cuda"}
    if len(devs) > 1:
        raise RuntimeError(f"trnblas_b200: operands on different CUDA devices: {sorted(map(str, devs))}")
    if devs:
        return devs.pop()
    if not torch.cuda.is_available():
        raise RuntimeError(
            "trnblas_b200 runs on NVIDIA B200 (sm_100a); no CUDA device is available"
        )
    return torch.device("cuda", torch.cuda.current_device())


def _home(r: torch.Tensor, home: torch.device, dev: torch.device) -> torch.Tensor:
    """The result on the caller's device. A host result comes down into
    pinned memory from torch's caching host allocator (a full-speed DMA; a
    pageable destination is staged and several times slower) and is returned
    once its data has arrived."""
    if home == dev:
        return r
    if home.type != "cpu" or r.numel() == 0:
        return r.to(home)
    out = torch.empty(r.shape, dtype=r.dtype, pin_memory=True)
    out.copy_(r, non_blocking=True)
    torch.cuda.current_stream(r.device).synchronize()
    return out


def _to(t, dev):
    if t is None or not isinstance(t, torch.Tensor):
        return t
    if t.device == dev:
        return t
    return t.to(dev, non_blocking=t.device.type == "cpu" and t.is_pinned())


# ── operand layout for the TMA path ─────────────────────────────────────────


def _tma_operand(x: torch.Tensor, esize: int):
    """(tensor, ld, transposed) for a 2-D logical operand x (rows x cols).

    transposed=False: x[r, c] = t[r * ld + c] (row-major, cols contiguous);
    transposed=True:  x[r, c] = t[c * ld + r] (t stores x^T row-major).
    The 16-byte TMA rule needs ld * esize % 16 == 0 and a 16-byte aligned base;
    otherwise a zero-padded row-major copy is made (small / ragged shapes only).
    """
    rows, cols = x.shape
    q = 16 // esize
    aligned = x.data_ptr() % 16 == 0
    s0, s1 = x.stride()
    if aligned and (s1 == 1 or cols == 1) and s0 % q == 0 and s0 >= cols and s0 > 0:
        return x, s0, False
    if aligned and (s0 == 1 or rows == 1) and s1 % q == 0 and s1 >= rows and s1 > 0:
        return x, s1, True
    ld = -(-max(cols, 1) // q) * q
    buf = torch.zeros((rows, ld), dtype=x.dtype, device=x.device)
    buf[:, :cols].copy_(x)
    return buf, ld, False


def _gemm2d(a: torch.Tensor, b: torch.Tensor, alpha: float, beta: float, C, tri: int = 0) -> torch.Tensor:
    """alpha * a @ b (+ beta * C when C is a same-shape, same-dtype matrix) on the kernel.
    tri: 1 / 2 when a is lower / upper triangular, 3 / 4 when b is (exact zeros
    outside the triangle): the all-zero K blocks are skipped."""
    M, K = a.shape
    K2, Nn = b.shape
    if K != K2:
        raise RuntimeError(f"mat1 and mat2 shapes cannot be multiplied ({M}x{K} and {K2}x{Nn})")
    dev = a.device
    out = torch.empty((M, Nn), dtype=a.dtype, device=dev)
    if M == 0 or Nn == 0:
        return out
    code = N.dtype_code(a.dtype)
    es = a.element_size()
    if code == N.F32:
        # The split pre-pass reads any unit-stride layout; no TMA constraints.
        at, lda, ta = _f32_operand(a)
        bt, ldb, tb = _f32_operand(b)
    else:
        # "transposed" storage of B means the tensor stores B^T (N x K) row-major.
        at, lda, ta = _tma_operand(a, es)
        bt, ldb, tb = _tma_operand(b, es)
    c_arg, ldc = None, 0
    if C is not None and beta != 0.0:
        c_arg = C if C.stride(1) == 1 and C.stride(0) >= Nn else C.contiguous()
        ldc = c_arg.stride(0)
    ws_bytes = N.lib().trnblas_gemm_workspace_size(code, 1, M, Nn, K, 0, 0)
    ws = N.workspace(ws_bytes, dev)
    args = (code, 1, M, Nn, K, float(alpha),
            N.ptr(at), lda, 0, int(ta),
            N.ptr(bt), ldb, 0, int(tb),
            float(beta) if c_arg is not None else 0.0, N.ptr(c_arg), ldc, 0,
            N.ptr(out), Nn, 0)
    if tri:
        rc = N.lib().trnblas_gemm_tri(*args, int(tri), N.ptr(ws), ws_bytes, N.stream_ptr(dev))
    else:
        rc = N.lib().trnblas_gemm(*args, N.ptr(ws), ws_bytes, N.stream_ptr(dev))
    N.check(rc, "trnblas_gemm")
    N.count_launches(3 if code == N.F32 and K > 0 else 1)  # (2 split kernels +) GEMM
    return out


def _fuse_c(C, beta: float, shape, dtype, dev) -> bool:
    return (
        C is not None
        and beta != 0.0
        and isinstance(C, torch.Tensor)
        and tuple(C.shape) == tuple(shape)
        and C.dtype == dtype
        and C.device == dev
    )


def _add_c(result: torch.Tensor, beta: float, C) -> torch.Tensor:
    """result + beta * C with torch broadcasting / promotion (non-fusable C)."""
    if C is None or beta == 0.0:
        return result
    if (
        isinstance(C, torch.Tensor)
        and C.dtype == result.dtype
        and torch.broadcast_shapes(result.shape, C.shape) == result.shape
    ):
        return result.add_(_to(C, result.device), alpha=beta)
    return result + beta * _to(C, result.device)


def _mixed_dtype_error(a: torch.Tensor, b: torch.Tensor):
    raise RuntimeError(
        f"expected m1 and m2 to have the same dtype, but got: {a.dtype} != {b.dtype}"
    )


# ── public API ───────────────────────────────────────────────────────────────


def gemm(
    alpha: float,
    A: torch.Tensor,
    B: torch.Tensor,
    beta: float = 0.0,
    C: torch.Tensor | None = None,
    transA: bool = False,
    transB: bool = False,
) -> torch.Tensor:
    """General matrix multiply: C = alpha * op(A) @ op(B) + beta * C.

    op(X) = X, or X^T when trans (for >= 3-D operands the last two dimensions,
    as in `batched_gemm`). alpha, beta and the C operand are fused into the
    kernel epilogue when C is a same-shape, same-dtype matrix; a broadcasting
    C is added afterwards with torch semantics. beta == 0 never reads C.
    fp32 runs as 3xTF32 (fp32-class error), bf16/fp16 natively with fp32
    accumulation; the result has the input dtype and a fresh buffer.
    """
    transA, transB = trans_flag(transA, "transA"), trans_flag(transB, "transB")
    a = A.mT if transA and A.dim() >= 2 else A
    b = B.mT if transB and B.dim() >= 2 else B
    if a.dim() >= 3 or b.dim() >= 3:
        return _batched(alpha, a, b, beta, C)
    return _gemm_public(alpha, a, b, beta, C)


def _gemm_public(alpha, a, b, beta, C):
    if a.dtype != b.dtype:
        _mixed_dtype_error(a, b)
    if a.dtype not in N.KERNEL_DTYPES:
        r = torch.matmul(a, b)
        r = alpha * r
        return r + beta * C if (C is not None and beta != 0.0) else r
    home = a.device
    dev = _cuda_device(a, b, C)
    if home.type == "cpu" and b.device.type == "cpu":
        r = _gemm_host_streamed(alpha, a, b, beta, C, dev)
        if r is not None:
            return r
    a2, b2 = _to(a, dev), _to(b, dev)
    squeeze = []
    if a2.dim() == 1:
        a2 = a2.unsqueeze(0)
        squeeze.append(-2)
    if b2.dim() == 1:
        b2 = b2.unsqueeze(1)
        squeeze.append(-1)
    if a2.dim() != 2 or b2.dim() != 2:
        raise RuntimeError("gemm: operands must be 1-D, 2-D or batched")
    shape = (a2.shape[0], b2.shape[1])
    Cd = _to(C, dev)
    fuse = not squeeze and _fuse_c(Cd, beta, shape, a.dtype, dev)
    r = _gemm2d(a2, b2, alpha, beta if fuse else 0.0, Cd if fuse else None)
    for d in squeeze:
        r = r.squeeze(d)
    if not fuse:
        r = _add_c(r, beta, Cd)
    return _home(r, home, dev)


# Host operands of at least this many flops stream through the GPU in row
# blocks of about STREAM_BLOCK_BYTES of A.
STREAM_MIN_FLOPS = 2.0 ** 34
STREAM_BLOCK_BYTES = 128 << 20


def _gemm_host_streamed(alpha, a, b, beta, C, dev):
    """alpha a @ b (+ beta C) for host operands, streamed: B is uploaded once,
    then row blocks of A (and of a fused C) go up on one stream, their GEMMs
    run on the current stream and the finished rows of the result come down
    on a third, so PCIe uploads, downloads (full duplex) and the tensor cores
    overlap instead of running one after another. Returns a host tensor
    (pinned, from torch's caching host allocator) once its data has arrived,
    or None when the problem is small or not a plain 2-D row-major product
    (the caller then takes the one-shot path). Pageable inputs work but their
    copies cannot overlap."""
    if a.dim() != 2 or b.dim() != 2 or a.stride(1) != 1 or a.shape[1] != b.shape[0]:
        return None
    M, K = a.shape
    Nn = b.shape[1]
    if 2.0 * M * Nn * K < STREAM_MIN_FLOPS or M < 512:
        return None
    fuse = C is not None and beta != 0.0
    if fuse and not (isinstance(C, torch.Tensor) and C.device.type == "cpu" and tuple(C.shape) == (M, Nn)
                     and C.dtype == a.dtype and C.stride(1) == 1):
        return None
    es = a.element_size()
    mb = max(128, min(M, STREAM_BLOCK_BYTES // max(K * es, 1)) // 128 * 128)
    main = torch.cuda.current_stream(dev)
    up = torch.cuda.Stream(dev)
    down = torch.cuda.Stream(dev)
    out = torch.empty((M, Nn), dtype=a.dtype, pin_memory=True)
    up.wait_stream(main)
    with torch.cuda.stream(up):
        b_d = b.to(dev, non_blocking=True)
    for r0 in range(0, M, mb):
        r1 = min(r0 + mb, M)
        with torch.cuda.stream(up):
            a_i = a[r0:r1].to(dev, non_blocking=True)
            c_i = C[r0:r1].to(dev, non_blocking=True) if fuse else None
        ready = torch.cuda.Event()
        ready.record(up)
        main.wait_event(ready)
        for t in (a_i, b_d, c_i):
            if t is not None:
                t.record_stream(main)
        r = _gemm2d(a_i, b_d, alpha, beta if fuse else 0.0, c_i)
        done = torch.cuda.Event()
        done.record(main)
        down.wait_event(done)
        with torch.cuda.stream(down):
            out[r0:r1].copy_(r, non_blocking=True)
        r.record_stream(down)
    down.synchronize()
    return out


def _flat_batch(x: torch.Tensor, batch: tuple, esize: int, f32: bool):
    """(tensor, ld, transposed, batch_stride) with x expanded to `batch`.

    A broadcast operand keeps batch stride 0 (one matrix read for all);
    otherwise the batch dims must collapse to one stride, else a copy is made.
    """
    rows, cols = x.shape[-2:]
    nb = math.prod(batch)
    xb = x.expand(*batch, rows, cols)
    bstr = [s for s, n in zip(xb.stride()[:-2], batch, strict=True) if n > 1]
    if nb <= 1 or all(s == 0 for s in bstr):
        m, ld, tr = (_tma_operand(xb.reshape(-1, rows, cols)[0], esize) if not f32 else _f32_operand(xb.reshape(-1, rows, cols)[0]))
        return m, ld, tr, 0
    try:
        flat = xb.view(nb, rows, cols)
    except RuntimeError:
        flat = xb.reshape(nb, rows, cols).contiguous()
    s0 = flat.stride(0)
    m2 = flat[0]
    if f32:
        m, ld, tr = _f32_operand(m2)
        if m is not m2:
            flat = flat.contiguous()
            return flat, cols, False, flat.stride(0)
        return flat, ld, tr, s0
    q = 16 // esize
    m, ld, tr = _tma_operand(m2, esize)
    if m is m2 and s0 % q == 0 and flat.data_ptr() % 16 == 0:
        return flat, ld, tr, s0
    ldp = -(-max(cols, 1) // q) * q
    buf = torch.zeros((nb, rows, ldp), dtype=x.dtype, device=x.device)
    buf[:, :, :cols].copy_(flat)
    return buf, ldp, False, rows * ldp


def _f32_operand(x: torch.Tensor):
    """(tensor, ld, transposed) for the fp32 split pre-pass (any unit-stride layout)."""
    rows, cols = x.shape
    s0, s1 = x.stride()
    if s1 == 1 or cols == 1:
        return x, max(s0, cols, 1), False
    if s0 == 1 or rows == 1:
        return x, max(s1, rows, 1), True
    c = x.contiguous()
    return c, max(cols, 1), False


def _batched(alpha, a, b, beta, C):
    if a.dtype != b.dtype:
        _mixed_dtype_error(a, b)
    if a.dim() < 2 or b.dim() < 2 or a.dtype not in N.KERNEL_DTYPES:
        r = alpha * torch.matmul(a, b)
        return r + beta * C if (C is not None and beta != 0.0) else r
    batch = tuple(torch.broadcast_shapes(a.shape[:-2], b.shape[:-2]))
    M, K = a.shape[-2:]
    K2, Nn = b.shape[-2:]
    if K != K2:
        raise RuntimeError(
            f"Expected size for first two dimensions of batch2 tensor to be: [{math.prod(batch)}, {K}] "
            f"but got: [{math.prod(batch)}, {K2}]."
        )
    home = a.device
    dev = _cuda_device(a, b, C)
    a2, b2 = _to(a, dev), _to(b, dev)
    nb = math.prod(batch)
    out = torch.empty((*batch, M, Nn), dtype=a.dtype, device=dev)
    Cd = _to(C, dev)
    fuse = _fuse_c(Cd, beta, out.shape, a.dtype, dev)
    if nb == 0 or M == 0 or Nn == 0:
        r = out
    else:
        code = N.dtype_code(a.dtype)
        es = a.element_size()
        f32 = code == N.F32
        at, lda, ta, sa = _flat_batch(a2, batch, es, f32)
        bt, ldb, tb, sb = _flat_batch(b2, batch, es, f32)
        c_arg, ldc, sc = None, 0, 0
        if fuse:
            c_arg = Cd.reshape(nb, M, Nn)
            if not (c_arg.stride(2) == 1 and c_arg.stride(1) >= Nn):
                c_arg = c_arg.contiguous()
            ldc, sc = c_arg.stride(1), c_arg.stride(0)
        ws_bytes = N.lib().trnblas_gemm_workspace_size(code, nb, M, Nn, K, sa, sb)
        ws = N.workspace(ws_bytes, dev)
        rc = N.lib().trnblas_gemm(
            code, nb, M, Nn, K, float(alpha),
            N.ptr(at), lda, sa, int(ta),
            N.ptr(bt), ldb, sb, int(tb),
            float(beta) if fuse else 0.0, N.ptr(c_arg), ldc, sc,
            N.ptr(out), Nn, M * Nn,
            N.ptr(ws), ws_bytes, N.stream_ptr(dev),
        )
        N.check(rc, "trnblas_gemm (batched)")
        N.count_launches(3 if code == N.F32 and K > 0 else 1)
        r = out
    if not fuse:
        r = _add_c(r, beta, Cd)
    return _home(r, home, dev)


def batched_gemm(
    alpha: float,
    A: torch.Tensor,
    B: torch.Tensor,
    beta: float = 0.0,
    C: torch.Tensor | None = None,
    transA: bool = False,
    transB: bool = False,
) -> torch.Tensor:
    """Batched GEMM: C[i] = alpha * op(A[i]) @ op(B[i]) + beta * C[i].

    torch.matmul batch semantics: batch dims broadcast, either operand may be
    2-D. One kernel launch covers every batch entry (the batch index is folded
    into the persistent tile walk); a broadcast operand is read, not copied.
    """
    transA, transB = trans_flag(transA, "transA"), trans_flag(transB, "transB")
    a = A.transpose(-2, -1) if transA else A
    b = B.transpose(-2, -1) if transB else B
    if a.dim() == 2 and b.dim() == 2:
        return _gemm_public(alpha, a, b, beta, C)
    return _batched(alpha, a, b, beta, C)


def _sym_from_triangle(C: torch.Tensor, uplo: str) -> torch.Tensor:
    """The symmetric matrix stored in the `uplo` triangle of C."""
    if uplo == "upper":
        return torch.triu(C) + torch.triu(C, diagonal=1).mT
    return torch.tril(C) + torch.tril(C, diagonal=-1).mT


def _resolve_syrk_uplo(C: torch.Tensor, uplo: str) -> str:
    """`uplo`, or the opposite triangle when only that one holds entries
    (with a DeprecationWarning), as trnblas/level3.py:305-329."""
    has_upper = bool(torch.triu(C, diagonal=1).ne(0).any())
    has_lower = bool(torch.tril(C, diagonal=-1).ne(0).any())
    other = "lower" if uplo == "upper" else "upper"
    in_uplo, in_other = (has_upper, has_lower) if uplo == "upper" else (has_lower, has_upper)
    if in_other and not in_uplo:
        warnings.warn(
            f"syrk: C stores its off-diagonal entries only in the {other} triangle "
            f"but uplo={uplo!r}; using the {other} triangle. Pass uplo={other!r}. "
            "Only the uplo triangle of C is referenced when both are stored.",
            DeprecationWarning,
            stacklevel=3,
        )
        return other
    return uplo


def _syrk_kernel(a_eff: torch.Tensor, alpha: float, beta: float, C, c_uplo: int) -> torch.Tensor:
    """alpha * a_eff @ a_eff^T (+ beta * sym(C)) on the lower-triangle kernel."""
    n, k = a_eff.shape
    dev = a_eff.device
    out = torch.empty((n, n), dtype=a_eff.dtype, device=dev)
    if n == 0:
        return out
    code = N.dtype_code(a_eff.dtype)
    if code == N.F32:
        at, lda, tr = _f32_operand(a_eff)
    else:
        at, lda, tr = _tma_operand(a_eff, a_eff.element_size())
    c_arg, ldc = None, 0
    if C is not None and c_uplo:
        c_arg = C if C.stride(1) == 1 and C.stride(0) >= n else C.contiguous()
        ldc = c_arg.stride(0)
    ws_bytes = N.lib().trnblas_syrk_workspace_size(code, n, k)
    ws = N.workspace(ws_bytes, dev)
    rc = N.lib().trnblas_syrk(
        code, n, k, float(alpha), N.ptr(at), lda, int(tr),
        float(beta) if c_arg is not None else 0.0, N.ptr(c_arg), ldc, c_uplo if c_arg is not None else 0,
        N.ptr(out), n, N.ptr(ws), ws_bytes, N.stream_ptr(dev),
    )
    N.check(rc, "trnblas_syrk")
    # (the fp32 split +) the GEMM, and for fp32 the mirror pass when the
    # CTA-pair kernel ran (a full wave of lower-triangle pair tiles, C absent
    # or lower-stored)
    T = -(-n // 256)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    pair = (code == N.F32 and T * (T + 1) // 2 >= sms // 2 and n > 128 and k >= 1024
            and not (c_arg is not None and c_uplo == 2)
            and os.environ.get("TRNBLAS_B200_GEMM_PAIR", "1") != "0")
    N.count_launches((2 if code == N.F32 else 1) + (1 if pair else 0))
    return out


def _symmetrize(R: torch.Tensor) -> torch.Tensor:
    return 0.5 * (R + R.mT)


def syrk(
    alpha: float,
    A: torch.Tensor,
    beta: float = 0.0,
    C: torch.Tensor | None = None,
    trans: bool = False,
    uplo: str = "upper",
) -> torch.Tensor:
    """Symmetric rank-k update: alpha * A @ A^T + beta * C (trans=False) or
    alpha * A^T @ A + beta * C (trans=True).

    Returns the full symmetric matrix. Only the lower-triangle tiles are
    computed on the tensor cores; each value is written to both triangles, so
    the result is exactly symmetric. As in BLAS, only the `uplo` triangle of an
    n x n C is referenced (a C stored only in the other triangle is still used,
    with a DeprecationWarning). A broadcasting C is added and the sum
    symmetrised.
    """
    trans = trans_flag(trans)
    uplo = uplo_flag(uplo)
    a_eff = A.mT if trans else A
    if a_eff.dim() != 2:
        raise ValueError(f"syrk expects a 2-D A, got shape {tuple(A.shape)}")
    n, k = a_eff.shape
    add = C is not None and beta != 0.0
    if a_eff.dtype not in N.KERNEL_DTYPES:
        S = torch.matmul(a_eff, a_eff.mT)
        S = _symmetrize(S)
        if add and C.dim() == 2 and tuple(C.shape) == (n, n):
            return alpha * S + beta * _sym_from_triangle(C, _resolve_syrk_uplo(C, uplo))
        R = alpha * S
        return _symmetrize(R + beta * C) if add else R
    home = A.device
    dev = _cuda_device(A, C)
    a2 = _to(a_eff, dev)
    Cd = _to(C, dev)
    square_c = add and Cd.dim() == 2 and tuple(Cd.shape) == (n, n)
    if k == 0:
        S = torch.zeros((n, n), dtype=a2.dtype, device=dev)
        if square_c:
            R = S + beta * _sym_from_triangle(Cd, _resolve_syrk_uplo(Cd, uplo))
        else:
            R = _symmetrize(S + beta * Cd) if add else S
        return _home(R, home, dev)
    if square_c:
        u = _resolve_syrk_uplo(Cd, uplo)
        if Cd.dtype == a2.dtype:
            R = _syrk_kernel(a2, alpha, beta, Cd, 1 if u == "lower" else 2)
        else:
            R = _syrk_kernel(a2, alpha, 0.0, None, 0) + beta * _sym_from_triangle(Cd, u)
    else:
        R = _syrk_kernel(a2, alpha, 0.0, None, 0)
        if add:
            R = _symmetrize(R + beta * Cd)
    return _home(R, home, dev)


# ── fp64-class GEMM (Ozaki on the int8 tensor cores) ─────────────────────────

MIN_SLICES, MAX_SLICES, DEFAULT_SLICES = 1, 12, 8


def check_slices(slices) -> int:
    """`slices` as an int in [1, 12]: TypeError for a non-int (or bool),
    ValueError out of range (trnblas/ozaki.py:51-58)."""
    import numpy as np

    if isinstance(slices, bool) or not isinstance(slices, (int, np.integer)):
        raise TypeError(f"slices must be an int, got {type(slices).__name__}")
    k = int(slices)
    if not MIN_SLICES <= k <= MAX_SLICES:
        raise ValueError(f"slices must be in [{MIN_SLICES}, {MAX_SLICES}], got {k}")
    return k


def _all_finite(*xs: torch.Tensor) -> bool:
    """True when no operand holds an Inf or NaN: one max-|x| reduction per
    operand (NaN propagates through it) and a single host synchronisation."""
    m = [torch.linalg.vector_norm(x, float("inf")) for x in xs if x.numel()]
    return not m or bool(torch.isfinite(torch.stack(m)).all())


def _gemm_fp64_device(a: torch.Tensor, b: torch.Tensor, k: int) -> torch.Tensor:
    """fp64 a @ b on the Ozaki int8 kernel (a, b finite fp64 on one CUDA device)."""
    M, K = a.shape
    Nn = b.shape[1]
    dev = a.device
    out = torch.empty((M, Nn), dtype=torch.float64, device=dev)
    if M == 0 or Nn == 0:
        return out
    at, lda, ta = _f32_operand(a)  # any unit-stride layout; the split kernels read strides
    bt, ldb, tb = _f32_operand(b)
    ws_bytes = N.lib().trnblas_gemm_fp64_workspace_size(M, Nn, K, k)
    ws = N.workspace(ws_bytes, dev)
    rc = N.lib().trnblas_gemm_fp64(
        M, Nn, K, N.ptr(at), lda, int(ta), N.ptr(bt), ldb, int(tb), k,
        N.ptr(out), Nn, N.ptr(ws), ws_bytes, N.stream_ptr(dev),
    )
    N.check(rc, "trnblas_gemm_fp64")
    N.count_launches(8 + 1)  # two 4-kernel splits + the int8 GEMM (one K block)
    return out


def gemm_fp64(
    A: torch.Tensor,
    B: torch.Tensor,
    *,
    slices: int = DEFAULT_SLICES,
    transA: bool = False,
    transB: bool = False,
) -> torch.Tensor:
    """fp64-class op(A) @ op(B) by Ozaki splitting on the int8 tensor cores.

    A is split per row and B per column into `slices` (k) balanced 7-bit
    integer digits with one power-of-two exponent per row / column (the
    reference's split, trnblas/ozaki.py:123-219, bit for bit). Each diagonal
    s + t = d <= k - 1 of slice products is summed exactly in int32 on the
    tensor cores, and the diagonals are recombined in fp64 (smallest first)
    with the exponents. k (k + 1) / 2 slice products; k = 8 (default) gives
    host fp64 BLAS accuracy on well-scaled data, wide dynamic ranges within a
    row / column need more slices. 1 <= slices <= 12.

    A (M, K) and B (K, N) are 2-D real tensors of any float dtype (computed as
    fp64); returns float64 (M, N) on A's device. Non-finite operands (which the
    digits cannot represent) are multiplied by torch.matmul in fp64, as the
    reference does (trnblas/nki/dispatch.py:958-980).
    """
    k = check_slices(slices)
    transA, transB = trans_flag(transA, "transA"), trans_flag(transB, "transB")
    for name, X in (("A", A), ("B", B)):
        if not isinstance(X, torch.Tensor) or X.dim() != 2:
            raise ValueError(f"gemm_fp64: {name} must be a 2-D tensor")
        if not X.is_floating_point():
            raise TypeError(f"gemm_fp64: {name} must be a real floating tensor, got {X.dtype}")
    a = A.mT if transA else A
    b = B.mT if transB else B
    if a.shape[1] != b.shape[0]:
        raise ValueError(
            f"gemm_fp64: inner dimensions differ: op(A) {tuple(a.shape)}, op(B) {tuple(b.shape)}"
        )
    home = A.device
    dev = _cuda_device(A, B)
    a = _to(a.detach(), dev).to(torch.float64)
    b = _to(b.detach(), dev).to(torch.float64)
    if a.shape[1] == 0:
        r = torch.zeros((a.shape[0], b.shape[1]), dtype=torch.float64, device=dev)
    elif not _all_finite(a, b):
        r = torch.matmul(a, b)
    else:
        r = _gemm_fp64_device(a, b, k)
    return _home(r, home, dev)


# ── triangular solve and the density-fitting metric factor ──────────────────

# Rows of one diagonal panel of the blocked solve. Panels solve with
# torch.linalg.solve_triangular (small, sequential); everything else is
# trailing-update GEMMs on the tcgen05 kernel, so larger panels shift work
# from the sequential solves to the GEMM.
TRSM_PANEL = 256


def _trsm_torch(alpha, A, B, side, uplo, trans, diag):
    """op(A) X = alpha B (left) / X op(A) = alpha B (right) with torch, for
    dtypes that have no kernel (as the reference's host route does,
    trnblas/nki/dispatch.py:1707-1738)."""
    tri = torch.triu(A) if uplo == "upper" else torch.tril(A)
    mat = tri.mT if trans else tri
    upper = (uplo == "upper") != trans
    X = torch.linalg.solve_triangular(mat, B, upper=upper, left=side == "left", unitriangular=diag == "unit")
    return alpha * X


def _trsm_left_blocked(alpha: float, A: torch.Tensor, B: torch.Tensor, uplo: str, trans: bool, unit: bool):
    """op(A) X = alpha B on the GPU in fp32: diagonal panels by
    solve_triangular, trailing updates X_rest -= op(A)_rest,panel X_panel by
    the 3xTF32 GEMM (beta = 1 fused). Forward substitution when op(A) is lower
    triangular, backward when upper. Reads only op(A)'s triangle (and not its
    diagonal for a unit diagonal)."""
    mat = A.mT if trans else A
    lower = (uplo == "lower") != trans
    n = mat.shape[0]
    X = (B * alpha) if alpha != 1.0 else B.clone()
    P = TRSM_PANEL
    if n <= P:
        return torch.linalg.solve_triangular(mat, X, upper=not lower, unitriangular=unit)
    if lower:
        for k0 in range(0, n, P):
            k1 = min(k0 + P, n)
            X[k0:k1] = torch.linalg.solve_triangular(mat[k0:k1, k0:k1], X[k0:k1], upper=False, unitriangular=unit)
            if k1 < n:
                X[k1:] = _gemm_public(-1.0, mat[k1:, k0:k1], X[k0:k1], 1.0, X[k1:])
    else:
        for k1 in range(n, 0, -P):
            k0 = max(k1 - P, 0)
            X[k0:k1] = torch.linalg.solve_triangular(mat[k0:k1, k0:k1], X[k0:k1], upper=True, unitriangular=unit)
            if k0 > 0:
                X[:k0] = _gemm_public(-1.0, mat[:k0, k0:k1], X[k0:k1], 1.0, X[:k0])
    return X


def trsm(
    alpha: float,
    A: torch.Tensor,
    B: torch.Tensor,
    side: str = "left",
    uplo: str = "upper",
    trans: bool = False,
    diag: str = "nonunit",
) -> torch.Tensor:
    """Triangular solve with multiple right-hand sides (trnblas/level3.py:332-362):
    op(A) @ X = alpha * B (side 'left') or X @ op(A) = alpha * B ('right');
    returns X. Only the `uplo` triangle of A is read; diag 'unit' takes its
    diagonal as ones.

    float32 / bfloat16 / float16 solve blocked on the GPU in fp32 (the
    trailing updates are the 3xTF32 GEMM kernel, the diagonal panels
    solve_triangular) and return B's dtype on B's device; a right-side solve
    is the left solve of the transposed system. Other dtypes run torch, as in
    the reference.
    """
    side, uplo, diag = side_flag(side), uplo_flag(uplo), diag_flag(diag)
    trans = trans_flag(trans)
    if A.dim() != 2 or A.shape[0] != A.shape[1]:
        raise ValueError(f"trsm: A must be a square matrix, got {tuple(A.shape)}")
    vec = B.dim() == 1
    b = B.unsqueeze(1 if side == "left" else 0) if vec else B
    if A.dtype not in N.KERNEL_DTYPES or B.dtype not in N.KERNEL_DTYPES:
        X = _trsm_torch(alpha, A, b, side, uplo, trans, diag)
        return X.reshape(-1) if vec else X
    if b.dim() != 2:
        raise ValueError(f"trsm: B must be 1-D or 2-D, got {tuple(B.shape)}")
    n = A.shape[0]
    if (side == "left" and b.shape[0] != n) or (side == "right" and b.shape[1] != n):
        raise ValueError(f"trsm: A is {n}x{n} but B is {tuple(B.shape)} for side={side!r}")
    home = B.device
    dev = _cuda_device(A, B)
    a32 = _to(A, dev).to(torch.float32)
    b32 = _to(b, dev).to(torch.float32)
    if side == "left":
        X = _trsm_left_blocked(alpha, a32, b32, uplo, trans, diag == "unit")
    else:  # X op(A) = alpha B  <=>  op(A)^T X^T = alpha B^T
        X = _trsm_left_blocked(alpha, a32, b32.mT.contiguous(), uplo, not trans, diag == "unit").mT.contiguous()
    if vec:
        X = X.reshape(-1)
    X = X.to(B.dtype)
    return _home(X, home, dev)


def metric_inv_half(J: torch.Tensor) -> torch.Tensor:
    """Cholesky inverse factor of a symmetric positive definite metric,
    X = L^-T with J = L L^T (trnblas/level3.py:365-380), so X X^T = J^-1 and
    (ia|Q) @ X is the density-fitting metric contraction of DF-MP2.

    Cholesky with torch.linalg.cholesky (cuSOLVER), then the blocked trsm
    (L^T X = I) on the GPU; float32 / bfloat16 / float16 compute in fp32.
    Returns J's dtype on J's device. Other float dtypes run torch; integer
    input raises NotImplementedError, as in the reference.
    """
    if not (J.is_floating_point() or J.is_complex()):
        raise NotImplementedError(f"metric_inv_half: expected a floating point or complex tensor; got {J.dtype}")
    if J.dim() != 2 or J.shape[0] != J.shape[1]:
        raise ValueError(f"metric_inv_half: J must be a square matrix, got {tuple(J.shape)}")
    if J.dtype not in N.KERNEL_DTYPES:
        L = torch.linalg.cholesky(J)
        eye = torch.eye(J.shape[0], dtype=J.dtype, device=J.device)
        return _trsm_torch(1.0, L, eye, "left", "lower", True, "nonunit")
    home = J.device
    dev = _cuda_device(J)
    L = torch.linalg.cholesky(_to(J, dev).to(torch.float32))
    eye = torch.eye(J.shape[0], dtype=torch.float32, device=dev)
    X = trsm(1.0, L, eye, uplo="lower", trans=True).to(J.dtype)
    return _home(X, home, dev)


# ── symmetric and triangular multiplies (on the GEMM kernel) ─────────────────


def _sym_full(A: torch.Tensor, uplo: str) -> torch.Tensor:
    """The symmetric matrix whose `uplo` triangle (with the diagonal) is A's."""
    if uplo == "upper":
        return torch.triu(A) + torch.triu(A, diagonal=1).mT
    return torch.tril(A) + torch.tril(A, diagonal=-1).mT


def symm(
    alpha: float,
    A: torch.Tensor,
    B: torch.Tensor,
    beta: float = 0.0,
    C: torch.Tensor | None = None,
    side: str = "left",
    uplo: str = "upper",
) -> torch.Tensor:
    """Symmetric matrix multiply (trnblas/level3.py:196-240):
    C = alpha * A @ B + beta * C (side 'left') or alpha * B @ A + beta * C
    ('right'), A symmetric with only its `uplo` triangle read.

    Kernel dtypes with a 2-D B run `trnblas_symm`: for fp32 the 3xTF32 split
    pass reads the symmetric operand from the stored triangle (no full matrix
    is formed), for bf16 / fp16 one pass writes the full matrix from the
    triangle into the workspace; then the GEMM kernel with alpha, beta and C
    fused (same C rules as `gemm`)."""
    side, uplo = side_flag(side), uplo_flag(uplo)
    if A.dim() != 2 or A.shape[0] != A.shape[1]:
        raise ValueError(f"symm: A must be a square matrix, got {tuple(A.shape)}")
    if A.dtype in N.KERNEL_DTYPES and B.dtype == A.dtype:
        dev = _cuda_device(A, B, C)
        if B.dim() == 2:
            r = _symm_kernel(alpha, _to(A, dev), _to(B, dev), beta, _to(C, dev), side, uplo)
            return _home(r, A.device, dev)
        S = _sym_full(_to(A, dev), uplo)
        if A.device != dev:
            r = gemm(alpha, S, _to(B, dev), beta, _to(C, dev)) if side == "left" else gemm(alpha, _to(B, dev), S, beta, _to(C, dev))
            return r.to(A.device)
    else:
        S = _sym_full(A, uplo)
    return gemm(alpha, S, B, beta, C) if side == "left" else gemm(alpha, B, S, beta, C)


def _symm_kernel(alpha, a, b, beta, Cd, side, uplo):
    """symm on the device through trnblas_symm (the symmetric operand read
    from its stored triangle)."""
    n = a.shape[0]
    if side == "left" and b.shape[0] != n or side == "right" and b.shape[1] != n:
        lhs, rhs = (a.shape, b.shape) if side == "left" else (b.shape, a.shape)
        raise RuntimeError(f"mat1 and mat2 shapes cannot be multiplied ({lhs[0]}x{lhs[1]} and {rhs[0]}x{rhs[1]})")
    if a.stride(1) != 1:
        if a.stride(0) == 1:
            # a column-major A is the row-major storage of A^T = A, whose
            # stored triangle is the other one
            a, uplo = a.mT, ("lower" if uplo == "upper" else "upper")
        else:
            a = a.contiguous()
    lda = max(a.stride(0), n, 1)
    M, Nn = b.shape
    dev = b.device
    dt = a.dtype
    code = N.dtype_code(dt)
    if code == N.F32:
        x = b if b.stride(1) == 1 and b.stride(0) >= Nn else b.contiguous()
        ldx = max(x.stride(0), Nn, 1)
    else:
        # 16-bit B goes to the GEMM kernel's TMA as it lies: row-major, 16-byte
        # rows and base (else a padded copy)
        x, ldx, tr = _tma_operand(b, b.element_size())
        if tr:
            x, ldx, _ = _tma_operand(b.contiguous(), b.element_size())
    out = torch.empty((M, Nn), dtype=dt, device=dev)
    if M == 0 or Nn == 0:
        return out
    fuse = _fuse_c(Cd, beta, (M, Nn), dt, dev)
    c_arg, ldc = None, 0
    if fuse:
        c_arg = Cd if Cd.stride(1) == 1 and Cd.stride(0) >= Nn else Cd.contiguous()
        ldc = c_arg.stride(0)
    ws_bytes = N.lib().trnblas_symm_workspace_size(code, int(side == "right"), M, Nn)
    ws = N.workspace(ws_bytes, dev)
    rc = N.lib().trnblas_symm(code, int(side == "right"), int(uplo == "lower"), M, Nn, float(alpha),
                              N.ptr(a), lda, N.ptr(x), ldx,
                              float(beta) if fuse else 0.0, N.ptr(c_arg), ldc, N.ptr(out), Nn,
                              N.ptr(ws), ws_bytes, N.stream_ptr(dev))
    N.check(rc, "trnblas_symm")
    N.count_launches(3 if code == N.F32 else 2)  # symmetric split / fill, (split of B,) GEMM
    return out if fuse else _add_c(out, beta, Cd)


def trmm(
    alpha: float,
    A: torch.Tensor,
    B: torch.Tensor,
    side: str = "left",
    uplo: str = "upper",
    trans: bool = False,
    diag: str = "nonunit",
) -> torch.Tensor:
    """Triangular matrix multiply (trnblas/level3.py:383-417):
    alpha * op(tri(A)) @ B (side 'left') or alpha * B @ op(tri(A)) ('right'),
    tri(A) the `uplo` triangle of A (diagonal ones for diag 'unit'). The
    triangle is masked on the operands' device and multiplied on the GEMM
    kernel, which skips the K blocks that lie wholly outside the triangle
    (about half the products of a dense GEMM); op = transpose is read in
    place (no transposed copy)."""
    side, uplo, diag = side_flag(side), uplo_flag(uplo), diag_flag(diag)
    trans = trans_flag(trans)
    if A.dim() != 2 or A.shape[0] != A.shape[1]:
        raise ValueError(f"trmm: A must be a square matrix, got {tuple(A.shape)}")
    home = A.device
    dev = _cuda_device(A, B) if A.dtype in N.KERNEL_DTYPES and B.dtype == A.dtype else A.device
    a = _to(A, dev)
    tri = torch.triu(a) if uplo == "upper" else torch.tril(a)
    if diag == "unit":
        tri.diagonal().fill_(1)
    mat = tri.mT if trans else tri
    b = _to(B, dev)
    if dev.type == "cuda" and a.dtype in N.KERNEL_DTYPES and b.dtype == a.dtype and b.dim() == 2:
        lower = (uplo == "lower") != trans  # op(tri(A)) is lower triangular
        if side == "left":
            if b.shape[0] != mat.shape[1]:
                raise ValueError(f"trmm: A is {tuple(A.shape)} but B is {tuple(B.shape)} for side='left'")
            r = _gemm2d(mat, b, alpha, 0.0, None, tri=1 if lower else 2)
        else:
            if b.shape[1] != mat.shape[0]:
                raise ValueError(f"trmm: A is {tuple(A.shape)} but B is {tuple(B.shape)} for side='right'")
            r = _gemm2d(b, mat, alpha, 0.0, None, tri=3 if lower else 4)
        return _home(r, home, dev)
    r = gemm(alpha, mat, b) if side == "left" else gemm(alpha, b, mat)
    return _home(r, home, dev)
