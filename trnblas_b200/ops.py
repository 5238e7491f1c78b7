"""The kernel boundary as functional torch ops: `torch.ops.trnblas.*`.

The analogue of the reference's op table (trnblas/nki/_native.py:49-259:
every kernel registered with `nki_op("trnblas::<name>", mutates_args={},
fake_fn=...)`, collected in `OPS` at :243-259 and wrapped by `_dtype_checked`
at :262-280). Here each op is a `torch.library.custom_op` whose CUDA
implementation calls the C ABI of include/trnblas_b200.h on the operands'
device and current stream, with a fake (meta) implementation that gives the
output's shape and dtype without touching data, so the ops trace under
FakeTensorMode and torch.compile. They are functional: inputs are read,
outputs are fresh.

    gemm(a, b, alpha, beta, c, ta, tb)            alpha op(a) op(b) + beta c  (2-D)
    batched_gemm(a, b, alpha, beta, c, ta, tb)    the same over a leading batch dim
    syrk(a, alpha, beta, c, lower_c, trans)       alpha a a^T + beta sym(c), full n x n
    ozaki_split(x, k) -> (digits, exps)           k int8 digit planes, per-row exponents
    ozaki_gemm(a, b, k) -> float64                fp64-class a @ b on the int8 pipe
    pair_energy(B, eo, ev, p0, p1) -> float64 0-d the pair-range DF-MP2 energy

`OPS[name](*args)` calls the op after the reference's operand dtype check:
a tensor of a dtype the kernel does not take raises TypeError naming the op.
"""

from __future__ import annotations

import torch

from . import _native as N
from . import level3 as _l3

_F16 = (torch.float32, torch.bfloat16, torch.float16)


def _check_2d(name, *xs):
    for x in xs:
        if x.dim() != 2:
            raise ValueError(f"trnblas::{name}: expected 2-D operands, got shape {tuple(x.shape)}")


def _gemm_shape(a, b, ta, tb):
    M = a.shape[1] if ta else a.shape[0]
    K = a.shape[0] if ta else a.shape[1]
    K2 = b.shape[1] if tb else b.shape[0]
    Nn = b.shape[0] if tb else b.shape[1]
    return M, K, K2, Nn


# ── GEMM ────────────────────────────────────────────────────────────────────


@torch.library.custom_op("trnblas::gemm", mutates_args=(), device_types="cuda")
def gemm(a: torch.Tensor, b: torch.Tensor, alpha: float = 1.0, beta: float = 0.0,
         c: torch.Tensor | None = None, ta: bool = False, tb: bool = False) -> torch.Tensor:
    _check_2d("gemm", a, b)
    if a.dtype != b.dtype:
        raise RuntimeError(f"trnblas::gemm: operand dtypes differ ({a.dtype}, {b.dtype})")
    M, K, K2, Nn = _gemm_shape(a, b, ta, tb)
    if K != K2:
        raise ValueError(f"trnblas::gemm: inner dimensions differ ({K}, {K2})")
    fuse = c is not None and beta != 0.0
    if fuse and (tuple(c.shape) != (M, Nn) or c.dtype != a.dtype):
        raise ValueError(f"trnblas::gemm: c must be ({M}, {Nn}) {a.dtype}, got {tuple(c.shape)} {c.dtype}")
    return _l3._gemm2d(a.mT if ta else a, b.mT if tb else b, alpha, beta if fuse else 0.0, c if fuse else None)


@gemm.register_fake
def _(a, b, alpha=1.0, beta=0.0, c=None, ta=False, tb=False):
    M, K, K2, Nn = _gemm_shape(a, b, ta, tb)
    torch._check(K == K2, lambda: "trnblas::gemm: inner dimensions differ")
    return a.new_empty((M, Nn))


@torch.library.custom_op("trnblas::batched_gemm", mutates_args=(), device_types="cuda")
def batched_gemm(a: torch.Tensor, b: torch.Tensor, alpha: float = 1.0, beta: float = 0.0,
                 c: torch.Tensor | None = None, ta: bool = False, tb: bool = False) -> torch.Tensor:
    if a.dim() != 3 or b.dim() != 3:
        raise ValueError("trnblas::batched_gemm: expected 3-D (batch, rows, cols) operands")
    r = _l3._batched(alpha, a.mT if ta else a, b.mT if tb else b, beta, c)
    return r if r.data_ptr() not in (a.data_ptr(), b.data_ptr()) else r.clone()


@batched_gemm.register_fake
def _(a, b, alpha=1.0, beta=0.0, c=None, ta=False, tb=False):
    M = a.shape[2] if ta else a.shape[1]
    Nn = b.shape[1] if tb else b.shape[2]
    batch = torch.broadcast_shapes(a.shape[:1], b.shape[:1])
    return a.new_empty((*batch, M, Nn))


@torch.library.custom_op("trnblas::syrk", mutates_args=(), device_types="cuda")
def syrk(a: torch.Tensor, alpha: float = 1.0, beta: float = 0.0, c: torch.Tensor | None = None,
         lower_c: bool = True, trans: bool = False) -> torch.Tensor:
    _check_2d("syrk", a)
    a_eff = a.mT if trans else a
    n = a_eff.shape[0]
    if c is not None and beta != 0.0:
        if tuple(c.shape) != (n, n) or c.dtype != a.dtype:
            raise ValueError(f"trnblas::syrk: c must be ({n}, {n}) {a.dtype}")
        return _l3._syrk_kernel(a_eff, alpha, beta, c, 1 if lower_c else 2)
    return _l3._syrk_kernel(a_eff, alpha, 0.0, None, 0)


@syrk.register_fake
def _(a, alpha=1.0, beta=0.0, c=None, lower_c=True, trans=False):
    n = a.shape[1] if trans else a.shape[0]
    return a.new_empty((n, n))


# ── fp64-class GEMM (Ozaki on the int8 tensor cores) ────────────────────────


@torch.library.custom_op("trnblas::ozaki_split", mutates_args=(), device_types="cuda")
def ozaki_split(x: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    _check_2d("ozaki_split", x)
    k = _l3.check_slices(k)
    R, K = x.shape
    dig = torch.empty((k, R, K), dtype=torch.int8, device=x.device)
    ex = torch.empty((R,), dtype=torch.int32, device=x.device)
    if R == 0 or K == 0:
        return dig, ex.zero_()
    xd = x.to(torch.float64)
    ws = N.workspace(8 * R + 256, x.device)
    N.check(N.lib().trnblas_ozaki_split(R, K, N.ptr(xd), xd.stride(0), xd.stride(1), k, N.ptr(dig), K,
                                        N.ptr(ex), N.ptr(ws), 8 * R + 256, N.stream_ptr(x.device)),
            "trnblas_ozaki_split")
    return dig, ex


@ozaki_split.register_fake
def _(x, k):
    R, K = x.shape
    return x.new_empty((k, R, K), dtype=torch.int8), x.new_empty((R,), dtype=torch.int32)


@torch.library.custom_op("trnblas::ozaki_gemm", mutates_args=(), device_types="cuda")
def ozaki_gemm(a: torch.Tensor, b: torch.Tensor, k: int = 8) -> torch.Tensor:
    _check_2d("ozaki_gemm", a, b)
    if a.shape[1] != b.shape[0]:
        raise ValueError("trnblas::ozaki_gemm: inner dimensions differ")
    k = _l3.check_slices(k)
    a64, b64 = a.to(torch.float64), b.to(torch.float64)
    if a.shape[1] == 0:
        return torch.zeros((a.shape[0], b.shape[1]), dtype=torch.float64, device=a.device)
    if not _l3._all_finite(a64, b64):
        return torch.matmul(a64, b64)
    return _l3._gemm_fp64_device(a64, b64, k)


@ozaki_gemm.register_fake
def _(a, b, k=8):
    return a.new_empty((a.shape[0], b.shape[1]), dtype=torch.float64)


# ── DF-MP2 pair energy ──────────────────────────────────────────────────────


@torch.library.custom_op("trnblas::pair_energy", mutates_args=(), device_types="cuda")
def pair_energy(B: torch.Tensor, eo: torch.Tensor, ev: torch.Tensor, pair_begin: int,
                pair_end: int) -> torch.Tensor:
    from .energy import pair_range_energy

    return pair_range_energy(B, eo, ev, pair_begin, pair_end)


@pair_energy.register_fake
def _(B, eo, ev, pair_begin, pair_end):
    return B.new_empty((), dtype=torch.float64)


# ── the op table with the reference's operand dtype check ───────────────────

# operand dtypes each kernel takes (trnblas/nki/dispatch.py:1259-1293,
# `_KERNEL_DTYPES`): the floating point tensors among an op's arguments
KERNEL_DTYPES = {
    "gemm": _F16,
    "batched_gemm": _F16,
    "syrk": _F16,
    "ozaki_split": (torch.float64, torch.float32),
    "ozaki_gemm": (torch.float64, torch.float32),
    "pair_energy": (torch.float32, torch.float64),
}

_RAW = {"gemm": gemm, "batched_gemm": batched_gemm, "syrk": syrk, "ozaki_split": ozaki_split,
        "ozaki_gemm": ozaki_gemm, "pair_energy": pair_energy}


def check_kernel_operands(name: str, *args) -> None:
    """TypeError when a tensor argument of op `name` has a dtype its kernel
    does not take (trnblas/nki/dispatch.py:1259-1293, `_check_kernel_operands`)."""
    ok = KERNEL_DTYPES[name]
    bad = [t.dtype for t in args if isinstance(t, torch.Tensor) and t.dtype not in ok]
    if bad:
        raise TypeError(f"trnblas::{name} takes {[str(d) for d in ok]} operands, got {[str(d) for d in bad]}")


def _dtype_checked(name, op):
    def checked(*args, **kwargs):
        check_kernel_operands(name, *args, *kwargs.values())
        return op(*args, **kwargs)

    checked.__name__ = name
    checked.op = op
    return checked


OPS = {name: _dtype_checked(name, op) for name, op in _RAW.items()}

__all__ = ["OPS", "KERNEL_DTYPES", "check_kernel_operands", "gemm", "batched_gemm", "syrk",
           "ozaki_split", "ozaki_gemm", "pair_energy"]
