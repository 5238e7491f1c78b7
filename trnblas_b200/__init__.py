"""trnblas_b200: the GEMM-family hot path of trnsci/trnblas on NVIDIA B200.

Drop-in for `trnblas.gemm`, `batched_gemm`, `syrk`, `gemm_fp64` and the
`trnblas.parallel` SPMD GEMM / DF-MP2 pair-energy entry points
(`import trnblas_b200 as trnblas`). The compute runs in hand-written sm_100a
kernels behind the C ABI of include/trnblas_b200.h.
"""

from __future__ import annotations

from . import _native
from ._flags import diag_flag, side_flag, trans_flag, uplo_flag
from . import energy, ops, parallel
from .energy import batched_pair_energy, nki_batched_pair_energy, pair_range_energy
from .level3 import batched_gemm, gemm, gemm_fp64, metric_inv_half, symm, syrk, trmm, trsm

__version__ = "0.1.0"

__all__ = [
    "gemm", "batched_gemm", "syrk", "gemm_fp64", "trsm", "metric_inv_half", "symm", "trmm",
    "batched_pair_energy", "nki_batched_pair_energy", "pair_range_energy",
    "energy", "ops", "parallel",
    "trans_flag", "uplo_flag", "side_flag", "diag_flag",
    "set_backend", "get_backend", "device_status",
]

_BACKENDS = ("auto", "pytorch", "nki", "cuda")
_backend = "auto"


def set_backend(backend: str) -> None:
    """Accepts the reference's backend names for drop-in compatibility.

    There is one backend here (the sm_100a kernels); "pytorch" and "nki" are
    accepted and change nothing, as no routing exists.
    """
    global _backend
    if backend not in _BACKENDS:
        raise ValueError(f"backend must be one of {_BACKENDS}, got {backend!r}")
    _backend = backend


def get_backend() -> str:
    return _backend


def device_status(device=None) -> int:
    """Synchronise and read (then clear) the device's kernel status word."""
    return _native.device_status(device)

