"""ctypes binding of the C ABI in include/trnblas_b200.h.

This is the kernel boundary: the analogue of the reference's
`trnblas/nki/_native.py` (`OPS[name](*tensors)`, trnblas/nki/_native.py:243-259)
and `dispatch._call_kernel` (trnblas/nki/dispatch.py:2168-2184), but the
kernels behind it are sm_100a CUDA in `libtrnblas_b200.so`. There is no
fallback: if the library is missing or a call fails, an exception is raised.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libtrnblas_b200.so"

F32, BF16, F16, F64 = 0, 1, 2, 3
_DTYPE_CODE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16, torch.float64: F64}
KERNEL_DTYPES = (torch.float32, torch.bfloat16, torch.float16)

ERR_ARG, ERR_ALIGN, ERR_CUDA, ERR_WORKSPACE = 1, 2, 3, 4

_lib = None
_lock = threading.Lock()

_i, _i64, _f, _p, _sz = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t
_SIGNATURES = {
    "trnblas_version": (_i, []),
    "trnblas_last_error": (ctypes.c_char_p, []),
    "trnblas_device_status": (_i, [_i, ctypes.POINTER(_i)]),
    "trnblas_gemm_workspace_size": (_sz, [_i, _i64, _i64, _i64, _i64, _i64, _i64]),
    "trnblas_gemm": (
        _i,
        [_i, _i64, _i64, _i64, _i64, _f, _p, _i64, _i64, _i, _p, _i64, _i64, _i, _f, _p, _i64,
         _i64, _p, _i64, _i64, _p, _sz, _p],
    ),
    "trnblas_gemm_tri": (
        _i,
        [_i, _i64, _i64, _i64, _i64, _f, _p, _i64, _i64, _i, _p, _i64, _i64, _i, _f, _p, _i64,
         _i64, _p, _i64, _i64, _i, _p, _sz, _p],
    ),
    "trnblas_symm_workspace_size": (_sz, [_i, _i, _i64, _i64]),
    "trnblas_symm": (
        _i, [_i, _i, _i, _i64, _i64, _f, _p, _i64, _p, _i64, _f, _p, _i64, _p, _i64, _p, _sz, _p]
    ),
    "trnblas_gemm_ready": (
        _i,
        [_i, _i64, _i64, _i64, _i64, _f, _p, _i64, _i64, _i, _p, _i64, _i64, _i, _f, _p, _i64,
         _i64, _p, _i64, _i64, _p, _i, _i64, _i, _i64, _i, _p],
    ),
    "trnblas_ipc_export": (_i, [_p, _p, ctypes.POINTER(_i64)]),
    "trnblas_ipc_open": (_i, [_p, _i64, ctypes.POINTER(_p)]),
    "trnblas_ipc_close_all": (_i, []),
    "trnblas_copy_async": (_i, [_p, _p, _sz, _p]),
    "trnblas_stream_signal": (_i, [_p, _i, _p]),
    "trnblas_gemm_f32_noalloc": (
        _i, [_i64, _i64, _i64, _f, _p, _i64, _i, _p, _i64, _i, _f, _p, _i64, _p, _i64, _p]
    ),
    "trnblas_syrk_workspace_size": (_sz, [_i, _i64, _i64]),
    "trnblas_syrk": (
        _i, [_i, _i64, _i64, _f, _p, _i64, _i, _f, _p, _i64, _i, _p, _i64, _p, _sz, _p]
    ),
    "trnblas_gemm_fp64_workspace_size": (_sz, [_i64, _i64, _i64, _i]),
    "trnblas_gemm_fp64": (
        _i, [_i64, _i64, _i64, _p, _i64, _i, _p, _i64, _i, _i, _p, _i64, _p, _sz, _p]
    ),
    "trnblas_ozaki_split": (_i, [_i64, _i64, _p, _i64, _i64, _i, _p, _i64, _p, _p, _sz, _p]),
    "trnblas_pair_energy_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "trnblas_pair_energy": (
        _i, [_i64, _i64, _i64, _p, _p, _p, _i64, _i64, _p, _p, _sz, _p]
    ),
    "trnblas_wait_selftest": (_i, [ctypes.c_ulonglong, _p]),
}


def exported_symbols() -> list[str]:
    """Every C entry point the binding declares (all must be exported)."""
    return sorted(_SIGNATURES)


def lib() -> ctypes.CDLL:
    """The loaded library (loads it on first use). Raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"trnblas_b200: native library {LIB_PATH} is missing; build it with "
                    "`python -m trnblas_b200._build` (there is no non-CUDA fallback)"
                )
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


# Kernels launched through this binding (for the benchmark's launch count).
launch_count = 0


def count_launches(n: int) -> None:
    global launch_count
    launch_count += int(n)


def last_error() -> str:
    msg = lib().trnblas_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    """Map a nonzero C status to the matching Python exception."""
    if rc == 0:
        return
    msg = f"{what}: {last_error()}"
    if rc in (ERR_ARG, ERR_ALIGN):
        raise ValueError(msg)
    raise RuntimeError(msg)


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise TypeError(f"trnblas_b200 kernels take float32/bfloat16/float16, got {dt}") from None


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def workspace(nbytes: int, device: torch.device) -> torch.Tensor | None:
    """Scratch from the caching allocator (stream-ordered, freed on return)."""
    if nbytes <= 0:
        return None
    return torch.empty(int(nbytes), dtype=torch.uint8, device=device)


def device_status(device: int | torch.device | None = None) -> int:
    """Synchronise the device, return and clear its kernel status word."""
    if device is None:
        device = torch.cuda.current_device()
    idx = device.index if isinstance(device, torch.device) else int(device)
    st = ctypes.c_int(0)
    check(lib().trnblas_device_status(int(idx if idx is not None else 0), ctypes.byref(st)),
          "trnblas_device_status")
    return st.value


def raise_on_device_status(device=None) -> None:
    """Raise RuntimeError if a kernel on `device` recorded a bounded-wait failure."""
    st = device_status(device)
    if st:
        raise RuntimeError(f"trnblas_b200: a kernel on the device gave up a bounded wait (status {st})")
