"""ctypes binding of libafa_b200.so (the C ABI declared in include/afa_b200.h).

The library is built in-tree (``algebraic_intelligence_b200/build.py``). There is
no fallback: if the library is missing or cannot be loaded, every entry point
raises, naming the file it looked for.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("AFA_B200_LIB", Path(__file__).resolve().parent / "libafa_b200.so"))

AFA_F32, AFA_BF16, AFA_F16, AFA_F64 = 0, 1, 2, 3
AFA_OK, AFA_ERR_INVALID, AFA_ERR_DTYPE, AFA_ERR_CUDA, AFA_ERR_DEVICE = 0, 1, 2, 3, 4
AFA_HOP_STORE, AFA_HOP_ACCUMULATE, AFA_HOP_FINALIZE, AFA_HOP_ONLY = 0, 1, 2, 3

# Every symbol include/afa_b200.h declares, with its ctypes signature.
_c_int, _c_void_p, _c_float, _c_double, _c_ll, _c_size = (
    ctypes.c_int, ctypes.c_void_p, ctypes.c_float, ctypes.c_double, ctypes.c_longlong, ctypes.c_size_t)
SIGNATURES = {
    "afa_version": (ctypes.c_char_p, []),
    "afa_last_error": (ctypes.c_char_p, []),
    "afa_fwd": (_c_int, [_c_void_p] * 5 + [_c_int] * 5 + [_c_float, _c_int, _c_int, _c_void_p]),
    "afa_fwd_hop": (_c_int, [_c_void_p] * 7 + [_c_int] * 6 + [_c_void_p, _c_int, _c_int, _c_int, _c_float,
                                                              _c_void_p]),
    "afa_finalize": (_c_int, [_c_void_p] * 4 + [_c_ll, _c_int, _c_int, _c_float, _c_void_p]),
    "afa_bwd": (_c_int, [_c_void_p] * 9 + [_c_int] * 5 + [_c_float, _c_int, _c_int, _c_void_p, _c_size,
                                                           _c_void_p]),
    "afa_bwd_workspace_bytes": (_c_size, [_c_int] * 5),
    "afa_ago_table": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, ctypes.POINTER(_c_double), _c_double, _c_int,
                               _c_void_p]),
    "afa_ago_rotate": (_c_int, [_c_void_p] * 6 + [_c_int, _c_ll, _c_int, _c_int, _c_ll, _c_int, _c_void_p]),
    "afa_ring_export": (_c_int, [_c_void_p, _c_void_p, ctypes.POINTER(ctypes.c_ulonglong)]),
    "afa_ring_open": (_c_int, [_c_void_p, ctypes.POINTER(_c_void_p)]),
    "afa_ring_close": (_c_int, [_c_void_p]),
    "afa_ring_pull": (_c_int, [_c_void_p, _c_void_p, _c_size, _c_void_p]),
    "afa_ring_pull2d": (_c_int, [_c_void_p, _c_size, _c_void_p, _c_size, _c_size, _c_size, _c_void_p]),
    "afa_decode": (_c_int, [_c_void_p] * 5 + [_c_int] * 5 + [_c_float, _c_void_p, _c_int, _c_void_p, _c_size,
                                                             _c_void_p]),
    "afa_decode_workspace_bytes": (_c_size, [_c_int] * 4),
    "afa_decode_noalloc": (_c_int, [_c_void_p] * 5 + [_c_int] * 5 + [_c_float, _c_void_p, _c_int, _c_void_p]),
    "algebraic_softmax_fwd": (_c_int, [_c_void_p, _c_void_p, _c_ll, _c_int, _c_int, _c_double, _c_double,
                                       _c_void_p]),
    "algebraic_softmax_bwd": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_ll, _c_int, _c_int, _c_double, _c_double,
                                       _c_void_p]),
    "afa_octic": (_c_int, [_c_void_p, _c_void_p, _c_ll, _c_int, _c_void_p]),
    "afa_octic_bwd": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_ll, _c_int, _c_void_p]),
    "afa_device_status": (_c_int, [_c_void_p, ctypes.POINTER(ctypes.c_int), _c_int]),
    "afa_selftest_bounded_wait": (_c_int, [_c_ll, _c_void_p]),
}

_LIB = None


class AfaLibraryError(RuntimeError):
    """libafa_b200.so is missing, failed to load, or reported a CUDA failure."""


def load() -> ctypes.CDLL:
    """Load (once) and return the library with typed signatures."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise AfaLibraryError(
                f"{LIB_PATH} not found: build it with `python -m algebraic_intelligence_b200.build` "
                "(there is no CPU fallback for this path)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


def check(rc: int, what: str) -> None:
    """Translate a status code into the reference's exception types."""
    if rc == AFA_OK:
        return
    msg = load().afa_last_error().decode(errors="replace")
    if rc == AFA_ERR_INVALID:
        raise ValueError(msg)
    if rc == AFA_ERR_DTYPE:
        raise TypeError(msg)
    raise AfaLibraryError(f"{what}: {msg}")


_DTYPE_CODES = {
    torch.float32: AFA_F32,
    torch.bfloat16: AFA_BF16,
    torch.float16: AFA_F16,
    torch.float64: AFA_F64,
}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dt]
    except KeyError:
        raise TypeError("expected a floating point array") from None


def accum_dtype(dt: torch.dtype) -> torch.dtype:
    """Accumulation dtype: float64 stays float64, everything else float32
    (src/primitives.py:17-21, src/kernels/pallas_afa.py:208)."""
    return torch.float64 if dt == torch.float64 else torch.float32


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_status(device: torch.device, clear: bool = True) -> int:
    """Synchronise the current stream and return the device status word
    (non-zero when a kernel's bounded wait ran out)."""
    out = ctypes.c_int(0)
    with torch.cuda.device(device):
        check(load().afa_device_status(stream_ptr(device), ctypes.byref(out), int(clear)), "afa_device_status")
    return out.value
