"""AGO (algebraic geometric oscillator) rotary rotations on B200, behind the
reference's signatures (src/attention.py:93-240):

* ``CayleyRotary``               -- the (c, s) table pair, with ``.matrix``
                                   (:93-106)
* ``build_cayley_rotary_matrix`` -- rational Cayley rotation tables without
                                   transcendentals (:156-207)
* ``apply_ago_rotations``        -- rotates q and k by the tables at their
                                   sequence positions (:210-240); the Q/K
                                   prologue of the attention layer
                                   (src/model.py:262-264)

Both run as CUDA kernels (``afa_ago_table`` / ``afa_ago_rotate``): the tables by
a per-pair recurrence over positions, the rotation as one pass over q and k.
"""
from __future__ import annotations

import ctypes
from typing import NamedTuple, Optional

import numpy as np
import torch

from . import _lib
from ._tensors import Staged, host_checks_float

__all__ = ["CayleyRotary", "build_cayley_rotary_matrix", "apply_ago_rotations"]


class CayleyRotary(NamedTuple):
    """Precomputed Cayley rotary rotation parameters (src/attention.py:93-106).

    Can be unpacked as (c, s), or accessed via .c, .s, or .matrix.
    """
    c: torch.Tensor
    s: torch.Tensor

    @property
    def matrix(self):
        """The 2x2 rotation blocks [[c, -s], [s, c]], shape (..., 2, 2)."""
        row0 = torch.stack([self.c, -self.s], dim=-1)
        row1 = torch.stack([self.s, self.c], dim=-1)
        return torch.stack([row0, row1], dim=-2)


_TORCH_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float64": torch.float64}


def _torch_dtype(dtype) -> torch.dtype:
    if isinstance(dtype, torch.dtype):
        return dtype
    name = np.dtype(dtype).name if not isinstance(dtype, str) else dtype
    if name in _TORCH_DTYPES:
        return _TORCH_DTYPES[name]
    raise TypeError(f"unsupported table dtype {dtype!r} (float32, bfloat16 or float64)")


def build_cayley_rotary_matrix(dim: int, max_seq_len: int, freqs=None, base: float = 10000.0,
                               dtype=torch.float32, device=None) -> CayleyRotary:
    """Rational Cayley rotation tables (src/attention.py:156-207).

    Returns CayleyRotary(c, s), each (max_seq_len, dim // 2) in ``dtype`` on the
    GPU: per pair k a frequency w_k (``freqs``, or 1 / (1 + alpha k)^2 with
    alpha = (sqrt(base) - 1) / max(dim/2 - 1, 1)), the step rotation
    ((1 - w^2) / (1 + w^2), 2w / (1 + w^2)), and row m = the m-fold product
    renormalised after every step. Computed in float32 (float64 for float64).
    """
    if dim <= 0 or dim % 2 != 0:
        raise ValueError("dim must be a positive even integer")
    if max_seq_len <= 0:
        raise ValueError("max_seq_len must be a positive integer")
    pairs = dim // 2
    tdt = _torch_dtype(dtype)
    fptr = None
    if freqs is not None:
        w = np.asarray(freqs.detach().cpu() if isinstance(freqs, torch.Tensor) else freqs, dtype=np.float64)
        if w.shape != (pairs,):
            raise ValueError(f"freqs must have shape ({pairs},), got {w.shape}")
        w = np.ascontiguousarray(w)
        fptr = w.ctypes.data_as(ctypes.POINTER(ctypes.c_double))
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    c = torch.empty((max_seq_len, pairs), dtype=tdt, device=dev)
    s = torch.empty((max_seq_len, pairs), dtype=tdt, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.load().afa_ago_table(c.data_ptr(), s.data_ptr(), dim, max_seq_len, fptr, float(base),
                                       _lib.dtype_code(tdt), _lib.stream_ptr(dev))
    _lib.check(rc, "afa_ago_table")
    return CayleyRotary(c, s)


def _extract_cs(rotary_params):
    """(c, s) from a CayleyRotary, a (c, s) pair, a (..., 2, 2) matrix or a
    (..., 2) stack (src/attention.py:109-119)."""
    if isinstance(rotary_params, (tuple, list)) and len(rotary_params) >= 2:
        return rotary_params[0], rotary_params[1]
    if hasattr(rotary_params, "c") and hasattr(rotary_params, "s"):
        return rotary_params.c, rotary_params.s
    if hasattr(rotary_params, "shape"):
        if rotary_params.ndim >= 4 and tuple(rotary_params.shape[-2:]) == (2, 2):
            return rotary_params[..., 0, 0], rotary_params[..., 1, 0]
        if rotary_params.ndim >= 3 and rotary_params.shape[-1] == 2:
            return rotary_params[..., 0], rotary_params[..., 1]
    raise TypeError(f"Unsupported rotary parameters type: {type(rotary_params)}")


def _default_seq_axis(shape) -> int:
    """src/attention.py:229-230."""
    ndim = len(shape)
    return 0 if ndim == 2 else 1 if ndim == 3 else (1 if shape[1] > shape[2] else 2)


def apply_ago_rotations(q, k, rotary_params=None, seq_axis: Optional[int] = None):
    """AGO Cayley rotations of q and k (src/attention.py:210-240).

    q, k: same shape (..., dim), dim even. Each channel pair (x0, x1) at
    sequence position m becomes (c_m x0 - s_m x1, s_m x0 + c_m x1), with the
    tables cast to the tensors' dtype. ``rotary_params`` defaults to
    ``build_cayley_rotary_matrix(dim, seq_len, dtype=q.dtype)``; ``seq_axis`` to
    the reference's choice (0 for 2-D, 1 for 3-D, for 4-D 1 if shape[1] >
    shape[2] else 2). Returns (q_rot, k_rot) with the input shapes and dtypes.
    """
    if tuple(q.shape) != tuple(k.shape):
        raise ValueError(f"q and k shapes must match, got {tuple(q.shape)} and {tuple(k.shape)}")
    dim = q.shape[-1]
    if dim % 2 != 0:
        raise ValueError(f"Feature dimension must be even, got {dim}")
    host_checks_float(q, k)
    st = Staged(q, k)
    qt, kt = st.tensors
    if qt.dtype != kt.dtype:
        raise TypeError("q and k must share a dtype")
    ndim = qt.ndim
    if ndim < 2:
        raise ValueError("q and k need a sequence axis and a feature axis")
    if seq_axis is None:
        seq_axis = _default_seq_axis(qt.shape)
    if seq_axis < 0:
        seq_axis += ndim
    if not 0 <= seq_axis < ndim - 1:
        raise ValueError(f"seq_axis {seq_axis} must name an axis before the feature axis")
    seq_len = qt.shape[seq_axis]
    if rotary_params is None:
        rotary_params = build_cayley_rotary_matrix(dim, seq_len, dtype=qt.dtype, device=qt.device)
    c, s = _extract_cs(rotary_params)
    c = torch.as_tensor(np.asarray(c)) if isinstance(c, np.ndarray) else c
    s = torch.as_tensor(np.asarray(s)) if isinstance(s, np.ndarray) else s
    c = c.reshape(-1, dim // 2).to(qt.device).contiguous()
    s = s.reshape(-1, dim // 2).to(qt.device).contiguous()
    if c.shape[0] < seq_len or s.shape != c.shape:
        raise ValueError(f"rotary tables hold {c.shape[0]} positions, the sequence needs {seq_len}")
    inner = int(np.prod(qt.shape[seq_axis + 1:-1])) if seq_axis + 1 < ndim - 1 else 1
    rows = qt.numel() // dim
    q_out, k_out = torch.empty_like(qt), torch.empty_like(kt)
    with torch.cuda.device(qt.device):
        rc = _lib.load().afa_ago_rotate(qt.data_ptr(), kt.data_ptr(), q_out.data_ptr(), k_out.data_ptr(),
                                        c.data_ptr(), s.data_ptr(), _lib.dtype_code(c.dtype), rows, dim, seq_len,
                                        inner, _lib.dtype_code(qt.dtype), _lib.stream_ptr(qt.device))
    _lib.check(rc, "afa_ago_rotate")
    return st.back(q_out), st.back(k_out)
