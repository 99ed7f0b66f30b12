"""algebraic_softmax and octic_kernel on B200, behind the reference's signatures.

* ``algebraic_softmax(scores, sink_omega=0.5, eps=1e-5)`` -- src/attention.py:88-91
  (forward of _attention_forward, :59-67): AVN over the last axis, then
  rho^8 / (sum rho^8 + sink). fp32 accumulation for half inputs, fp64 kept,
  output in the input dtype. ValueError / TypeError conditions follow
  attention.py:60-63 and primitives.py:17-21, 56-61.
  Differentiable: for torch tensors that require gradients, autograd runs the
  reference's custom VJP (attention.py:70-85) on the GPU.
* ``algebraic_softmax_vjp(scores, g, sink_omega=0.5, eps=1e-5)`` -- that VJP as a
  plain function (the cotangent of the scores given the output cotangent g).
* ``octic_kernel(x)`` -- src/attention.py:47-50: rho(x)^8 elementwise,
  differentiable under torch autograd (its VJP, attention.py:38-44).
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from ._tensors import Staged, host_checks_float

__all__ = ["algebraic_softmax", "algebraic_softmax_vjp", "octic_kernel"]


def _as_array(x):
    if isinstance(x, (torch.Tensor, np.ndarray)):
        return x
    return np.asarray(x)


def _check_softmax_args(scores, sink_omega, eps):
    """attention.py:60-63 and primitives.py:17-21, 56-61."""
    if not 0 <= sink_omega < float("inf"):
        raise ValueError("sink_omega must be finite and nonnegative")
    if not 0 < eps < float("inf"):
        raise ValueError("eps must be finite and positive")
    host_checks_float(scores)
    if scores.ndim == 0 or scores.shape[-1] == 0:
        raise ValueError("AVN needs a nonempty feature axis")


def _softmax_fwd(x, sink_omega, eps):
    y = torch.empty_like(x)
    cols = x.shape[-1]
    rows = x.numel() // cols
    with torch.cuda.device(x.device):
        rc = _lib.load().algebraic_softmax_fwd(x.data_ptr(), y.data_ptr(), rows, cols, _lib.dtype_code(x.dtype),
                                               float(sink_omega), float(eps), _lib.stream_ptr(x.device))
    _lib.check(rc, "algebraic_softmax")
    return y


def _softmax_bwd(x, g, sink_omega, eps):
    dx = torch.empty_like(x)
    cols = x.shape[-1]
    rows = x.numel() // cols
    with torch.cuda.device(x.device):
        rc = _lib.load().algebraic_softmax_bwd(x.data_ptr(), g.data_ptr(), dx.data_ptr(), rows, cols,
                                               _lib.dtype_code(x.dtype), float(sink_omega), float(eps),
                                               _lib.stream_ptr(x.device))
    _lib.check(rc, "algebraic_softmax backward")
    return dx


class _AlgebraicSoftmax(torch.autograd.Function):
    """algebraic_softmax with its custom VJP (attention.py:70-85)."""

    @staticmethod
    def forward(ctx, x, sink_omega, eps):
        ctx.save_for_backward(x)
        ctx.sink_omega, ctx.eps = sink_omega, eps
        return _softmax_fwd(x, sink_omega, eps)

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        return _softmax_bwd(x, g.to(x.dtype).contiguous(), ctx.sink_omega, ctx.eps), None, None


def algebraic_softmax(scores, sink_omega: float = 0.5, eps: float = 1e-5):
    """AVN-bounded octic attention weights over the last axis (src/attention.py:88-91)."""
    scores = _as_array(scores)
    _check_softmax_args(scores, sink_omega, eps)
    if isinstance(scores, torch.Tensor) and scores.requires_grad:
        if not scores.is_cuda:
            raise ValueError("a differentiable algebraic_softmax needs a CUDA tensor")
        return _AlgebraicSoftmax.apply(scores.contiguous(), float(sink_omega), float(eps))
    st = Staged(scores)
    (x,) = st.tensors
    return st.back(_softmax_fwd(x, sink_omega, eps))


def algebraic_softmax_vjp(scores, g, sink_omega: float = 0.5, eps: float = 1e-5):
    """Cotangent of the scores of ``algebraic_softmax`` given the output's
    cotangent ``g`` (the custom VJP, attention.py:70-85 with primitives.py:73-79),
    in g's dtype (scores and g must share it)."""
    scores, g = _as_array(scores), _as_array(g)
    _check_softmax_args(scores, sink_omega, eps)
    host_checks_float(g)
    if tuple(scores.shape) != tuple(g.shape):
        raise ValueError(f"g must have the scores' shape {tuple(scores.shape)}, got {tuple(g.shape)}")
    st = Staged(scores, g)
    x, gt = st.tensors
    if x.dtype != gt.dtype:
        raise TypeError("scores and g must share a dtype")
    return st.back(_softmax_bwd(x, gt, sink_omega, eps))


def _octic_fwd(x):
    y = torch.empty_like(x)
    with torch.cuda.device(x.device):
        rc = _lib.load().afa_octic(x.data_ptr(), y.data_ptr(), x.numel(), _lib.dtype_code(x.dtype),
                                   _lib.stream_ptr(x.device))
    _lib.check(rc, "octic_kernel")
    return y


class _Octic(torch.autograd.Function):
    """octic_kernel with its custom VJP (attention.py:38-44)."""

    @staticmethod
    def forward(ctx, x):
        ctx.save_for_backward(x)
        return _octic_fwd(x)

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        g = g.to(x.dtype).contiguous()
        dx = torch.empty_like(x)
        with torch.cuda.device(x.device):
            rc = _lib.load().afa_octic_bwd(x.data_ptr(), g.data_ptr(), dx.data_ptr(), x.numel(),
                                           _lib.dtype_code(x.dtype), _lib.stream_ptr(x.device))
        _lib.check(rc, "octic_kernel backward")
        return dx


def octic_kernel(x):
    """rho(x)^8 via three squarings after evaluating rho (src/attention.py:47-50).

    Evaluated in the accumulation dtype with the reference's cancellation-free
    branch for negative x (attention.py:18-26), returned in x's dtype. For CUDA
    tensors that require gradients, autograd applies the reference's VJP,
    8 rsqrt(1 + x^2) rho(x)^8 (attention.py:38-44).
    """
    x = _as_array(x)
    host_checks_float(x)
    if isinstance(x, torch.Tensor) and x.requires_grad:
        if not x.is_cuda:
            raise ValueError("a differentiable octic_kernel needs a CUDA tensor")
        return _Octic.apply(x.contiguous())
    st = Staged(x)
    (xt,) = st.tensors
    return st.back(_octic_fwd(xt))
