"""Algebraic FlashAttention forward on B200, behind the reference's signatures.

Drop-in for the forward entry points of src/kernels/pallas_afa.py
(tasmaikeni13/algebraic-intelligence):

* ``pallas_afa_forward``        -- pallas_afa.py:154-264 (same arguments, same
                                   ValueError conditions and messages)
* ``tiled_afa_forward``         -- pallas_afa.py:330-406 (the reference's XLA
                                   path; same math, so the same kernels)
* ``pallas_afa``                -- pallas_afa.py:579-615, differentiable: torch
                                   autograd runs the analytical backward
* ``tiled_afa_backward``        -- pallas_afa.py:409-522
* ``algebraic_flash_attention`` -- pallas_afa.py:695-739; any sequence length,
                                   handled in-kernel by masking instead of
                                   padding copies
* ``afa_decode``                -- no reference counterpart: one query token per
                                   (batch, head) over a KV cache

Arrays are torch CUDA tensors shaped (batch, heads, sequence, dim); NumPy arrays
and CPU tensors are accepted too. Host inputs of the forward are streamed
through the GPU in chunks of (batch x heads), the copies of one chunk
overlapping the kernels of its neighbours (``_launch_fwd_host``). ``block_q`` /
``block_k`` and ``interpret`` are validated like the reference but do not
change the computation: the B200 kernels tile at 128 x 128 on the tensor cores
and the result of the additive accumulation does not depend on the tiling
(the reference's own associativity test, tests/test_pallas_afa.py:207-224).
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._tensors import Staged, host_checks_float

__all__ = [
    "pallas_afa_forward",
    "tiled_afa_forward",
    "tiled_afa_backward",
    "pallas_afa",
    "algebraic_flash_attention",
    "afa_decode",
]


def _sink_ok(sink_omega) -> bool:
    try:
        return 0.0 <= float(sink_omega) < float("inf")
    except (TypeError, ValueError):
        return False


def _is_host(a) -> bool:
    return isinstance(a, np.ndarray) or (isinstance(a, torch.Tensor) and not a.is_cuda)


def _host_chunks(bh, per):
    """(start, end) ranges of the (batch x heads) chunks of a host-input forward.

    Middle chunks hold `per` heads. The first and the last hold about half as
    many: the first chunk's upload and the last chunk's download are the only
    transfers no kernel overlaps.
    """
    edge = max(1, per // 2)
    first = min(bh, edge)
    last = min(bh - first, edge)
    bounds = [0, first]
    while bounds[-1] < bh - last:
        bounds.append(min(bounds[-1] + per, bh - last))
    if last:
        bounds.append(bh)
    return list(zip(bounds[:-1], bounds[1:]))


def _launch_fwd_host(q, k, v, sink_omega, causal, valid_seq_len, return_denominator):
    """Forward of host arrays, pipelined over chunks of (batch x heads).

    Chunk c's H2D copies run on an upload stream while chunk c-1 computes, and
    chunk c's output copies back on a download stream while chunk c+1
    computes, so PCIe traffic and the kernels overlap (the copy engines carry
    the transfers; from pinned memory they are fully asynchronous). Middle
    chunks hold about two SM-waves of query pairs, the first and last about
    half that (``_host_chunks``). Returns host arrays of the input kind once the
    results are in host memory.
    """
    as_numpy = isinstance(q, np.ndarray)
    qh, kh, vh = (torch.from_numpy(np.ascontiguousarray(a)) if isinstance(a, np.ndarray) else a.contiguous()
                  for a in (q, k, v))
    if not (qh.dtype == kh.dtype == vh.dtype):
        raise TypeError(f"q, k and v must share a dtype, got {qh.dtype}, {kh.dtype} and {vh.dtype}")
    if not torch.cuda.is_available():
        raise RuntimeError("a CUDA device is required: this library has no CPU execution path")
    code = _lib.dtype_code(qh.dtype)
    b, h, l, d = qh.shape
    bh = b * h
    dev = torch.device("cuda", torch.cuda.current_device())
    props = torch.cuda.get_device_properties(dev)
    per = max(1, min(bh, -(-2 * props.multi_processor_count // max(1, -(-l // 256)))))
    acc = _lib.accum_dtype(qh.dtype)
    qd, kd, vd = (torch.empty((bh, l, d), dtype=qh.dtype, device=dev) for _ in range(3))
    od = torch.empty((bh, l, d), dtype=qh.dtype, device=dev)
    dd = torch.empty((bh, l), dtype=acc, device=dev)
    pin = torch.cuda.is_available()
    oh = torch.empty((b, h, l, d), dtype=qh.dtype, pin_memory=pin)
    dh = torch.empty((b, h, l, 1), dtype=acc, pin_memory=pin) if return_denominator else None
    srcs = [t.reshape(bh, l, d) for t in (qh, kh, vh)]
    of = oh.view(bh, l, d)
    df = dh.view(bh, l) if dh is not None else None
    lib = _lib.load()
    with torch.cuda.device(dev):
        cur = torch.cuda.current_stream(dev)
        up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        # The fresh device buffers come from the compute stream's pool: order
        # the uploads after the work already queued there. Chunks use disjoint
        # slices, so nothing else orders one chunk's upload after another's use.
        up.wait_stream(cur)
        for c0, c1 in _host_chunks(bh, per):
            with torch.cuda.stream(up):
                for dst, src in zip((qd, kd, vd), srcs):
                    dst[c0:c1].copy_(src[c0:c1], non_blocking=True)
            cur.wait_stream(up)
            rc = lib.afa_fwd(qd[c0].data_ptr(), kd[c0].data_ptr(), vd[c0].data_ptr(), od[c0].data_ptr(),
                             dd[c0].data_ptr(), 1, c1 - c0, l, d, code, float(sink_omega), int(bool(causal)),
                             int(valid_seq_len or 0), cur.cuda_stream)
            _lib.check(rc, "afa_fwd")
            down.wait_stream(cur)
            with torch.cuda.stream(down):
                of[c0:c1].copy_(od[c0:c1], non_blocking=True)
                if df is not None:
                    df[c0:c1].copy_(dd[c0:c1], non_blocking=True)
        cur.wait_stream(down)
        down.synchronize()
    outs = (oh, dh) if return_denominator else (oh,)
    if as_numpy:
        outs = tuple(t.numpy() for t in outs)
    return outs if return_denominator else outs[0]


def _resident(*ts) -> bool:
    """Contiguous CUDA tensors on one device: no staging needed."""
    t0 = ts[0]
    return all(isinstance(t, torch.Tensor) and t.is_cuda and t.device == t0.device and t.is_contiguous() for t in ts)


def _launch_fwd(q, k, v, sink_omega, causal, valid_seq_len, return_denominator):
    if _is_host(q) and _is_host(k) and _is_host(v):
        return _launch_fwd_host(q, k, v, sink_omega, causal, valid_seq_len, return_denominator)
    # Resident inputs (the common case) skip the staging wrapper and, when their
    # device is already current, the device guard: tens of microseconds of
    # host work per call, which short launches would otherwise wait on.
    st = None
    if not _resident(q, k, v):
        st = Staged(q, k, v)
        q, k, v = st.tensors
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError(f"q, k and v must share a dtype, got {q.dtype}, {k.dtype} and {v.dtype}")
    code = _lib.dtype_code(q.dtype)
    b, h, l, d = q.shape
    out = torch.empty_like(q)
    den = torch.empty((b, h, l, 1), dtype=_lib.accum_dtype(q.dtype), device=q.device)
    lib = _lib.load()
    args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), den.data_ptr(), b, h, l, d, code,
            float(sink_omega), int(bool(causal)), int(valid_seq_len or 0),
            torch.cuda.current_stream(q.device).cuda_stream)
    if q.device.index == torch.cuda.current_device():
        rc = lib.afa_fwd(*args)
    else:
        with torch.cuda.device(q.device):
            rc = lib.afa_fwd(*args)
    _lib.check(rc, "afa_fwd")
    if st is None:
        return (out, den) if return_denominator else out
    if return_denominator:
        return st.back(out), st.back(den)
    return st.back(out)


def pallas_afa_forward(q, k, v, sink_omega: float = 0.5, causal: bool = False, block_q: int = 128,
                       block_k: int = 128, valid_seq_len: Optional[int] = None, interpret: Optional[bool] = None,
                       return_denominator: bool = False):
    """AFA forward (src/kernels/pallas_afa.py:154-264).

    Returns ``out`` (q's shape and dtype) or ``(out, d_total)`` where
    ``d_total`` = row sum + sink, shape (B, H, L, 1), float32 (float64 for
    float64 inputs). bfloat16 inputs with head_dim 64 or 128 run on the tcgen05
    tensor cores; float32 / float64 on the CUDA cores at full precision
    (the reference's Precision.HIGHEST, pallas_afa.py:224-228).
    """
    del interpret  # there is one execution path: the GPU kernels
    _check_pallas_args(q, k, v, sink_omega, block_q, block_k, valid_seq_len)
    return _launch_fwd(q, k, v, sink_omega, causal, valid_seq_len, return_denominator)


def _check_pallas_args(q, k, v, sink_omega, block_q, block_k, valid_seq_len):
    """The argument checks of pallas_afa_forward (pallas_afa.py:167-186)."""
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k, and v must all have shape (batch, heads, sequence, dimension)")
    if tuple(q.shape) != tuple(k.shape) or tuple(q.shape) != tuple(v.shape):
        raise ValueError(f"q, k, and v shapes must match, got {tuple(q.shape)}, {tuple(k.shape)}, and {tuple(v.shape)}")
    if not _sink_ok(sink_omega):
        raise ValueError("sink_omega must be finite and nonnegative")
    if block_q <= 0 or block_k <= 0:
        raise ValueError("block_q and block_k must be positive")
    _, _, seq_len, head_dim = q.shape
    if head_dim <= 0:
        raise ValueError("head dimension must be positive")
    if head_dim > 128 and head_dim % 128 != 0:
        raise ValueError("head dimensions above 128 must be divisible by 128 for TPU layout")
    if seq_len % block_q != 0 or seq_len % block_k != 0:
        raise ValueError(f"seq_len ({seq_len}) must be divisible by block_q ({block_q}) and block_k ({block_k})")
    if valid_seq_len is not None and not 0 < valid_seq_len <= seq_len:
        raise ValueError("valid_seq_len must be in [1, seq_len]")
    host_checks_float(q, k, v)


def tiled_afa_forward(q, k, v, sink_omega: float = 0.5, causal: bool = False, block_q: int = 128,
                      block_k: int = 128, valid_seq_len: Optional[int] = None, return_denominator: bool = False):
    """The reference's XLA-tiled forward (src/kernels/pallas_afa.py:330-406).

    Same math as ``pallas_afa_forward``; argument checks and messages follow
    pallas_afa.py:342-353.
    """
    if q.ndim != 4 or tuple(q.shape) != tuple(k.shape) or tuple(q.shape) != tuple(v.shape):
        raise ValueError("q, k, and v must have the same four-dimensional shape")
    if not _sink_ok(sink_omega):
        raise ValueError("sink_omega must be finite and nonnegative")
    if block_q <= 0 or block_k <= 0:
        raise ValueError("block_q and block_k must be positive")
    seq_len = q.shape[2]
    if seq_len % block_q != 0 or seq_len % block_k != 0:
        raise ValueError("sequence length must be divisible by both tile dimensions")
    if valid_seq_len is not None and not 0 < valid_seq_len <= seq_len:
        raise ValueError("valid_seq_len must be in [1, seq_len]")
    host_checks_float(q, k, v)
    return _launch_fwd(q, k, v, sink_omega, causal, valid_seq_len, return_denominator)


def _launch_bwd(q, k, v, out, d_total, g_out, sink_omega, causal, valid_seq_len):
    """dq, dk, dv through afa_bwd; all arguments are contiguous CUDA tensors."""
    b, h, l, d = q.shape
    code = _lib.dtype_code(q.dtype)
    lib = _lib.load()
    den = d_total.reshape(b, h, l).to(_lib.accum_dtype(q.dtype)).contiguous()
    need = lib.afa_bwd_workspace_bytes(b, h, l, d, code)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    with torch.cuda.device(q.device):
        rc = lib.afa_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), den.data_ptr(), g_out.data_ptr(),
                         dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), b, h, l, d, code, float(sink_omega),
                         int(bool(causal)),
                         int(valid_seq_len or 0), ws.data_ptr(), need, _lib.stream_ptr(q.device))
    _lib.check(rc, "afa_bwd")
    return dq, dk, dv


def tiled_afa_backward(q, k, v, out, d_total, g_out, sink_omega: float = 0.5, causal: bool = False,
                       block_q: int = 128, block_k: int = 128, valid_seq_len: Optional[int] = None):
    """Analytical single-pass backward (src/kernels/pallas_afa.py:409-522).

    Returns (dq, dk, dv) in q's dtype: the gradients of sum(out * g_out) for
    out = AFA(q, k, v), given the forward's ``out`` and ``d_total`` (row sum +
    sink, from ``return_denominator=True``). As in the reference the gradient
    math uses the sink only through ``d_total`` (:429); ``d_total - sink_omega``
    (a row's weight sum) tells the kernels which rows lie wholly in the negative
    tail of the weight map. bfloat16 inputs round the weights and score
    gradients to bfloat16 before the three products with fp32 accumulation
    (:440-448). ``block_q`` / ``block_k`` do not change the result.
    """
    if not _sink_ok(sink_omega):
        raise ValueError("sink_omega must be finite and nonnegative")
    arrays = (q, k, v, out, g_out)
    if any(a.ndim != 4 for a in arrays) or any(tuple(a.shape) != tuple(q.shape) for a in arrays):
        raise ValueError("q, k, v, out and g_out must have the same four-dimensional shape")
    if block_q <= 0 or block_k <= 0:
        raise ValueError("block_q and block_k must be positive")
    b, h, l, _ = q.shape
    if int(np.prod(d_total.shape)) != b * h * l:
        raise ValueError(f"d_total must hold one value per query row, shape (B, H, L, 1); got {tuple(d_total.shape)}")
    if valid_seq_len is not None and not 0 < valid_seq_len <= l:
        raise ValueError("valid_seq_len must be in [1, seq_len]")
    host_checks_float(q, k, v, out, g_out)
    st = Staged(q, k, v, out, d_total, g_out)
    q, k, v, out, d_total, g_out = st.tensors
    if len({t.dtype for t in (q, k, v, out, g_out)}) != 1:
        raise TypeError("q, k, v, out and g_out must share a dtype")
    return tuple(st.back(t) for t in _launch_bwd(q, k, v, out, d_total, g_out, sink_omega, causal, valid_seq_len))


class _PallasAfa(torch.autograd.Function):
    """pallas_afa with its analytical VJP (pallas_afa.py:532-575, :615)."""

    @staticmethod
    def forward(ctx, q, k, v, sink_omega, causal, valid_seq_len):
        out, den = _launch_fwd(q, k, v, sink_omega, causal, valid_seq_len, True)
        ctx.save_for_backward(q, k, v, out, den)
        ctx.sink, ctx.causal, ctx.valid_seq_len = sink_omega, causal, valid_seq_len
        return out

    @staticmethod
    def backward(ctx, g_out):
        q, k, v, out, den = ctx.saved_tensors
        dq, dk, dv = _launch_bwd(q, k, v, out, den, g_out.contiguous(), ctx.sink, ctx.causal, ctx.valid_seq_len)
        return dq, dk, dv, None, None, None


def pallas_afa(q, k, v, sink_omega: float = 0.5, causal: bool = False, block_q: int = 128, block_k: int = 128,
               valid_seq_len: Optional[int] = None):
    """The reference's custom-VJP entry (src/kernels/pallas_afa.py:579-615).

    Same forward as ``pallas_afa_forward``. For CUDA tensors that require
    gradients the result is differentiable: torch autograd calls the analytical
    backward (``tiled_afa_backward``), as jax.grad does through ``defvjp``.
    """
    if any(isinstance(t, torch.Tensor) and t.requires_grad for t in (q, k, v)):
        # The forward's argument checks, before anything is recorded.
        _check_pallas_args(q, k, v, sink_omega, block_q, block_k, valid_seq_len)
        if not (q.is_cuda and k.is_cuda and v.is_cuda):
            raise ValueError("a differentiable pallas_afa needs CUDA tensors")
        return _PallasAfa.apply(q.contiguous(), k.contiguous(), v.contiguous(), float(sink_omega), bool(causal),
                                valid_seq_len)
    return pallas_afa_forward(q, k, v, sink_omega=sink_omega, causal=causal, block_q=block_q, block_k=block_k,
                              valid_seq_len=valid_seq_len)


def algebraic_flash_attention(q, k, v, sink_omega: float = 0.5, causal: bool = False, block_q: int = 128,
                              block_k: int = 128):
    """Unified entry for any sequence length (src/kernels/pallas_afa.py:695-739).

    The reference pads L up to lcm(block_q, block_k) with zero rows and masks
    the padded keys through ``valid_seq_len``; the padded query rows are sliced
    off. The B200 kernels mask keys at index >= L and skip stores of rows >= L
    directly, which gives the same result with no padding copies.
    """
    if q.ndim != 4 or tuple(q.shape) != tuple(k.shape) or tuple(q.shape) != tuple(v.shape):
        raise ValueError("q, k, and v must have the same four-dimensional shape")
    if block_q <= 0 or block_k <= 0:
        raise ValueError("block_q and block_k must be positive")
    if not _sink_ok(sink_omega):
        raise ValueError("sink_omega must be finite and nonnegative")
    host_checks_float(q, k, v)
    del block_q, block_k
    return _launch_fwd(q, k, v, sink_omega, causal, None, False)


def afa_decode(q, k_cache, v_cache, sink_omega: float = 0.5, kv_len=None, return_denominator: bool = False,
               workspace: Optional[torch.Tensor] = None):
    """One decode step: exact AFA for a single query token over a KV cache.

    q: (B, H, D) or (B, H, 1, D); k_cache, v_cache: (B, H, Lkv, D). ``kv_len``
    is an int (visible prefix for every batch row) or a per-batch int tensor
    (host entries must lie in [0, Lkv]; device entries are clamped to it). A
    row of length 0 gives output 0 and d_total = sink_omega.
    Math = ``pallas_afa_forward`` with one query row, non-causal; oracle =
    reference_afa with Lq = 1 (tests/reference_attention.py:44-59).
    """
    if not _sink_ok(sink_omega):
        raise ValueError("sink_omega must be finite and nonnegative")
    if k_cache.ndim != 4 or tuple(k_cache.shape) != tuple(v_cache.shape):
        raise ValueError("k_cache and v_cache must have the same (batch, heads, length, dim) shape")
    squeeze = q.ndim == 3
    b, h, lkv, d = k_cache.shape
    if tuple(q.shape) not in ((b, h, d), (b, h, 1, d)):
        raise ValueError(f"q must have shape (B, H, D) or (B, H, 1, D) matching the cache, got {tuple(q.shape)}")
    host_checks_float(q, k_cache, v_cache)
    lens_t = None
    scalar_len = 0
    if kv_len is not None:
        if isinstance(kv_len, int):
            if not 0 < kv_len <= lkv:
                raise ValueError("kv_len must be in [1, cache length]")
            scalar_len = kv_len
        else:
            lens_t = torch.as_tensor(kv_len, dtype=torch.int32)
            if not lens_t.is_cuda and bool(((lens_t < 0) | (lens_t > lkv)).any()):
                raise ValueError("kv_len entries must be in [0, cache length]")
    st = Staged(q, k_cache, v_cache)
    qt, kt, vt = st.tensors
    if lens_t is not None:
        lens_t = lens_t.to(st.device).contiguous()
        if lens_t.numel() != b:
            raise ValueError("kv_len must have one entry per batch row")
    code = _lib.dtype_code(qt.dtype)
    out = torch.empty((b, h, d), dtype=qt.dtype, device=qt.device)
    den = torch.empty((b, h), dtype=_lib.accum_dtype(qt.dtype), device=qt.device)
    lib = _lib.load()
    need = lib.afa_decode_workspace_bytes(b, h, lkv, d)
    if need:
        if workspace is None or workspace.numel() * workspace.element_size() < need:
            workspace = torch.empty(need, dtype=torch.uint8, device=qt.device)
        ws_ptr, ws_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    else:
        ws_ptr, ws_bytes = None, 0
    with torch.cuda.device(qt.device):
        rc = lib.afa_decode(qt.data_ptr(), kt.data_ptr(), vt.data_ptr(), out.data_ptr(), den.data_ptr(), b, h, lkv, d,
                            code, float(sink_omega), lens_t.data_ptr() if lens_t is not None else None, scalar_len,
                            ws_ptr, ws_bytes, _lib.stream_ptr(qt.device))
    _lib.check(rc, "afa_decode")
    if not squeeze:
        out = out.unsqueeze(2)
        den = den.unsqueeze(2)
    if return_denominator:
        return st.back(out), st.back(den.unsqueeze(-1))
    return st.back(out)


def decode_workspace_bytes(batch: int, heads: int, kv_capacity: int, head_dim: int) -> int:
    """Scratch bytes ``afa_decode`` needs for this shape (0 when it needs none)."""
    return int(_lib.load().afa_decode_workspace_bytes(batch, heads, kv_capacity, head_dim))


def hop_forward(q, k, v, problems, causal, mode, o_acc=None, d_acc=None, out=None, d_total=None,
                sink_omega: float = 0.5) -> None:
    """Grouped partial forward over up to four (query segment, key segments)
    problems -- one ring hop (src/kernels/pallas_afa.py:634-654). All tensors are
    CUDA tensors; ``problems`` is a list of
    ``(q_row0, q_len, q_pos0, [(k_row0, k_len, k_pos0), ...])``.
    """
    flat = []
    for qr, ql, qp, segs in problems:
        if not 1 <= len(segs) <= 2:
            raise ValueError("each problem needs one or two key segments")
        row = [qr, ql, qp, len(segs)]
        for s in segs:
            row += list(s)
        if len(segs) == 1:
            row += [0, 0, 0]
        flat += row
    arr = (ctypes.c_int * len(flat))(*flat)
    b, h, lq, d = q.shape
    lk = k.shape[2]
    lib = _lib.load()
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    with torch.cuda.device(q.device):
        rc = lib.afa_fwd_hop(q.data_ptr(), k.data_ptr(), v.data_ptr(), ptr(o_acc), ptr(d_acc), ptr(out), ptr(d_total),
                             b, h, lq, lk, d, _lib.dtype_code(q.dtype), arr, len(problems), int(bool(causal)),
                             int(mode), float(sink_omega), _lib.stream_ptr(q.device))
    _lib.check(rc, "afa_fwd_hop")


def scale_for(head_dim: int) -> float:
    """Score scale of the reference, float(1/sqrt(D)) (pallas_afa.py:190)."""
    return float(1.0 / math.sqrt(head_dim))
