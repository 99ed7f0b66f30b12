"""B200-native (sm_100a) Algebraic FlashAttention.

A drop-in for the AFA hot path of tasmaikeni13/algebraic-intelligence:
``pallas_afa_forward`` / ``tiled_afa_forward`` / ``pallas_afa`` (differentiable)
/ ``tiled_afa_backward`` / ``algebraic_flash_attention``
(src/kernels/pallas_afa.py), ``algebraic_softmax`` and ``octic_kernel``
(src/attention.py), ``distributed_ring_afa`` (ring AFA across the GPUs of one
node), the AGO rotary prologue (``build_cayley_rotary_matrix``,
``apply_ago_rotations``, src/attention.py), plus an HBM-bound decode step
(``afa_decode``). The compute is
hand-written CUDA for sm_100a in ``libafa_b200.so`` (C ABI: include/afa_b200.h);
this package is the host side.
"""
from .afa import (afa_decode, algebraic_flash_attention, decode_workspace_bytes, pallas_afa, pallas_afa_forward,
                  tiled_afa_backward, tiled_afa_forward)
from .ago import CayleyRotary, apply_ago_rotations, build_cayley_rotary_matrix
from .attention import algebraic_softmax, algebraic_softmax_vjp, octic_kernel
from .ring import distributed_ring_afa, ring_plan, shard_sequence, unshard_sequence

__all__ = [
    "pallas_afa_forward",
    "tiled_afa_forward",
    "tiled_afa_backward",
    "pallas_afa",
    "algebraic_flash_attention",
    "afa_decode",
    "decode_workspace_bytes",
    "algebraic_softmax",
    "algebraic_softmax_vjp",
    "octic_kernel",
    "CayleyRotary",
    "build_cayley_rotary_matrix",
    "apply_ago_rotations",
    "distributed_ring_afa",
    "ring_plan",
    "shard_sequence",
    "unshard_sequence",
]
