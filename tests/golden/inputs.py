"""Seeded inputs shared by the golden-fixture generator and the tests.

Each function returns NumPy arrays drawn from ``numpy.random.default_rng`` with a
fixed seed. ``golden.npz`` stores a SHA-256 of the bytes of every generated
input, so a change in NumPy's random streams shows up as a checksum failure
instead of a silent parity mismatch.
"""
from __future__ import annotations

import hashlib

import numpy as np


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def octic_grid():
    """Dense grid plus the tails of tests/test_attention.py:28-34 and
    tests/test_pallas_afa.py:90-96."""
    return np.r_[np.linspace(-64.0, 64.0, 1001), -1e4, -1e3, -1e2, 1e2, 1e3, 2.0, 3.0, -3.0, 0.0]


def softmax_rows():
    """(4,128) float64 rows, as in tests/test_attention.py:14-25."""
    return np.random.default_rng(42).normal(size=(4, 128))


def softmax_long_rows():
    """(2,4096) rows at 1e15 magnitude, as in tests/test_attention.py:56-64."""
    return np.random.default_rng(9).normal(size=(2, 4096)) * 1e15


def afa_small():
    """(1,2,64,32) float64 Q, K, V (tests/test_pallas_afa.py:74-87 shape)."""
    rng = np.random.default_rng(101)
    return tuple(rng.normal(size=(1, 2, 64, 32)) for _ in range(3))


def afa_l180():
    """(1,2,180,64) float32 Q, K, V: a length that is not a tile multiple
    (tests/test_pallas_afa.py:173-186)."""
    rng = np.random.default_rng(105)
    return tuple(rng.normal(size=(1, 2, 180, 64)).astype(np.float32) for _ in range(3))


def config1():
    """B=1,H=4,L=256,D=64 fp32, N(0,1)/sqrt(D), seed 0, drawn Q, K, V."""
    rng = np.random.default_rng(0)
    d = 64
    return tuple((rng.normal(size=(1, 4, 256, d)) / np.sqrt(d)).astype(np.float32) for _ in range(3))


def decode_small():
    """q (2,4,1,64) and a (2,4,300,64) KV cache, float32."""
    rng = np.random.default_rng(7)
    q = rng.normal(size=(2, 4, 1, 64)).astype(np.float32)
    k = rng.normal(size=(2, 4, 300, 64)).astype(np.float32)
    v = rng.normal(size=(2, 4, 300, 64)).astype(np.float32)
    return q, k, v


def ago_small():
    """AGO rotation input in the reference test's (batch, seq, heads, dim)
    layout (tests/test_ago.py:29-38), seed 42, shorter sequence."""
    rng = np.random.default_rng(42)
    q = rng.standard_normal((2, 16, 4, 32))
    k = rng.standard_normal((2, 16, 4, 32))
    return q, k


def ago_bhtd():
    """AGO rotation input in the attention layout (batch, heads, seq, dim)."""
    rng = np.random.default_rng(43)
    q = rng.standard_normal((1, 2, 32, 16))
    k = rng.standard_normal((1, 2, 32, 16))
    return q, k


def softmax_vjp():
    """Scores and cotangents as tests/test_attention.py:16-20 draws them
    (default_rng(42), normal (4, 128)), plus one 3000-column pair."""
    rng = np.random.default_rng(42)
    x = rng.normal(size=(4, 128))
    g = rng.normal(size=(4, 128))
    rng = np.random.default_rng(9)
    xl = rng.normal(size=(2, 3000)) * 3.0
    gl = rng.normal(size=(2, 3000))
    return x, g, xl, gl
