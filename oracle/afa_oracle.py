"""CPU oracle for the Algebraic FlashAttention (AFA) hot path.

TEST INFRASTRUCTURE ONLY. This module is the checker, never the thing measured or
shipped: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it. The product path (``algebraic_intelligence_b200``)
never calls it and fails loudly when its CUDA library is missing.

It restates, in float64 NumPy, the reference's own ground truth
(tasmaikeni13/algebraic-intelligence):

* ``octic``            -- tests/reference_attention.py:5-13 (``kernel``): the
                          branch form rho = sqrt(1+x^2)+x for x >= 0 and
                          1/(sqrt(1+x^2)-x) for x < 0, then rho**8.
* ``normalized``       -- tests/reference_attention.py:16-18.
* ``attention``        -- tests/reference_attention.py:21-24 (AVN over the last
                          axis, then the sink-normalised octic weights); this is
                          the math of ``algebraic_softmax`` (src/attention.py:59-67).
* ``attention_vjp``    -- tests/reference_attention.py:27-36: the cotangent of
                          the scores of ``attention`` by the quotient rule,
                          independent of the production VJP's cached-p form
                          (src/attention.py:70-85).
* ``afa``              -- tests/reference_attention.py:44-59 (``reference_afa``),
                          the exact float64 AFA forward, causal = top-left
                          aligned ``tril``.
* ``afa_blocked``      -- the same math evaluated in query-row blocks with
                          explicit global positions, so configurations whose
                          full score matrix would not fit in host memory can be
                          checked; a key at global position c is visible from a
                          query at position r iff c <= r (src/kernels/pallas_afa.py:
                          121-124 and :640-646), keys at local index >=
                          ``valid_len`` are dropped (pallas_afa.py:116-118).
* ``ring_simulation``  -- the sequence-sharded ring of
                          src/kernels/pallas_afa.py:618-662, simulated hop by hop
                          with additive numerator/denominator merging (the CPU
                          test of the reference does the same by hand,
                          tests/test_pallas_afa.py:227-271).
* ``decode``           -- exact AFA for one query token over a KV cache; the
                          reference has no decode kernel, so its oracle is
                          ``afa`` with Lq = 1, non-causal.
* ``cayley_tables``    -- the AGO rotary tables (c, s) of
                          tests/reference_ago.py:21-53 (the float64 oracle of
                          build_cayley_rotary_matrix, src/attention.py:156-207):
                          rational Cayley frequencies and a renormalised
                          rotation recurrence over positions.
* ``ago_rotate``       -- apply_ago_rotations (tests/reference_ago.py:56-94,
                          src/attention.py:210-240): each channel pair (x0, x1)
                          at position m becomes (c x0 - s x1, s x0 + c x1).
* ``afa_backward``     -- gradients of sum(afa(q, k, v) * g_out) by the
                          analytical single-pass backward of
                          src/kernels/pallas_afa.py:409-522
                          (``tiled_afa_backward``), in query-row blocks. The
                          reference pins it against JAX autodiff
                          (tests/test_pallas_afa.py:292-322); JAX is absent
                          here, so ``tests/test_oracle.py`` pins it against
                          central finite differences of ``afa``.

Parity is pinned by ``tests/test_oracle.py`` against golden vectors that
``tests/golden/make_golden.py`` produced by importing the reference's own
``tests/reference_attention.py``, and against the reference's known answers
(rho(2)^8 = 51841 + 23184*sqrt(5), the negative-tail values, ...).
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "octic",
    "normalized",
    "attention",
    "attention_vjp",
    "afa",
    "afa_blocked",
    "afa_with_denominator",
    "ring_simulation",
    "zigzag_chunks",
    "decode",
    "afa_backward",
    "cayley_tables",
    "ago_rotate",
    "ago_seq_axis",
    "rel_err",
]


def octic(x):
    """rho(x)^8 in float64 (tests/reference_attention.py:5-13).

    Only the stable branch of each sign is evaluated, so the negative tail keeps
    full relative precision (x = -1e4 gives a finite, positive value).
    """
    x = np.asarray(x, dtype=np.float64)
    root = np.sqrt(1.0 + x * x)
    rho = np.empty_like(x)
    nonneg = x >= 0
    rho[nonneg] = root[nonneg] + x[nonneg]
    rho[~nonneg] = 1.0 / (root[~nonneg] - x[~nonneg])
    return rho ** 8


def normalized(x, sink=0.5):
    """Octic weights over the last axis with a rational sink (reference_attention.py:16-18)."""
    k = octic(x)
    return k / (k.sum(axis=-1, keepdims=True) + sink)


def attention(x, sink=0.5, eps=1e-5):
    """algebraic_softmax ground truth (reference_attention.py:21-24).

    AVN: z = x / sqrt(mean(x^2) + eps) over the last axis, then octic weights
    divided by (sum + sink).
    """
    x = np.asarray(x, dtype=np.float64)
    z = x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return normalized(z, sink)


def attention_vjp(x, g, sink=0.5, eps=1e-5):
    """d/dx of sum(attention(x) * g) in float64 (reference_attention.py:27-36).

    With tau = 1/sqrt(mean(x^2) + eps), z = tau x, k = rho(z)^8 and D = sum(k) +
    sink: dz = 8 k / sqrt(1 + z^2) * (g / D - sum(g k) / D^2), and the AVN
    chain gives dx = tau dz - x tau^3 mean(x dz).
    """
    x = np.asarray(x, dtype=np.float64)
    g = np.asarray(g, dtype=np.float64)
    tau = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    z = tau * x
    k = octic(z)
    den = np.sum(k, axis=-1, keepdims=True) + sink
    dk = 8.0 * k / np.sqrt(1.0 + z * z)
    dz = dk * (g / den - np.sum(g * k, axis=-1, keepdims=True) / den ** 2)
    return tau * dz - x * tau ** 3 * np.mean(x * dz, axis=-1, keepdims=True)


def afa(q, k, v, sink=0.5, causal=False):
    """Exact AFA forward (reference_attention.py:44-59).

    o = (rho(QK^T/sqrt(D))^8 [masked]) V / (row_sum + sink).
    """
    out, _ = afa_with_denominator(q, k, v, sink=sink, causal=causal)
    return out


def afa_with_denominator(q, k, v, sink=0.5, causal=False):
    """``afa`` plus the per-row denominator d + sink, shape (..., L, 1).

    The denominator is what ``pallas_afa_forward(return_denominator=True)``
    returns (src/kernels/pallas_afa.py:148-151, :262-263).
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    scale = 1.0 / np.sqrt(q.shape[-1])
    s = np.matmul(q, np.swapaxes(k, -1, -2)) * scale
    p = octic(s)
    if causal:
        lq, lk = s.shape[-2], s.shape[-1]
        visible = np.tril(np.ones((lq, lk), dtype=bool))
        p = np.where(visible, p, 0.0)
    denom = p.sum(axis=-1, keepdims=True) + sink
    return np.matmul(p, v) / denom, denom


def afa_blocked(q, k, v, sink=0.5, causal=False, q_pos0=0, k_pos0=0,
                valid_len=None, block=512, rows=None, raw=False):
    """AFA in query-row blocks with global positions (float64).

    q: (..., Lq, D), k/v: (..., Lk, D). Query row i sits at global position
    ``q_pos0 + i``; key j at ``k_pos0 + j``. Causal visibility is
    ``key_pos <= query_pos``; keys with local index >= ``valid_len`` are
    dropped. ``rows`` optionally restricts the evaluation to a subset of query
    rows (an index array), which the bounded CPU baseline uses.

    Returns (out, denom) with denom = row_sum + sink, or, with ``raw=True``,
    the unnormalised (numerator, row_sum) pair that a ring hop accumulates.
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    lq, lk = q.shape[-2], k.shape[-2]
    scale = 1.0 / np.sqrt(q.shape[-1])
    limit = lk if valid_len is None else min(int(valid_len), lk)
    row_ids = np.arange(lq) if rows is None else np.asarray(rows)
    kt = np.swapaxes(k, -1, -2)
    key_pos = k_pos0 + np.arange(lk)
    key_ok = np.arange(lk) < limit
    num = np.zeros(q.shape[:-2] + (len(row_ids), v.shape[-1]))
    rsum = np.zeros(q.shape[:-2] + (len(row_ids), 1))
    for start in range(0, len(row_ids), block):
        sel = row_ids[start:start + block]
        s = np.matmul(q[..., sel, :], kt) * scale
        p = octic(s)
        visible = np.broadcast_to(key_ok, (len(sel), lk))
        if causal:
            visible = visible & (key_pos[None, :] <= (q_pos0 + sel)[:, None])
        p = np.where(visible, p, 0.0)
        num[..., start:start + len(sel), :] = np.matmul(p, v)
        rsum[..., start:start + len(sel), :] = p.sum(axis=-1, keepdims=True)
    if raw:
        return num, rsum
    denom = rsum + sink
    return num / denom, denom


def afa_backward(q, k, v, g_out, sink=0.5, causal=False, valid_len=None, block=512):
    """(dq, dk, dv) of sum(afa(q, k, v) * g_out) in float64.

    Restates tiled_afa_backward (src/kernels/pallas_afa.py:409-522):
      E_i   = sum_d g_out[i, d] * out[i, d]                  (:459)
      w_ij  = rho(s_ij)^8 / D_i, D_i = row_sum + sink         (:475-499)
      g_w   = g_out_i . v_j                                   (:500)
      ds_ij = 8 * scale * r_ij * w_ij * (g_w,ij - E_i),
              r = 1 / sqrt(1 + s^2)                           (:502)
      dq = ds k, dk = ds^T q, dv = w^T g_out                  (:507-510)
    with the forward's masks (causal key_pos <= query_pos, keys at index >=
    valid_len dropped). Query and key positions start at 0 (square attention,
    as the reference's backward).
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    g = np.asarray(g_out, dtype=np.float64)
    lq, lk = q.shape[-2], k.shape[-2]
    scale = 1.0 / np.sqrt(q.shape[-1])
    limit = lk if valid_len is None else min(int(valid_len), lk)
    key_ok = np.arange(lk) < limit
    kt = np.swapaxes(k, -1, -2)
    vt = np.swapaxes(v, -1, -2)
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    for start in range(0, lq, block):
        sel = np.arange(start, min(start + block, lq))
        qb, gb = q[..., sel, :], g[..., sel, :]
        s = np.matmul(qb, kt) * scale
        visible = np.broadcast_to(key_ok, (len(sel), lk))
        if causal:
            visible = visible & (np.arange(lk)[None, :] <= sel[:, None])
        p = np.where(visible, octic(s), 0.0)
        denom = p.sum(axis=-1, keepdims=True) + sink
        w = p / denom
        out = np.matmul(w, v)
        e = np.sum(gb * out, axis=-1, keepdims=True)
        r = 1.0 / np.sqrt(1.0 + s * s)
        ds = 8.0 * scale * r * w * (np.matmul(gb, vt) - e)
        dq[..., sel, :] = np.matmul(ds, k)
        dk += np.matmul(np.swapaxes(ds, -1, -2), qb)
        dv += np.matmul(np.swapaxes(w, -1, -2), gb)
    return dq, dk, dv


def cayley_tables(dim, max_seq_len, freqs=None, base=10000.0):
    """(c, s), each (max_seq_len, dim // 2), float64 (reference_ago.py:21-53).

    w_k = 1 / (1 + alpha k)^2 with alpha = (sqrt(base) - 1) / max(pairs - 1, 1),
    unless ``freqs`` gives w; the per-step rotation is the Cayley form
    ((1 - w^2) / (1 + w^2), 2w / (1 + w^2)); row m is the m-fold product,
    renormalised to unit length after every step.
    """
    if dim <= 0 or dim % 2 != 0:
        raise ValueError("dim must be a positive even integer")
    if max_seq_len <= 0:
        raise ValueError("max_seq_len must be a positive integer")
    pairs = dim // 2
    if freqs is not None:
        w = np.asarray(freqs, dtype=np.float64)
    else:
        kk = np.arange(pairs, dtype=np.float64)
        alpha = (np.sqrt(base) - 1.0) / max(float(pairs - 1), 1.0)
        lin = 1.0 + alpha * kk
        w = 1.0 / (lin * lin)
    c_step = (1.0 - w * w) / (1.0 + w * w)
    s_step = (2.0 * w) / (1.0 + w * w)
    c = np.empty((max_seq_len, pairs))
    s = np.empty((max_seq_len, pairs))
    cur_c, cur_s = np.ones(pairs), np.zeros(pairs)
    for m in range(max_seq_len):
        c[m], s[m] = cur_c, cur_s
        nc = c_step * cur_c - s_step * cur_s
        ns = s_step * cur_c + c_step * cur_s
        norm = 1.0 / np.sqrt(nc * nc + ns * ns)
        cur_c, cur_s = nc * norm, ns * norm
    return c, s


def ago_seq_axis(shape):
    """The reference's default sequence axis (reference_ago.py:65-66): 0 for 2-D,
    1 for 3-D, and for 4-D axis 1 if shape[1] > shape[2] else 2."""
    ndim = len(shape)
    return 0 if ndim == 2 else 1 if ndim == 3 else (1 if shape[1] > shape[2] else 2)


def ago_rotate(q, k, c=None, s=None, seq_axis=None):
    """(q_rot, k_rot) in float64 (reference_ago.py:56-94); tables from
    ``cayley_tables(dim, seq_len)`` when not given."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    pairs = q.shape[-1] // 2
    if seq_axis is None:
        seq_axis = ago_seq_axis(q.shape)
    n = q.shape[seq_axis]
    if c is None:
        c, s = cayley_tables(q.shape[-1], n)
    shape = [1] * (q.ndim - 1) + [pairs]
    shape[seq_axis] = n
    cb = np.asarray(c, dtype=np.float64)[:n].reshape(shape)
    sb = np.asarray(s, dtype=np.float64)[:n].reshape(shape)

    def rot(x):
        xp = x.reshape(x.shape[:-1] + (pairs, 2))
        return np.stack([cb * xp[..., 0] - sb * xp[..., 1], sb * xp[..., 0] + cb * xp[..., 1]],
                        axis=-1).reshape(x.shape)

    return rot(q), rot(k)


def zigzag_chunks(rank, world):
    """Chunk ids held by ``rank`` under zigzag sequence sharding.

    The sequence is cut into 2*world equal chunks; rank r keeps chunks r and
    2*world-1-r, which balances causal work across ranks.
    """
    return rank, 2 * world - 1 - rank


def ring_simulation(q, k, v, world, sink=0.5, causal=False, zigzag=True):
    """Hop-by-hop simulation of ring AFA (src/kernels/pallas_afa.py:618-662).

    Each simulated rank keeps its query shard; K/V shards travel around the
    ring; per hop the rank adds the hop's unnormalised numerator and row sum to
    its accumulators (pallas_afa.py:648-649) and divides once at the end
    (pallas_afa.py:661). With ``zigzag`` the shards are zigzag chunk pairs,
    otherwise contiguous blocks as in the reference. Returns the full output in
    global row order.
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    length = q.shape[-2]
    if zigzag:
        chunk = length // (2 * world)
        shards = []
        for r in range(world):
            a, b = zigzag_chunks(r, world)
            shards.append([(a * chunk, chunk), (b * chunk, chunk)])
    else:
        shard = length // world
        shards = [[(r * shard, shard)] for r in range(world)]
    out = np.zeros_like(q)
    for r in range(world):
        q_segs = shards[r]
        acc = [(np.zeros(q.shape[:-2] + (n, v.shape[-1])), np.zeros(q.shape[:-2] + (n, 1)))
               for _, n in q_segs]
        for hop in range(world):
            src = (r - hop) % world
            for qi, (qp, qn) in enumerate(q_segs):
                for kp, kn in shards[src]:
                    num, rs = afa_blocked(q[..., qp:qp + qn, :], k[..., kp:kp + kn, :],
                                          v[..., kp:kp + kn, :], causal=causal,
                                          q_pos0=qp, k_pos0=kp, raw=True)
                    acc[qi][0][...] += num
                    acc[qi][1][...] += rs
        for (qp, qn), (num, rs) in zip(q_segs, acc):
            out[..., qp:qp + qn, :] = num / (rs + sink)
    return out


def decode(q, k_cache, v_cache, sink=0.5, kv_len=None):
    """Exact AFA for a single query token per (batch, head) over a KV cache.

    q: (B, H, 1, D) or (B, H, D); caches: (B, H, Lkv, D). ``kv_len`` (int or
    per-batch sequence) limits the visible cache prefix.
    """
    q = np.asarray(q, dtype=np.float64)
    squeeze = q.ndim == 3
    if squeeze:
        q = q[:, :, None, :]
    k_cache = np.asarray(k_cache, dtype=np.float64)
    v_cache = np.asarray(v_cache, dtype=np.float64)
    bsz, lkv = q.shape[0], k_cache.shape[2]
    if kv_len is None:
        lens = np.full(bsz, lkv)
    else:
        lens = np.broadcast_to(np.asarray(kv_len), (bsz,))
    outs, dens = [], []
    for b in range(bsz):
        n = int(lens[b])
        o, d = afa_with_denominator(q[b:b + 1], k_cache[b:b + 1, :, :n], v_cache[b:b + 1, :, :n],
                                    sink=sink, causal=False)
        outs.append(o)
        dens.append(d)
    out = np.concatenate(outs, axis=0)
    den = np.concatenate(dens, axis=0)
    if squeeze:
        out, den = out[:, :, 0, :], den[:, :, 0, :]
    return out, den


def rel_err(actual, expected):
    """max|actual - expected| / max|expected| -- the reference's parity metric
    (tests/test_pallas_afa.py:85-87, scripts/run_phase6_tpu.py:120-122)."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    return float(np.max(np.abs(a - e)) / max(float(np.max(np.abs(e))), 1e-300))
