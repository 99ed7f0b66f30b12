"""The negative tail of the octic weight map on the bf16 fast paths.

The reference evaluates rho = r / (1 - u) for s < 0 "to avoid catastrophic
cancellation in s + sqrt(1+s^2)" (src/kernels/pallas_afa.py:44-46) and pins the
tail (tests/test_pallas_afa.py:88-96). The bf16 tensor-core kernels map scores
with the single-MUFU form (1 + s^2) rsqrt(1 + s^2) + s, whose relative error
grows as s^2 for s < 0, and switch to the conjugate branch on every chunk (or,
in the backward, every query row) whose weights all sit in the tail. These
tests put every score of a row near -16, -64 or -256 (Q rows a_i * (1, ..., 1)
plus noise against K rows -(1, ..., 1) plus noise, a_i per row), where the
single-MUFU form alone is off by up to 13% at -256, and
compare with the float64 oracle at the north star's bf16 bound, 2e-2, with the
sink at 0 (the output is then sum(w v) / sum(w) over tail weights only), 0.5
and 1. Decode and the backward are checked the same way.
"""
import numpy as np
import pytest
import torch

import algebraic_intelligence_b200 as afa
from oracle import afa_oracle as orc

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2


def tail_qkv(shape, levels, seed, sigma=0.25):
    """bf16 Q, K, V on the GPU and their float64 values. Row i of Q is
    a_i * 1 + N(0, sigma^2) and every K row is -1 + N(0, sigma^2), so
    s_ij = q_i . k_j / sqrt(D) ~ -a_i sqrt(D) + sigma * N(0, a_i^2 + 1): every
    score of row i sits near -levels[i % len(levels)]."""
    b, h, l, d = shape
    rng = np.random.default_rng(seed)
    a = np.resize(np.asarray(levels, dtype=np.float64), l) / np.sqrt(d)
    q = a[None, None, :, None] + sigma * rng.normal(size=shape)
    k = -1.0 + sigma * rng.normal(size=shape)
    v = rng.normal(size=shape)
    ts = [torch.as_tensor(x, dtype=torch.float32).to("cuda").to(torch.bfloat16).contiguous() for x in (q, k, v)]
    return ts, [t.double().cpu().numpy() for t in ts]


LEVELS = {"s-16": [16.0], "s-64": [64.0], "s-256": [256.0], "mixed": [16.0, 64.0, 256.0, 40.0]}


@pytest.mark.parametrize("level", list(LEVELS))
@pytest.mark.parametrize("sink", [0.0, 0.5, 1.0])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_forward_tail_scores(level, sink, d, causal):
    (q, k, v), (qh, kh, vh) = tail_qkv((1, 2, 384, d), LEVELS[level], seed=d + len(level))
    y, den = afa.pallas_afa_forward(q, k, v, sink_omega=sink, causal=causal, return_denominator=True)
    ref, rden = orc.afa_with_denominator(qh, kh, vh, sink=sink, causal=causal)
    s = np.einsum("bhid,bhjd->bhij", qh, kh) / np.sqrt(d)
    assert s.max() < -10.0  # every score is in the tail
    assert np.isfinite(y.double().cpu().numpy()).all()
    assert orc.rel_err(y.double().cpu().numpy(), ref) <= TOL_BF16
    if sink == 0.0:
        # d_total is then the row's weight sum alone: fp32 accuracy per row
        got_w = den.double().cpu().numpy()
        assert np.max(np.abs(got_w - rden) / rden) <= 1e-3
    else:
        assert orc.rel_err(den.double().cpu().numpy(), rden) <= 1e-6


def test_forward_tail_persistent_kernel():
    """More query pairs than SMs with short rows: the persistent final-output
    kernel, every score near -256 or -64, no sink."""
    shape = (2, 40, 512, 128)
    (q, k, v), (qh, kh, vh) = tail_qkv(shape, [256.0, 64.0], seed=5)
    y = afa.pallas_afa_forward(q, k, v, sink_omega=0.0, causal=True)
    yh = y.double().cpu().numpy()
    worst = 0.0
    for b, h in ((0, 0), (1, 39), (1, 17)):
        ref = orc.afa(qh[b:b + 1, h:h + 1], kh[b:b + 1, h:h + 1], vh[b:b + 1, h:h + 1], sink=0.0, causal=True)
        worst = max(worst, orc.rel_err(yh[b:b + 1, h:h + 1], ref))
    assert worst <= TOL_BF16


def test_forward_tail_rows_next_to_normal_rows():
    """Tail rows and ordinary N(0,1) rows in the same tiles: the switch is per
    chunk, so the ordinary rows keep the fast form and the result stays within
    bounds for both."""
    (q, k, v), (qh, kh, vh) = tail_qkv((1, 2, 512, 128), [256.0], seed=8)
    rng = np.random.default_rng(9)
    normal = torch.as_tensor(rng.normal(size=(1, 2, 256, 128)), dtype=torch.float32).to("cuda").to(torch.bfloat16)
    q[:, :, ::2] = normal
    qh = q.double().cpu().numpy()
    for sink in (0.0, 0.5):
        y = afa.pallas_afa_forward(q, k, v, sink_omega=sink, causal=False)
        ref = orc.afa(qh, kh, vh, sink=sink, causal=False)
        yh = y.double().cpu().numpy()
        # each kind of row against its own scale
        assert orc.rel_err(yh[:, :, ::2], ref[:, :, ::2]) <= TOL_BF16
        assert orc.rel_err(yh[:, :, 1::2], ref[:, :, 1::2]) <= TOL_BF16


@pytest.mark.parametrize("level", ["s-64", "s-256", "mixed"])
@pytest.mark.parametrize("sink", [0.0, 0.5])
@pytest.mark.parametrize("d", [64, 128])
def test_decode_tail_scores(level, sink, d):
    b, h, lkv = 4, 8, 3000
    rng = np.random.default_rng(d)
    lv = np.resize(np.asarray(LEVELS[level]), b * h).reshape(b, h) / np.sqrt(d)
    q = lv[:, :, None] + 0.25 * rng.normal(size=(b, h, d))
    kc = -1.0 + 0.25 * rng.normal(size=(b, h, lkv, d))
    vc = rng.normal(size=(b, h, lkv, d))
    qt, kt, vt = (torch.as_tensor(x, dtype=torch.float32).to("cuda").to(torch.bfloat16) for x in (q, kc, vc))
    out = afa.afa_decode(qt, kt, vt, sink_omega=sink)
    ref, _ = orc.decode(qt.double().cpu().numpy(), kt.double().cpu().numpy(), vt.double().cpu().numpy(), sink=sink)
    assert orc.rel_err(out.double().cpu().numpy(), ref) <= TOL_BF16


@pytest.mark.parametrize("level", ["s-64", "s-256", "mixed"])
@pytest.mark.parametrize("sink", [0.0, 0.5, 1.0])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_backward_tail_scores(level, sink, d, causal):
    """The tensor-core backward (bf16, head_dim 64/128): tail rows are told
    apart by d_total - sink and take the conjugate branch."""
    shape = (1, 2, 256, d)
    (q, k, v), (qh, kh, vh) = tail_qkv(shape, LEVELS[level], seed=d + 3)
    g = torch.as_tensor(np.random.default_rng(4).normal(size=shape), dtype=torch.float32).to("cuda").to(
        torch.bfloat16)
    out, den = afa.pallas_afa_forward(q, k, v, sink_omega=sink, causal=causal, block_q=256, block_k=256,
                                      return_denominator=True)
    dq, dk, dv = afa.tiled_afa_backward(q, k, v, out, den, g, sink_omega=sink, causal=causal)
    want = orc.afa_backward(qh, kh, vh, g.double().cpu().numpy(), sink=sink, causal=causal)
    for got, ref in zip((dq, dk, dv), want):
        assert np.isfinite(got.double().cpu().numpy()).all()
        assert orc.rel_err(got.double().cpu().numpy(), ref) <= TOL_BF16
