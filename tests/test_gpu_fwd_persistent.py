"""The persistent whole-pair forward (afa_tc_sk_kernel in final-output mode)
against the one-CTA-per-pair kernel (afa_tc_fwd_kernel).

A bf16 forward launch with more (batch x head x 256-row query pair) items than
the GPU has SMs, whose pairs average at most 32 key tiles (causal L up to about 8K),
runs persistent CTAs over whole pairs in snake order; other launches run one
CTA per pair. The two kernels share the octic map, the MMA order and the
row-sum order, so a head computed alone (few pairs: one CTA per pair) must give
bit-identical output and denominators to the same head inside a many-head
launch. test_gpu_afa.py checks both paths against the float64 oracle at the
north-star tolerance; these tests pin them to each other.
"""
import numpy as np
import pytest
import torch

import algebraic_intelligence_b200 as afa
from algebraic_intelligence_b200 import _lib
from oracle import afa_oracle as orc

pytestmark = pytest.mark.gpu

MAX_AVG_TILES = 32  # the library's threshold for the persistent final-output kernel


def _qkv(shape, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(shape, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3)]


def _takes_persistent_path(b, h, l, causal):
    """Mirror of the dispatch rule: more pairs than SMs, few key tiles per pair."""
    npair = (l + 255) // 256
    # key tiles of pair p: those visible from its last row (causal) or all of them
    tiles = [(min(256 * p + 256, l) + 127) // 128 if causal else (l + 127) // 128 for p in range(npair)]
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return b * h * npair > sms and sum(tiles) <= MAX_AVG_TILES * npair


@pytest.mark.parametrize("shape,causal", [
    ((2, 8, 4096, 128), True),    # config 3's sequence length: 256 pairs of 2-32 key tiles
    ((2, 12, 2048, 128), True),   # config 2's sequence length: 192 pairs of 2-16 key tiles
    ((3, 8, 2000, 128), True),    # ragged last pair (tile 1 partly past the end)
    ((2, 40, 1024, 64), False),   # head_dim 64, non-causal, 320 pairs
    ((1, 160, 200, 128), True),   # one short pair per head
])
def test_persistent_matches_per_head_launches_bitwise(shape, causal):
    b, h, l, d = shape
    assert _takes_persistent_path(b, h, l, causal), "shape must launch the persistent kernel"
    q, k, v = _qkv(shape, seed=l + h)
    kw = dict(causal=causal, block_q=l, block_k=l, return_denominator=True)
    out, den = afa.pallas_afa_forward(q, k, v, **kw)
    for bi in range(b):
        for hi in range(0, h, max(1, h // 3)):
            sl = (slice(bi, bi + 1), slice(hi, hi + 1))
            o1, d1 = afa.pallas_afa_forward(q[sl].contiguous(), k[sl].contiguous(), v[sl].contiguous(), **kw)
            assert torch.equal(out[sl], o1), f"output of (b={bi}, h={hi}) differs"
            assert torch.equal(den[sl], d1), f"denominator of (b={bi}, h={hi}) differs"
    assert _lib.device_status(q.device) == 0


def test_persistent_ragged_against_oracle():
    """The ragged persistent shape against the float64 oracle at the bf16
    tolerance, on the last pair (tile 1 partly past the end) and the first."""
    b, h, l, d = 3, 8, 2000, 128
    q, k, v = _qkv((b, h, l, d), seed=l + h)
    out = afa.pallas_afa_forward(q, k, v, causal=True, block_q=l, block_k=l)
    for bi, hi, rows in ((2, 7, np.arange(1792, 2000)), (0, 3, np.arange(0, 256))):
        h64 = [t[bi, hi].double().cpu().numpy() for t in (q, k, v)]
        ref, _ = orc.afa_blocked(h64[0], h64[1], h64[2], causal=True, rows=rows)
        got = out[bi, hi, rows].double().cpu().numpy()
        assert orc.rel_err(got, ref) <= 2e-2
