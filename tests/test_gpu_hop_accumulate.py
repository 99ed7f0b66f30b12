"""Accumulate-mode hops: the persistent stream-K kernel.

AFA_HOP_ACCUMULATE and AFA_HOP_FINALIZE launches run one CTA per SM over equal
shares of the hop's key-tile iterations; a query pair whose iterations straddle
two shares is computed in two pieces, each added into the fp32 accumulators
with reductions, and FINALIZE divides in a separate pass. The shapes below are
chosen so that pieces really split: with 4 heads x 16 query pairs the 64 items
are fewer than the SMs (every item is split), with 16 heads x 16 pairs one round
of whole items is followed by a split tail.

Reference: the same problems run in AFA_HOP_STORE mode, which takes the
non-persistent kernel (itself checked against the float64 oracle elsewhere).
Accumulating from random prior accumulators must give prior + STORE result to
fp32 summation-order accuracy, and FINALIZE the divide of pallas_afa.py:661.
One case also checks the finalised output against the oracle directly.
"""
import numpy as np
import pytest
import torch

from algebraic_intelligence_b200 import _lib
from algebraic_intelligence_b200.afa import hop_forward
from oracle import afa_oracle as orc

pytestmark = pytest.mark.gpu

SINK = 0.5
TOL_ACC = 1e-5   # fp32 accumulators: only the summation order differs
TOL_BF16 = 1e-2  # bf16 outputs


def _rel(a, b):
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    return float((a - b).abs().max() / b.abs().max())


def _inputs(h, lq, lk, d, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn((1, h, lq, d), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((1, h, lk, d), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((1, h, lk, d), generator=g, device="cuda").to(torch.bfloat16)
    return q, k, v


def _store(q, k, v, problems, causal):
    """Raw numerator and row sums of `problems` from the non-persistent kernel."""
    b, h, lq, d = q.shape
    o = torch.zeros((b, h, lq, d), dtype=torch.float32, device="cuda")
    s = torch.zeros((b, h, lq), dtype=torch.float32, device="cuda")
    hop_forward(q, k, v, problems, causal, _lib.AFA_HOP_STORE, o_acc=o, d_acc=s, sink_omega=SINK)
    return o, s


# (heads, Lq, Lk, D, causal, problems)
CASES = {
    "every_item_split": (4, 4096, 4096, 128, False, [(0, 4096, 0, [(0, 4096, 0)])]),
    "round_then_split_tail": (16, 4096, 2048, 128, False, [(0, 4096, 0, [(0, 1024, 0), (1024, 1024, 5000)])]),
    "causal_two_problems": (8, 4096, 4096, 128, True,
                            [(0, 2048, 2048, [(0, 2048, 0), (2048, 2048, 2048)]),
                             (2048, 2048, 6144, [(0, 2048, 0), (2048, 2048, 2048)])]),
    "head_dim_64": (4, 4096, 4096, 64, False, [(0, 4096, 0, [(0, 4096, 0)])]),
}


@pytest.mark.parametrize("name", list(CASES))
def test_accumulate_adds_store_result(name):
    h, lq, lk, d, causal, problems = CASES[name]
    q, k, v = _inputs(h, lq, lk, d, seed=list(CASES).index(name))
    ref_o, ref_s = _store(q, k, v, problems, causal)
    g = torch.Generator(device="cuda").manual_seed(5)
    prev_o = torch.randn(ref_o.shape, generator=g, device="cuda") * ref_o.abs().max()
    prev_s = torch.rand(ref_s.shape, generator=g, device="cuda") * ref_s.max()
    o, s = prev_o.clone(), prev_s.clone()
    hop_forward(q, k, v, problems, causal, _lib.AFA_HOP_ACCUMULATE, o_acc=o, d_acc=s, sink_omega=SINK)
    torch.cuda.synchronize()
    assert _rel(o, prev_o + ref_o) <= TOL_ACC
    assert _rel(s, prev_s + ref_s) <= TOL_ACC
    assert _lib.device_status(q.device) == 0


@pytest.mark.parametrize("name", list(CASES))
def test_finalize_divides_the_sum(name):
    h, lq, lk, d, causal, problems = CASES[name]
    q, k, v = _inputs(h, lq, lk, d, seed=101 + list(CASES).index(name))
    ref_o, ref_s = _store(q, k, v, problems, causal)
    g = torch.Generator(device="cuda").manual_seed(6)
    prev_o = torch.randn(ref_o.shape, generator=g, device="cuda") * ref_o.abs().max()
    prev_s = torch.rand(ref_s.shape, generator=g, device="cuda") * ref_s.max()
    out = torch.full_like(q, float("nan"))
    den = torch.full((1, h, lq, 1), float("nan"), dtype=torch.float32, device="cuda")
    hop_forward(q, k, v, problems, causal, _lib.AFA_HOP_FINALIZE, o_acc=prev_o.clone(), d_acc=prev_s.clone(),
                out=out, d_total=den, sink_omega=SINK)
    torch.cuda.synchronize()
    want_den = prev_s + ref_s + SINK
    want = (prev_o + ref_o) / want_den[..., None]
    rows = torch.zeros(lq, dtype=torch.bool)
    for qr, ql, _, _ in problems:
        rows[qr:qr + ql] = True
    assert torch.isfinite(out[:, :, rows].float()).all()
    assert _rel(out[:, :, rows], want[:, :, rows]) <= TOL_BF16
    assert _rel(den[:, :, rows, 0], want_den[:, :, rows]) <= TOL_ACC


def test_finalize_rows_with_no_visible_keys():
    """A FINALIZE problem whose keys are all masked adds nothing but still gets
    its divide (the ring's last hop for ranks whose early rows see no keys)."""
    h, lq, lk, d = 4, 2048, 2048, 128
    q, k, v = _inputs(h, lq, lk, d, seed=17)
    masked = (0, 1024, 0, [(0, 1024, 4096)])          # keys after every query
    live = (1024, 1024, 8192, [(0, 2048, 0)])
    ref_o, ref_s = _store(q, k, v, [live], True)
    g = torch.Generator(device="cuda").manual_seed(7)
    prev_o = torch.randn(ref_o.shape, generator=g, device="cuda")
    prev_s = torch.rand(ref_s.shape, generator=g, device="cuda") + 1.0
    out = torch.full_like(q, float("nan"))
    hop_forward(q, k, v, [masked, live], True, _lib.AFA_HOP_FINALIZE, o_acc=prev_o.clone(), d_acc=prev_s.clone(),
                out=out, sink_omega=SINK)
    torch.cuda.synchronize()
    want = (prev_o + ref_o) / (prev_s + ref_s + SINK)[..., None]
    assert _rel(out, want) <= TOL_BF16


def test_split_finalize_matches_oracle():
    """Non-causal attention of every query over every key, computed as one
    FINALIZE hop from zero accumulators (every item split across CTAs), against
    the float64 oracle on the bf16-rounded inputs."""
    h, l, d = 4, 4096, 128
    q, k, v = _inputs(h, l, l, d, seed=23)
    o = torch.zeros((1, h, l, d), dtype=torch.float32, device="cuda")
    s = torch.zeros((1, h, l), dtype=torch.float32, device="cuda")
    out = torch.empty_like(q)
    hop_forward(q, k, v, [(0, l, 0, [(0, l, 0)])], False, _lib.AFA_HOP_FINALIZE, o_acc=o, d_acc=s, out=out,
                sink_omega=SINK)
    heads = [0, 3]
    qn, kn, vn = (t[:, heads].double().cpu().numpy() for t in (q, k, v))
    want = orc.afa(qn, kn, vn, sink=SINK, causal=False)
    got = out[:, heads].double().cpu().numpy()
    assert float(np.max(np.abs(got - want)) / np.max(np.abs(want))) <= 2e-2


def test_large_hop_non_persistent_epilogues():
    """Hops with more than 1024 query pairs per head take the non-persistent
    kernel in ACCUMULATE and FINALIZE too, whose epilogues read (and write) the
    fp32 accumulator rows in groups of consecutive rows. Two problems split the
    rows off any tile or group boundary, so groups straddle a problem's end."""
    h, lq, lk, d = 1, 263000, 512, 128
    split = 131085
    problems = [(0, split, 0, [(0, lk, 0)]), (split, lq - split, 0, [(0, lk, 0)])]
    q, k, v = _inputs(h, lq, lk, d, seed=31)
    ref_o, ref_s = _store(q, k, v, problems, False)
    g = torch.Generator(device="cuda").manual_seed(8)
    prev_o = torch.randn(ref_o.shape, generator=g, device="cuda") * ref_o.abs().max()
    prev_s = torch.rand(ref_s.shape, generator=g, device="cuda") * ref_s.max()
    o, s = prev_o.clone(), prev_s.clone()
    hop_forward(q, k, v, problems, False, _lib.AFA_HOP_ACCUMULATE, o_acc=o, d_acc=s, sink_omega=SINK)
    torch.cuda.synchronize()
    assert _rel(o, prev_o + ref_o) <= TOL_ACC
    assert _rel(s, prev_s + ref_s) <= TOL_ACC
    out = torch.full_like(q, float("nan"))
    hop_forward(q, k, v, problems, False, _lib.AFA_HOP_FINALIZE, o_acc=prev_o.clone(), d_acc=prev_s.clone(),
                out=out, sink_omega=SINK)
    torch.cuda.synchronize()
    want = (prev_o + ref_o) / (prev_s + ref_s + SINK)[..., None]
    assert torch.isfinite(out.float()).all()
    assert _rel(out, want) <= TOL_BF16
    assert _lib.device_status(q.device) == 0
