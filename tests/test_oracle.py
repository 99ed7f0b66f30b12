"""Pins the CPU oracle to the reference (no GPU needed).

The oracle (oracle/afa_oracle.py) restates tests/reference_attention.py of the
reference; here it is checked against golden vectors that
tests/golden/make_golden.py produced by running the reference's own oracle, and
against the reference's known answers.
"""
import numpy as np
import pytest

import inputs
from oracle import afa_oracle as orc


def test_golden_inputs_regenerate(golden_meta):
    """Seeded inputs are bit-identical to the ones the fixtures were made from."""
    want = golden_meta["input_sha256"]
    assert inputs.digest(inputs.octic_grid()) == want["octic_grid"]
    assert inputs.digest(inputs.softmax_rows()) == want["softmax_rows"]
    assert inputs.digest(inputs.softmax_long_rows()) == want["softmax_long_rows"]
    assert inputs.digest(*inputs.afa_small()) == want["afa_small"]
    assert inputs.digest(*inputs.afa_l180()) == want["afa_l180"]
    assert inputs.digest(*inputs.config1()) == want["config1"]
    assert inputs.digest(*inputs.decode_small()) == want["decode_small"]


def test_octic_matches_reference_kernel(golden):
    np.testing.assert_allclose(orc.octic(inputs.octic_grid()), golden["octic_y"], rtol=1e-15, atol=0)


def test_octic_known_answers():
    # tests/test_attention.py:33-34 of the reference
    np.testing.assert_allclose(orc.octic(2.0), 51841 + 23184 * np.sqrt(5), rtol=2e-15)
    assert orc.octic(3.0) / orc.octic(-3.0) > 1e5
    # rho(x) * rho(-x) = 1 exactly in exact arithmetic
    x = np.linspace(0.0, 30.0, 301)
    np.testing.assert_allclose(orc.octic(x) * orc.octic(-x), 1.0, rtol=1e-12)
    # negative tail stays positive and finite (tests/test_pallas_afa.py:90-96)
    tail = orc.octic(np.array([-1e2, -1e3, -1e4]))
    assert np.all(tail > 0) and np.all(np.isfinite(tail))


@pytest.mark.parametrize("sink", [0.0, 0.5, 1.0])
def test_attention_matches_reference(golden, sink):
    np.testing.assert_allclose(orc.attention(inputs.softmax_rows(), sink), golden[f"asm_y_sink{sink}"],
                               rtol=1e-14, atol=1e-300)


def test_attention_long_rows(golden):
    y = orc.attention(inputs.softmax_long_rows(), 0.5)
    np.testing.assert_allclose(y, golden["asm_long_y"], rtol=2e-7, atol=1e-30)


def test_afa_matches_reference(golden):
    q, k, v = inputs.afa_small()
    assert orc.rel_err(orc.afa(q, k, v, causal=False), golden["afa_small_y"]) <= 1e-13
    assert orc.rel_err(orc.afa(q, k, v, causal=True), golden["afa_small_y_causal"]) <= 1e-13


def test_afa_ragged_and_config1(golden):
    q, k, v = inputs.afa_l180()
    assert orc.rel_err(orc.afa(q, k, v), golden["afa_l180_y"]) <= 1e-6
    assert orc.rel_err(orc.afa(q, k, v, causal=True), golden["afa_l180_y_causal"]) <= 1e-6
    q, k, v = inputs.config1()
    assert orc.rel_err(orc.afa(q, k, v), golden["cfg1_afa_o"]) <= 1e-6
    s = np.matmul(q.astype(np.float64), np.swapaxes(k.astype(np.float64), -1, -2)) / np.sqrt(q.shape[-1])
    o = np.matmul(orc.attention(s, 0.5, 1e-5), v.astype(np.float64))
    assert orc.rel_err(o, golden["cfg1_softmax_o"]) <= 1e-6


def test_decode_matches_reference(golden):
    q, k, v = inputs.decode_small()
    out, den = orc.decode(q, k, v)
    assert orc.rel_err(out, golden["dec_y"]) <= 1e-13
    assert den.shape == (2, 4, 1, 1)


@pytest.mark.parametrize("causal", [False, True])
def test_blocked_equals_full(causal):
    rng = np.random.default_rng(3)
    q, k, v = (rng.normal(size=(1, 2, 300, 16)) for _ in range(3))
    full, den = orc.afa_with_denominator(q, k, v, causal=causal)
    blk, bden = orc.afa_blocked(q, k, v, causal=causal, block=64)
    assert orc.rel_err(blk, full) <= 1e-13
    assert orc.rel_err(bden, den) <= 1e-13


def test_blocked_valid_len_and_positions():
    rng = np.random.default_rng(4)
    q, k, v = (rng.normal(size=(1, 1, 64, 8)) for _ in range(3))
    out, _ = orc.afa_blocked(q, k, v, valid_len=40)
    ref = orc.afa(q, k[..., :40, :], v[..., :40, :])
    assert orc.rel_err(out, ref) <= 1e-13
    # shifting every position by the same offset changes nothing
    a, _ = orc.afa_blocked(q, k, v, causal=True)
    b, _ = orc.afa_blocked(q, k, v, causal=True, q_pos0=1000, k_pos0=1000)
    assert orc.rel_err(a, b) == 0.0


@pytest.mark.parametrize("world", [2, 3, 4])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("zigzag", [False, True])
def test_ring_simulation_equals_global(world, causal, zigzag):
    """The reference's ring-equivalence property (tests/test_pallas_afa.py:227-271)."""
    rng = np.random.default_rng(107)
    q, k, v = (rng.normal(size=(1, 2, 24 * world, 8)) for _ in range(3))
    ring = orc.ring_simulation(q, k, v, world, causal=causal, zigzag=zigzag)
    assert orc.rel_err(ring, orc.afa(q, k, v, causal=causal)) <= 1e-12


# ---------------------------------------------------------------------------
# Backward oracle, pinned by finite differences of the pinned forward
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("causal,valid_len", [(False, None), (True, None), (False, 11), (True, 13)])
def test_backward_oracle_matches_finite_differences(causal, valid_len):
    """afa_backward restates tiled_afa_backward (pallas_afa.py:409-522). The
    reference checks it against JAX autodiff of the exact forward
    (tests/test_pallas_afa.py:292-322, 1e-5); here central differences of the
    golden-pinned float64 forward play that role."""
    rng = np.random.default_rng(3)
    shape = (1, 2, 16, 8)
    q, k, v, g = (rng.standard_normal(shape) for _ in range(4))

    def loss(q_, k_, v_):
        if valid_len is None:
            out = orc.afa(q_, k_, v_, causal=causal)
        else:
            out, _ = orc.afa_blocked(q_, k_, v_, causal=causal, valid_len=valid_len)
        return float(np.sum(out * g))

    dq, dk, dv = orc.afa_backward(q, k, v, g, causal=causal, valid_len=valid_len)
    h = 1e-6
    for name, arr, grad in (("q", q, dq), ("k", k, dk), ("v", v, dv)):
        for idx in [tuple(rng.integers(0, n) for n in shape) for _ in range(12)]:
            plus, minus = arr.copy(), arr.copy()
            plus[idx] += h
            minus[idx] -= h
            args_p = {"q": q, "k": k, "v": v}
            args_m = dict(args_p)
            args_p[name], args_m[name] = plus, minus
            fd = (loss(**{x + "_": a for x, a in args_p.items()}) - loss(**{x + "_": a for x, a in args_m.items()})) / (2 * h)
            assert abs(fd - grad[idx]) <= 1e-6 * max(1.0, np.abs(grad).max()), (name, idx, fd, grad[idx])


def test_backward_oracle_blocking_is_exact():
    rng = np.random.default_rng(4)
    q, k, v, g = (rng.standard_normal((2, 1, 40, 16)) for _ in range(4))
    a = orc.afa_backward(q, k, v, g, causal=True, block=7)
    b = orc.afa_backward(q, k, v, g, causal=True, block=512)
    for x, y in zip(a, b):
        assert np.max(np.abs(x - y)) <= 1e-12 * np.max(np.abs(y))


# ---------------------------------------------------------------------------
# AGO rotary tables and rotation (tests/reference_ago.py)
# ---------------------------------------------------------------------------
def test_ago_inputs_regenerate(golden_ago):
    want = golden_ago["_meta"]["input_sha256"]
    assert inputs.digest(*inputs.ago_small()) == want["ago_small"]
    assert inputs.digest(*inputs.ago_bhtd()) == want["ago_bhtd"]


def test_cayley_tables_match_reference(golden_ago):
    for key, args in (("table_d32_l64", dict(dim=32, max_seq_len=64)),
                      ("table_d8_l16_freqs", dict(dim=8, max_seq_len=16, freqs=[0.9, 0.5, 0.1, 0.01])),
                      ("table_d16_l8_base500", dict(dim=16, max_seq_len=8, base=500.0))):
        c, s = orc.cayley_tables(**args)
        assert np.array_equal(c, golden_ago[key + "_c"]) and np.array_equal(s, golden_ago[key + "_s"]), key
    rows = golden_ago["_meta"]["table_d128_l4096_rows"]
    c, s = orc.cayley_tables(128, 4096)
    assert np.array_equal(c[rows], golden_ago["table_d128_l4096_rows_c"])
    assert np.array_equal(s[rows], golden_ago["table_d128_l4096_rows_s"])


def test_cayley_tables_are_unit_rotations():
    """|R| = 1 at every position (the renormalisation), R_0 = identity."""
    c, s = orc.cayley_tables(64, 2048)
    assert np.max(np.abs(c * c + s * s - 1.0)) <= 1e-14
    assert np.all(c[0] == 1.0) and np.all(s[0] == 0.0)


def test_ago_rotation_matches_reference(golden_ago):
    q, k = inputs.ago_small()
    qr, kr = orc.ago_rotate(q, k)
    assert np.array_equal(qr, golden_ago["ago_small_q"]) and np.array_equal(kr, golden_ago["ago_small_k"])
    q, k = inputs.ago_bhtd()
    qr, kr = orc.ago_rotate(q, k, seq_axis=2)
    assert np.array_equal(qr, golden_ago["ago_bhtd_q"]) and np.array_equal(kr, golden_ago["ago_bhtd_k"])


def test_ago_seq_axis_defaults():
    assert orc.ago_seq_axis((64, 8)) == 0
    assert orc.ago_seq_axis((2, 64, 8)) == 1
    assert orc.ago_seq_axis((2, 64, 4, 8)) == 1
    assert orc.ago_seq_axis((2, 4, 64, 8)) == 2


# ---------------------------------------------------------------------------
# algebraic_softmax VJP (tests/reference_attention.py:27-36)
# ---------------------------------------------------------------------------
def test_softmax_vjp_matches_reference(golden, golden_meta):
    assert inputs.digest(*inputs.softmax_vjp()) == golden_meta["input_sha256"]["softmax_vjp"]
    x, g, xl, gl = inputs.softmax_vjp()
    for sink in (0.0, 0.5, 1.0):
        assert np.array_equal(orc.attention_vjp(x, g, sink), golden[f"asm_vjp_sink{sink}"])
    assert np.array_equal(orc.attention_vjp(xl, gl, 0.5), golden["asm_vjp_long"])


def test_softmax_vjp_finite_differences():
    rng = np.random.default_rng(5)
    x, g = rng.normal(size=(3, 17)), rng.normal(size=(3, 17))
    grad = orc.attention_vjp(x, g, 0.5)
    h = 1e-6
    for idx in [(0, 0), (1, 5), (2, 16)]:
        xp, xm = x.copy(), x.copy()
        xp[idx] += h
        xm[idx] -= h
        fd = (np.sum(orc.attention(xp, 0.5) * g) - np.sum(orc.attention(xm, 0.5) * g)) / (2 * h)
        assert abs(fd - grad[idx]) <= 1e-7 * max(1.0, abs(grad[idx]))
