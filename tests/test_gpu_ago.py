"""AGO rotary tables and rotations on the GPU against the reference's float64
oracle (tests/reference_ago.py, committed as tests/golden/golden_ago.npz) and
the oracle restatement in oracle/afa_oracle.py.

Tolerances follow tests/test_ago.py:25-50: float64 1e-12, float32 2e-5,
bfloat16 0.04 (rtol = atol).
"""
import numpy as np
import pytest
import torch

import algebraic_intelligence_b200 as afa
import inputs
from oracle import afa_oracle as orc

pytestmark = pytest.mark.gpu

TOL = {torch.float64: 1e-12, torch.float32: 2e-5, torch.bfloat16: 0.04}


def _np(t):
    return t.detach().double().cpu().numpy()


def test_tables_float64_reproduce_reference(golden_ago):
    c, s = afa.build_cayley_rotary_matrix(32, 64, dtype=torch.float64)
    assert np.max(np.abs(_np(c) - golden_ago["table_d32_l64_c"])) <= 1e-15
    assert np.max(np.abs(_np(s) - golden_ago["table_d32_l64_s"])) <= 1e-15
    rows = golden_ago["_meta"]["table_d128_l4096_rows"]
    c, s = afa.build_cayley_rotary_matrix(128, 4096, dtype=torch.float64)
    assert np.max(np.abs(_np(c)[rows] - golden_ago["table_d128_l4096_rows_c"])) <= 1e-13
    assert np.max(np.abs(_np(s)[rows] - golden_ago["table_d128_l4096_rows_s"])) <= 1e-13


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_tables_reduced_precision(golden_ago, dtype):
    tol = 2e-5 if dtype == torch.float32 else 8e-3
    c, s = afa.build_cayley_rotary_matrix(32, 64, dtype=dtype)
    assert c.dtype == dtype and tuple(c.shape) == (64, 16)
    np.testing.assert_allclose(_np(c), golden_ago["table_d32_l64_c"], rtol=tol, atol=tol)
    np.testing.assert_allclose(_np(s), golden_ago["table_d32_l64_s"], rtol=tol, atol=tol)
    rows = golden_ago["_meta"]["table_d128_l4096_rows"]
    c, s = afa.build_cayley_rotary_matrix(128, 4096, dtype=dtype)
    np.testing.assert_allclose(_np(c)[rows], golden_ago["table_d128_l4096_rows_c"], rtol=tol, atol=tol)
    np.testing.assert_allclose(_np(s)[rows], golden_ago["table_d128_l4096_rows_s"], rtol=tol, atol=tol)


def test_tables_explicit_freqs_and_base(golden_ago):
    c, s = afa.build_cayley_rotary_matrix(8, 16, freqs=[0.9, 0.5, 0.1, 0.01], dtype=torch.float64)
    assert np.max(np.abs(_np(c) - golden_ago["table_d8_l16_freqs_c"])) <= 1e-15
    assert np.max(np.abs(_np(s) - golden_ago["table_d8_l16_freqs_s"])) <= 1e-15
    c, s = afa.build_cayley_rotary_matrix(16, 8, base=500.0, dtype=torch.float64)
    assert np.max(np.abs(_np(c) - golden_ago["table_d16_l8_base500_c"])) <= 1e-15


def test_matrix_property_is_a_rotation():
    rot = afa.build_cayley_rotary_matrix(16, 32, dtype=torch.float64)
    m = rot.matrix
    assert tuple(m.shape) == (32, 8, 2, 2)
    det = m[..., 0, 0] * m[..., 1, 1] - m[..., 0, 1] * m[..., 1, 0]
    assert torch.max(torch.abs(det - 1)) <= 1e-14


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32, torch.bfloat16])
def test_rotation_matches_reference(golden_ago, dtype):
    """tests/test_ago.py:25-50: (batch, seq, heads, dim) with the default
    sequence axis and tables built in the tensors' dtype."""
    q, k = inputs.ago_small()
    qt = torch.as_tensor(q, device="cuda").to(dtype)
    kt = torch.as_tensor(k, device="cuda").to(dtype)
    rot = afa.build_cayley_rotary_matrix(32, q.shape[1], dtype=dtype)
    qr, kr = afa.apply_ago_rotations(qt, kt, rotary_params=rot)
    assert qr.dtype == dtype and kr.dtype == dtype
    tol = TOL[dtype]
    np.testing.assert_allclose(_np(qr), golden_ago["ago_small_q"], rtol=tol, atol=tol)
    np.testing.assert_allclose(_np(kr), golden_ago["ago_small_k"], rtol=tol, atol=tol)


def test_rotation_attention_layout(golden_ago):
    """(batch, heads, seq, dim) with seq_axis=2: the layout the attention
    kernels take (src/model.py:262-264)."""
    q, k = inputs.ago_bhtd()
    qr, kr = afa.apply_ago_rotations(torch.as_tensor(q, device="cuda"), torch.as_tensor(k, device="cuda"),
                                     seq_axis=2)
    np.testing.assert_allclose(_np(qr), golden_ago["ago_bhtd_q"], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(_np(kr), golden_ago["ago_bhtd_k"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("shape", [(32, 16), (4, 32, 16), (2, 8, 40, 24), (3, 50, 2, 10)])
def test_rotation_shapes(shape):
    """tests/test_ago.py:115-140: 2-D, 3-D and 4-D layouts, odd pair counts
    (the per-element path) and the vectorised path."""
    rng = np.random.default_rng(7)
    q, k = rng.standard_normal(shape), rng.standard_normal(shape)
    qr, kr = afa.apply_ago_rotations(q, k)
    assert isinstance(qr, np.ndarray) and qr.shape == shape
    wq, wk = orc.ago_rotate(q, k)
    assert np.max(np.abs(qr - wq)) <= 1e-12 and np.max(np.abs(kr - wk)) <= 1e-12


def test_rotation_preserves_pair_norms():
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn((2, 4, 1000, 64), generator=g, device="cuda", dtype=torch.float64)
    k = torch.randn_like(q)
    qr, kr = afa.apply_ago_rotations(q, k, seq_axis=2)
    n0 = q.reshape(2, 4, 1000, 32, 2).norm(dim=-1)
    n1 = qr.reshape(2, 4, 1000, 32, 2).norm(dim=-1)
    assert torch.max(torch.abs(n0 - n1)) <= 1e-13


def test_rotation_bf16_config3_shape_with_float32_tables():
    """Config 3's Q/K shape in bf16 with float32 tables (cast to bf16 before
    use, src/attention.py:148-149), against the oracle on two heads."""
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn((2, 32, 4096, 128), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn_like(q)
    rot = afa.build_cayley_rotary_matrix(128, 4096, dtype=torch.float32)
    qr, kr = afa.apply_ago_rotations(q, k, rotary_params=rot, seq_axis=2)
    c16 = rot.c.to(torch.bfloat16).double().cpu().numpy()
    s16 = rot.s.to(torch.bfloat16).double().cpu().numpy()
    sel = (slice(0, 1), slice(0, 2))
    wq, wk = orc.ago_rotate(_np(q[sel]), _np(k[sel]), c16, s16, seq_axis=2)
    assert np.max(np.abs(_np(qr[sel]) - wq)) <= 0.04
    assert np.max(np.abs(_np(kr[sel]) - wk)) <= 0.04
