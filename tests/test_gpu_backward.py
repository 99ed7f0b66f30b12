"""AFA backward on the GPU (tiled_afa_backward, src/kernels/pallas_afa.py:409-522)
against the float64 oracle ``afa_backward``, which is pinned by finite
differences of the golden-pinned forward.

Cases follow the reference's backward tests (tests/test_pallas_afa.py:292-396):
  - float64 agreement with exact autodiff (there rtol 2e-6 / 1e-5; here 1e-10,
    the oracle being the exact gradient);
  - bf16 inputs with fp32 accumulation within 6e-3 of the float32 backward
    (:325-352), and within the north star's 2e-2 of the float64 oracle;
  - pallas_afa differentiable end to end (:355-396), now through torch autograd.
Plus float32 at the north star's 1e-5, ragged lengths, valid_seq_len, head dims
8 to 256.
"""
import numpy as np
import pytest
import torch

import algebraic_intelligence_b200 as afa
from algebraic_intelligence_b200 import _lib
from oracle import afa_oracle as orc

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b)) / np.max(np.abs(b)))


def _inputs(shape, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(shape, generator=g, device="cuda", dtype=torch.float64).to(dtype) for _ in range(4)]


def _gpu_backward(q, k, v, g, causal, valid=None):
    n = q.shape[2]  # one tile per block: pallas_afa_forward keeps the reference's divisibility rule
    out, den = afa.pallas_afa_forward(q, k, v, causal=causal, block_q=n, block_k=n, valid_seq_len=valid,
                                      return_denominator=True)
    return afa.tiled_afa_backward(q, k, v, out, den, g, causal=causal, valid_seq_len=valid)


def _oracle(q, k, v, g, causal, valid=None):
    qn, kn, vn, gn = (t.double().cpu().numpy() for t in (q, k, v, g))
    return orc.afa_backward(qn, kn, vn, gn, causal=causal, valid_len=valid)


@pytest.mark.parametrize("shape", [(1, 2, 256, 64), (2, 1, 200, 8), (1, 1, 130, 256)])
@pytest.mark.parametrize("causal", [False, True])
def test_backward_fp64_matches_oracle(shape, causal):
    q, k, v, g = _inputs(shape, torch.float64, 301)
    got = _gpu_backward(q, k, v, g, causal)
    want = _oracle(q, k, v, g, causal)
    for a, b in zip(got, want):
        assert a.dtype == torch.float64
        assert _rel(a.cpu().numpy(), b) <= 1e-10


@pytest.mark.parametrize("shape", [(1, 2, 256, 64), (1, 2, 300, 128), (2, 2, 128, 32), (1, 1, 96, 256)])
@pytest.mark.parametrize("causal", [False, True])
def test_backward_fp32_matches_oracle(shape, causal):
    q, k, v, g = _inputs(shape, torch.float32, 302)
    got = _gpu_backward(q, k, v, g, causal)
    want = _oracle(q, k, v, g, causal)
    for a, b in zip(got, want):
        assert _rel(a.cpu().numpy(), b) <= 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_backward_valid_seq_len(dtype):
    q, k, v, g = _inputs((1, 2, 256, 64), dtype, 303)
    got = _gpu_backward(q, k, v, g, True, valid=150)
    want = _oracle(q, k, v, g, True, valid=150)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    for a, b in zip(got, want):
        assert _rel(a.float().cpu().numpy(), b) <= tol
    # Keys at index >= valid_seq_len receive no gradient.
    assert torch.count_nonzero(got[1][:, :, 150:]) == 0
    assert torch.count_nonzero(got[2][:, :, 150:]) == 0


@pytest.mark.parametrize("shape", [(1, 1, 128, 32), (1, 2, 512, 64), (1, 2, 384, 128)])
def test_backward_bf16_close_to_fp32(shape):
    """tests/test_pallas_afa.py:325-352: bf16 products with fp32 accumulation
    stay within 6e-3 of the float32 backward on the same (bf16-valued) inputs."""
    q, k, v, g = _inputs(shape, torch.bfloat16, 812)
    out, den = afa.pallas_afa_forward(q, k, v, causal=True, return_denominator=True)
    mixed = afa.tiled_afa_backward(q, k, v, out, den, g, causal=True)
    fp32 = afa.tiled_afa_backward(q.float(), k.float(), v.float(), out.float(), den, g.float(), causal=True)
    for a, b in zip(mixed, fp32):
        assert a.dtype == torch.bfloat16
        assert _rel(a.float().cpu().numpy(), b.cpu().numpy()) <= 6e-3


@pytest.mark.parametrize("shape", [(1, 2, 512, 128), (1, 2, 300, 64), (2, 1, 256, 96)])
@pytest.mark.parametrize("causal", [False, True])
def test_backward_bf16_matches_oracle(shape, causal):
    q, k, v, g = _inputs(shape, torch.bfloat16, 304)
    got = _gpu_backward(q, k, v, g, causal)
    want = _oracle(q, k, v, g, causal)
    for a, b in zip(got, want):
        assert _rel(a.float().cpu().numpy(), b) <= 2e-2


def test_backward_config3_subset_bf16():
    """Two heads of config 3's shape (L=4096, D=128, causal) against the oracle."""
    q, k, v, g = _inputs((1, 2, 4096, 128), torch.bfloat16, 305)
    got = _gpu_backward(q, k, v, g, True)
    want = _oracle(q, k, v, g, True)
    for a, b in zip(got, want):
        assert _rel(a.float().cpu().numpy(), b) <= 2e-2


def test_pallas_afa_autograd_matches_oracle():
    """tests/test_pallas_afa.py:375-396: jax.grad through pallas_afa equals
    autodiff of the exact reference (rtol 2e-6); here torch autograd through
    the float64 path against the exact oracle gradient."""
    q, k, v, g = _inputs((1, 1, 64, 8), torch.float64, 304)
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    out = afa.pallas_afa(*leaves, causal=True, block_q=32, block_k=64)
    torch.autograd.backward(out, g)
    want = _oracle(q, k, v, g, True)
    for leaf, b in zip(leaves, want):
        np.testing.assert_allclose(leaf.grad.cpu().numpy(), b, rtol=2e-6, atol=2e-7)


def test_pallas_afa_autograd_fp32_finite():
    """tests/test_pallas_afa.py:355-372: value_and_grad of sum(pallas_afa)."""
    q, k, v, _ = _inputs((1, 1, 128, 32), torch.float32, 302)
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    loss = afa.pallas_afa(*leaves, sink_omega=0.5, causal=True, block_q=64, block_k=64).sum()
    loss.backward()
    assert torch.isfinite(loss)
    for leaf in leaves:
        assert leaf.grad is not None and torch.isfinite(leaf.grad).all()


def test_backward_numpy_host_buffers():
    rng = np.random.default_rng(9)
    q, k, v, g = (rng.standard_normal((1, 1, 64, 16)) for _ in range(4))
    out, den = afa.pallas_afa_forward(q, k, v, causal=True, block_q=64, block_k=64, return_denominator=True)
    dq, dk, dv = afa.tiled_afa_backward(q, k, v, out, den, g, causal=True)
    assert isinstance(dq, np.ndarray)
    want = orc.afa_backward(q, k, v, g, causal=True)
    for a, b in zip((dq, dk, dv), want):
        assert _rel(a, b) <= 1e-10
    assert _lib.device_status(torch.device("cuda", 0)) == 0
