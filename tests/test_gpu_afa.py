"""GPU parity of the AFA forward, algebraic_softmax and octic kernels against the
float64 oracle (oracle/afa_oracle.py, pinned to the reference in
test_oracle.py) and the golden fixtures.

Tolerances (max|y - ref| / max|ref|, the reference's metric,
tests/test_pallas_afa.py:85-87):
  float32 1e-5 and bfloat16 2e-2; float64 1e-12.
The oracle always sees the exact values the GPU saw (inputs rounded to the
kernel dtype first).
"""
import numpy as np
import pytest
import torch

import algebraic_intelligence_b200 as afa
from algebraic_intelligence_b200 import _lib
import inputs
from oracle import afa_oracle as orc

pytestmark = pytest.mark.gpu

TOL = {torch.float64: 1e-12, torch.float32: 1e-5, torch.bfloat16: 2e-2}


def to_dev(a, dtype):
    return torch.as_tensor(np.asarray(a)).to("cuda").to(dtype).contiguous()


def host64(t):
    return t.detach().to("cpu", torch.float64).numpy()


def make_qkv(shape, dtype, seed=0, outlier_frac=0.0, outlier_shift=8.0, scale=1.0):
    """Q, K, V ~ N(0,1) (float32 draw, then cast), optionally with a fraction of
    key rows per (batch, head) shifted by +outlier_shift in every coordinate."""
    rng = np.random.default_rng(seed)
    q, k, v = ((rng.normal(size=shape) * scale).astype(np.float32) for _ in range(3))
    if outlier_frac:
        b, h, l, _ = shape
        n = int(round(outlier_frac * l))
        for bi in range(b):
            for hi in range(h):
                rows = rng.choice(l, size=n, replace=False)
                k[bi, hi, rows, :] += outlier_shift
    ts = [to_dev(x, dtype) for x in (q, k, v)]
    return ts, [host64(t) for t in ts]


# ---------------------------------------------------------------------------
# octic map
# ---------------------------------------------------------------------------
def test_octic_kernel_golden_fp64(golden):
    y = afa.octic_kernel(to_dev(inputs.octic_grid(), torch.float64))
    np.testing.assert_allclose(host64(y), golden["octic_y"], rtol=1e-13, atol=0)


def test_octic_kernel_fp32_and_negative_tail():
    # tests/test_pallas_afa.py:90-96: the negative tail stays positive and matches
    x = np.r_[np.linspace(-64, 64, 4001), -1e2, -1e3, -1e4].astype(np.float32)
    y = host64(afa.octic_kernel(to_dev(x, torch.float32)))
    ref = orc.octic(x.astype(np.float64))
    assert np.all(y > 0)
    np.testing.assert_allclose(y, ref, rtol=2e-5, atol=0)
    assert afa.octic_kernel(to_dev([2.0], torch.float64)).item() == pytest.approx(51841 + 23184 * 5 ** 0.5,
                                                                                  rel=2e-15)


# ---------------------------------------------------------------------------
# algebraic_softmax (tests/test_attention.py:14-25, :56-64 of the reference)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype,tol", [(torch.float64, 2e-13), (torch.float32, 2e-5), (torch.bfloat16, 0.016),
                                       (torch.float16, 0.016)])
@pytest.mark.parametrize("sink", [0.0, 0.5, 1.0])
def test_softmax_matches_oracle(golden, dtype, tol, sink):
    x = to_dev(inputs.softmax_rows(), dtype)
    y = afa.algebraic_softmax(x, sink)
    assert y.dtype == dtype and y.shape == x.shape
    ref = golden[f"asm_y_sink{sink}"] if dtype == torch.float64 else orc.attention(host64(x), sink)
    np.testing.assert_allclose(host64(y), ref, rtol=tol, atol=tol)


@pytest.mark.parametrize("length", [1, 64, 4096])
def test_softmax_simplex_extremes(length):
    rng = np.random.default_rng(9)
    for x in (np.zeros((2, length)), np.full((2, length), -1e15), rng.normal(size=(2, length)) * 1e15):
        for sink in (0.0, 0.5, 1.0):
            p = host64(afa.algebraic_softmax(to_dev(x, torch.float64), sink))
            assert np.isfinite(p).all() and np.all(p > 0)
            assert np.max(p.sum(axis=-1)) <= 1 + 16 * np.finfo(np.float64).eps


def test_softmax_long_rows_golden(golden):
    y = afa.algebraic_softmax(to_dev(inputs.softmax_long_rows(), torch.float64), 0.5)
    np.testing.assert_allclose(host64(y), golden["asm_long_y"], rtol=2e-7, atol=1e-30)


@pytest.mark.parametrize("cols", [3, 100, 1000, 1500, 5000])
def test_softmax_row_kernels_fp32(cols):
    x = to_dev(np.random.default_rng(cols).normal(size=(37, cols)), torch.float32)
    y = afa.algebraic_softmax(x)
    np.testing.assert_allclose(host64(y), orc.attention(host64(x)), rtol=2e-5, atol=2e-5)


def test_softmax_numpy_in_numpy_out():
    x = inputs.softmax_rows()
    y = afa.algebraic_softmax(x)
    assert isinstance(y, np.ndarray) and y.dtype == np.float64
    np.testing.assert_allclose(y, orc.attention(x), rtol=2e-13, atol=2e-13)


def test_config1_algebraic_softmax_path(golden):
    """S = QK^T/sqrt(D) -> algebraic_softmax -> P V, fp32."""
    q, k, v = (to_dev(a, torch.float32) for a in inputs.config1())
    torch.backends.cuda.matmul.allow_tf32 = False
    s = torch.matmul(q, k.transpose(-1, -2)) / (q.shape[-1] ** 0.5)
    o = torch.matmul(afa.algebraic_softmax(s, 0.5, 1e-5), v)
    assert orc.rel_err(host64(o), golden["cfg1_softmax_o"]) <= TOL[torch.float32]


# ---------------------------------------------------------------------------
# AFA forward
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("causal", [False, True])
def test_fwd_fp64_golden(golden, causal):
    q, k, v = (to_dev(a, torch.float64) for a in inputs.afa_small())
    y = afa.pallas_afa_forward(q, k, v, causal=causal, block_q=64, block_k=64)
    ref = golden["afa_small_y_causal" if causal else "afa_small_y"]
    assert orc.rel_err(host64(y), ref) <= TOL[torch.float64]


def test_fwd_config1_fp32_golden(golden):
    q, k, v = (to_dev(a, torch.float32) for a in inputs.config1())
    y = afa.pallas_afa_forward(q, k, v)
    assert y.dtype == torch.float32
    assert orc.rel_err(host64(y), golden["cfg1_afa_o"]) <= TOL[torch.float32]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("causal", [False, True])
def test_unified_entry_ragged_l180(golden, dtype, causal):
    """tests/test_pallas_afa.py:173-186: L = 180 is not a tile multiple."""
    q, k, v = (to_dev(a, dtype) for a in inputs.afa_l180())
    y = afa.algebraic_flash_attention(q, k, v, causal=causal)
    assert y.shape == q.shape
    if dtype == torch.float32:
        ref = golden["afa_l180_y_causal" if causal else "afa_l180_y"]
    else:
        ref = orc.afa(host64(q), host64(k), host64(v), causal=causal)
    assert orc.rel_err(host64(y), ref) <= TOL[dtype]


# The reference's hardware parity grid (scripts/run_phase6_tpu.py:59-68) plus
# D=128 and the tensor-core D=64 path.
PARITY = [
    ((1, 4, 256, 64), torch.float32),
    ((1, 8, 512, 64), torch.float32),
    ((1, 8, 1024, 64), torch.bfloat16),
    ((1, 8, 2048, 64), torch.bfloat16),
    ((1, 4, 1024, 128), torch.bfloat16),
    ((2, 2, 640, 128), torch.bfloat16),
    ((1, 2, 384, 128), torch.float32),
    ((1, 2, 256, 32), torch.bfloat16),   # CUDA-core bf16 path (head_dim 32)
    ((1, 1, 256, 256), torch.bfloat16),  # CUDA-core bf16 path (head_dim 256)
]


@pytest.mark.parametrize("shape,dtype", PARITY)
@pytest.mark.parametrize("causal", [False, True])
def test_fwd_parity_grid(shape, dtype, causal):
    (q, k, v), (qh, kh, vh) = make_qkv(shape, dtype, seed=642)
    y, den = afa.pallas_afa_forward(q, k, v, causal=causal, return_denominator=True)
    ref, rden = orc.afa_with_denominator(qh, kh, vh, causal=causal)
    assert y.dtype == dtype and den.dtype == torch.float32
    assert orc.rel_err(host64(y), ref) <= TOL[dtype]
    assert orc.rel_err(host64(den), rden) <= (1e-5 if dtype == torch.float32 else 1e-3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("length", [1, 100, 129, 300, 1000])
def test_fwd_any_length(dtype, length):
    (q, k, v), (qh, kh, vh) = make_qkv((1, 3, length, 128), dtype, seed=length)
    for causal in (False, True):
        y = afa.algebraic_flash_attention(q, k, v, causal=causal)
        assert orc.rel_err(host64(y), orc.afa(qh, kh, vh, causal=causal)) <= TOL[dtype]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fwd_valid_seq_len(dtype):
    (q, k, v), (qh, kh, vh) = make_qkv((1, 2, 512, 128), dtype, seed=11)
    for valid, causal in ((300, False), (129, True), (512, False)):
        y = afa.pallas_afa_forward(q, k, v, causal=causal, valid_seq_len=valid)
        ref, _ = orc.afa_blocked(qh, kh, vh, causal=causal, valid_len=valid)
        assert orc.rel_err(host64(y), ref) <= TOL[dtype]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_causal_prefix_invariance(dtype):
    """tests/test_pallas_afa.py:151-158: perturbing keys/values at positions >= 150
    must leave every output row before 150 bit-identical."""
    (q, k, v), _ = make_qkv((1, 1, 256, 128), dtype, seed=104)
    y = afa.pallas_afa_forward(q, k, v, causal=True)
    k2, v2 = k.clone(), v.clone()
    k2[:, :, 150:] += 10.0
    v2[:, :, 150:] += 10.0
    y2 = afa.pallas_afa_forward(q, k2, v2, causal=True)
    assert torch.equal(y[:, :, :150], y2[:, :, :150])


def test_fwd_deterministic():
    (q, k, v), _ = make_qkv((2, 4, 1024, 128), torch.bfloat16, seed=1)
    a = afa.pallas_afa_forward(q, k, v, causal=True)
    b = afa.pallas_afa_forward(q, k, v, causal=True)
    assert torch.equal(a, b)


def test_fwd_numpy_host_buffers():
    rng = np.random.default_rng(2)
    q, k, v = (rng.normal(size=(1, 2, 256, 64)).astype(np.float32) for _ in range(3))
    y = afa.pallas_afa_forward(q, k, v, causal=True)
    assert isinstance(y, np.ndarray) and y.dtype == np.float32
    assert orc.rel_err(y, orc.afa(q, k, v, causal=True)) <= TOL[torch.float32]


def test_fwd_float16_rejected():
    x = torch.zeros((1, 1, 128, 64), dtype=torch.float16, device="cuda")
    with pytest.raises(TypeError, match="float16"):
        afa.pallas_afa_forward(x, x, x)


def _subset_rel_err(y, qh, kh, vh, heads, rows, causal):
    worst = 0.0
    for b, h in heads:
        ref, _ = orc.afa_blocked(qh[b, h], kh[b, h], vh[b, h], causal=causal, rows=rows, block=256)
        worst = max(worst, orc.rel_err(host64(y[b, h, rows]), ref))
    return worst


def test_config2_prefill_outliers():
    """B=4,H=16,L=2048,D=128 bf16 causal, 5% of K rows +8."""
    shape = (4, 16, 2048, 128)
    (q, k, v), _ = make_qkv(shape, torch.bfloat16, seed=0, outlier_frac=0.05)
    y = afa.pallas_afa_forward(q, k, v, causal=True)
    qh, kh, vh = (host64(t[:, :4]) for t in (q, k, v))  # oracle on 4 heads per batch row
    heads = [(b, h) for b in range(4) for h in (0, 3)]
    rows = np.arange(2048)
    assert _subset_rel_err(y[:, :4], qh, kh, vh, heads, rows, True) <= TOL[torch.bfloat16]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_config3_prefill(dtype):
    """B=2,H=32,L=4096,D=128 causal (bf16, and the fp32 rerun)."""
    shape = (2, 32, 4096, 128)
    (q, k, v), _ = make_qkv(shape, dtype, seed=0)
    y = afa.pallas_afa_forward(q, k, v, causal=True)
    sel = [(0, 0), (1, 31)]
    qh, kh, vh = ({(b, h): host64(t[b, h]) for b, h in sel} for t in (q, k, v))
    rows = np.r_[0:256, 1900:2100, 3840:4096]
    worst = 0.0
    for key in sel:
        ref, _ = orc.afa_blocked(qh[key], kh[key], vh[key], causal=True, rows=rows, block=256)
        worst = max(worst, orc.rel_err(host64(y[key[0], key[1], rows]), ref))
    assert worst <= TOL[dtype]


def test_config5_prefill_l65536():
    """BASELINE config 5 at one GPU (the bench's headline launch): B=1, H=16,
    L=65536, D=128 bf16 causal, 256 key tiles for the last query pairs. As the
    reference checked its long runs on hardware (scripts/run_phase6_tpu.py:54-126),
    the float64 oracle covers a subset: heads 0 and 15, rows at the start, the
    middle and the end of the sequence. Output at 2e-2, d_total at 1e-3."""
    shape = (1, 16, 65536, 128)
    g = torch.Generator(device="cuda").manual_seed(65536)
    q, k, v = (torch.randn(shape, generator=g, device="cuda", dtype=torch.float32).to(torch.bfloat16)
               for _ in range(3))
    y, den = afa.pallas_afa_forward(q, k, v, causal=True, return_denominator=True)
    rows = np.r_[0:256, 32640:32896, 65280:65536]
    worst_o = worst_d = 0.0
    for h in (0, 15):
        qh, kh, vh = (host64(t[0, h]) for t in (q, k, v))
        ref, rden = orc.afa_blocked(qh, kh, vh, causal=True, rows=rows, block=256)
        worst_o = max(worst_o, orc.rel_err(host64(y[0, h, rows]), ref))
        worst_d = max(worst_d, orc.rel_err(host64(den[0, h, rows]).reshape(rden.shape), rden))
    assert worst_o <= TOL[torch.bfloat16]
    assert worst_d <= 1e-3


def test_device_status_clean_after_runs():
    (q, k, v), _ = make_qkv((1, 2, 512, 128), torch.bfloat16, seed=3)
    afa.pallas_afa_forward(q, k, v, causal=True)
    assert _lib.device_status(q.device) == 0


def test_bounded_wait_reports_instead_of_hanging():
    """Failure detection: a wait on a barrier nothing releases gives up after
    its budget (1 ms here) and the host reads the status; the context stays
    usable afterwards."""
    lib = _lib.load()
    dev = torch.device("cuda")
    assert _lib.device_status(dev) == 0
    _lib.check(lib.afa_selftest_bounded_wait(1_000_000, _lib.stream_ptr(dev)), "selftest")
    assert _lib.device_status(dev, clear=True) == 0x1FF
    assert _lib.device_status(dev) == 0
    x = to_dev(inputs.softmax_rows(), torch.float32)
    np.testing.assert_allclose(host64(afa.algebraic_softmax(x)), orc.attention(host64(x)), rtol=2e-5, atol=2e-5)


# ---------------------------------------------------------------------------
# algebraic_softmax backward (the custom VJP, src/attention.py:70-85)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype,tol", [(torch.float64, 2e-13), (torch.float32, 2e-5), (torch.bfloat16, 0.016)])
@pytest.mark.parametrize("sink", [0.0, 0.5, 1.0])
def test_softmax_vjp_golden(golden, dtype, tol, sink):
    """tests/test_attention.py:14-26: the VJP against the reference oracle's
    attention_vjp, with the same rtol = atol per dtype."""
    x, g, _, _ = inputs.softmax_vjp()
    xt = torch.as_tensor(x, device="cuda").to(dtype)
    gt = torch.as_tensor(g, device="cuda").to(dtype)
    dx = afa.algebraic_softmax_vjp(xt, gt, sink)
    assert dx.dtype == dtype
    # The oracle ran on the float64 draws; for bf16 compare on the rounded inputs.
    want = golden[f"asm_vjp_sink{sink}"] if dtype != torch.bfloat16 else orc.attention_vjp(
        xt.double().cpu().numpy(), gt.double().cpu().numpy(), sink)
    np.testing.assert_allclose(dx.double().cpu().numpy(), want, rtol=tol, atol=tol)


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-12), (torch.float32, 2e-5)])
def test_softmax_vjp_long_rows(golden, dtype, tol):
    """3000 columns: the CTA-per-row backward kernel."""
    _, _, xl, gl = inputs.softmax_vjp()
    dx = afa.algebraic_softmax_vjp(torch.as_tensor(xl, device="cuda").to(dtype),
                                   torch.as_tensor(gl, device="cuda").to(dtype), 0.5)
    want = golden["asm_vjp_long"]
    assert np.max(np.abs(dx.double().cpu().numpy() - want)) <= tol * np.max(np.abs(want)) * 10


@pytest.mark.parametrize("cols", [1, 31, 200, 512, 1000, 1024, 1500])
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_softmax_autograd_against_oracle(cols, dtype):
    """torch autograd through algebraic_softmax (jax.vjp in the reference),
    every warp-row width and the CTA path."""
    g0 = torch.Generator(device="cuda").manual_seed(cols)
    x = torch.randn((5, cols), generator=g0, device="cuda", dtype=torch.float64).to(dtype).requires_grad_(True)
    g = torch.randn((5, cols), generator=g0, device="cuda", dtype=torch.float64).to(dtype)
    y = afa.algebraic_softmax(x, 0.5)
    y.backward(g)
    want = orc.attention_vjp(x.detach().double().cpu().numpy(), g.double().cpu().numpy(), 0.5)
    tol = 1e-12 if dtype == torch.float64 else 2e-5
    assert np.max(np.abs(x.grad.double().cpu().numpy() - want)) <= tol * max(1.0, np.max(np.abs(want)))


def test_softmax_vjp_float16_and_numpy():
    rng = np.random.default_rng(3)
    x, g = rng.normal(size=(4, 64)), rng.normal(size=(4, 64))
    dx = afa.algebraic_softmax_vjp(x, g, 0.5)
    assert isinstance(dx, np.ndarray)
    assert np.max(np.abs(dx - orc.attention_vjp(x, g, 0.5))) <= 1e-12
    xh = torch.as_tensor(x, device="cuda").half()
    gh = torch.as_tensor(g, device="cuda").half()
    dxh = afa.algebraic_softmax_vjp(xh, gh, 0.5)
    want = orc.attention_vjp(xh.double().cpu().numpy(), gh.double().cpu().numpy(), 0.5)
    assert dxh.dtype == torch.float16
    np.testing.assert_allclose(dxh.double().cpu().numpy(), want, rtol=0.016, atol=0.016)


# ---------------------------------------------------------------------------
# Host inputs: the pipelined chunked path (copies overlapping kernels)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("shape,causal", [((2, 8, 1024, 128), True), ((1, 3, 700, 64), False), ((3, 2, 300, 128), True)])
def test_host_inputs_match_device_path(shape, causal):
    """pallas_afa_forward on pinned CPU tensors and on NumPy arrays gives the
    device path's output bit for bit (the chunks run the same kernel on the same
    rows), including d_total."""
    g = torch.Generator(device="cuda").manual_seed(31)
    q, k, v = (torch.randn(shape, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    n = shape[2]
    want, wden = afa.pallas_afa_forward(q, k, v, causal=causal, block_q=n, block_k=n, return_denominator=True)
    qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
    got, gden = afa.pallas_afa_forward(qh, kh, vh, causal=causal, block_q=n, block_k=n, return_denominator=True)
    assert not got.is_cuda and got.dtype == torch.bfloat16
    assert torch.equal(got, want.cpu()) and torch.equal(gden, wden.cpu())
    qn, kn, vn = (t.float().cpu().numpy() for t in (q, k, v))
    out_np = afa.pallas_afa_forward(qn, kn, vn, causal=causal, block_q=n, block_k=n)
    assert isinstance(out_np, np.ndarray) and out_np.shape == shape
    ref = afa.pallas_afa_forward(*(torch.as_tensor(a, device="cuda") for a in (qn, kn, vn)), causal=causal,
                                 block_q=n, block_k=n)
    assert np.array_equal(out_np, ref.cpu().numpy())


def test_octic_kernel_gradient():
    """tests/test_attention.py:28-35: grad of sum(octic_kernel(x)) equals
    8 rho(x)^8 / sqrt(1 + x^2) (rtol 2e-13 in float64), tails included."""
    x = np.r_[np.linspace(-64, 64, 1001), -1e3, 1e3]
    xt = torch.as_tensor(x, device="cuda").requires_grad_(True)
    afa.octic_kernel(xt).sum().backward()
    want = 8 * orc.octic(x) / np.sqrt(1 + x ** 2)
    np.testing.assert_allclose(xt.grad.cpu().numpy(), want, rtol=2e-13)
    x32 = torch.linspace(-8, 8, 4097, device="cuda", dtype=torch.float32).requires_grad_(True)
    g = torch.randn(4097, device="cuda")
    afa.octic_kernel(x32).backward(g)
    want32 = 8 * orc.octic(x32.detach().double().cpu().numpy()) / np.sqrt(1 + x32.detach().double().cpu().numpy() ** 2)
    np.testing.assert_allclose(x32.grad.double().cpu().numpy(), want32 * g.double().cpu().numpy(), rtol=2e-5, atol=1e-30)
