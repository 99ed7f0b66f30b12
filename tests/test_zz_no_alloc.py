"""The allocation-free decode entry point, afa_decode_noalloc.

Some callers cannot hand the library device scratch memory:
- code captured into a CUDA graph;
- plugin hosts whose allocator belongs to another runtime;
- serving loops that forbid allocation on the per-token path.

afa_decode_noalloc runs the same decode kernels as afa_decode but keeps the
split-KV scratch in a fixed 1 MiB device array inside the library. These tests
call it through the C ABI and check it against afa_decode, the entry point that
takes a caller workspace: the same kernels on the same inputs with the same
split count, so the results must be bit-identical (a stale or misplaced scratch
would shift them). They run two calls in a row with different inputs, so a
second call must not see the first one's scratch contents; the float64 oracle
checks the values themselves at the decode tolerances. This file is collected
last and works both alone and after the rest of the suite.
"""
import pytest
import torch

from algebraic_intelligence_b200 import _lib
from oracle import afa_oracle as orc

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2   # the bf16 bound every decode parity test uses
TOL_F32 = 1e-5


def _decode_with_workspace(lib, q, k, v, out, den, dtype_code):
    b, h, lkv, d = k.shape
    need = lib.afa_decode_workspace_bytes(b, h, lkv, d)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    rc = lib.afa_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), den.data_ptr(), b, h, lkv, d,
                        dtype_code, 0.5, None, 0, ws.data_ptr(), need, _lib.stream_ptr(q.device))
    _lib.check(rc, "afa_decode")
    return need


def _decode_noalloc(lib, q, k, v, out, den, dtype_code):
    b, h, lkv, d = k.shape
    rc = lib.afa_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), den.data_ptr(), b, h, lkv,
                                d, dtype_code, 0.5, None, 0, _lib.stream_ptr(q.device))
    _lib.check(rc, "afa_decode_noalloc")


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, TOL_BF16), (torch.float32, TOL_F32)])
def test_noalloc_matches_workspace_entry_two_calls(dtype, tol):
    lib = _lib.load()
    code = _lib.dtype_code(dtype)
    dev = torch.device("cuda", torch.cuda.current_device())
    # Few heads over a long cache: the step splits the keys across CTAs and needs scratch.
    b, h, lkv, d = 1, 2, 70000, 128
    assert lib.afa_decode_workspace_bytes(b, h, lkv, d) > 0
    g = torch.Generator(device=dev).manual_seed(123)
    for call in range(2):
        q = torch.randn((b, h, d), generator=g, device=dev).to(dtype)
        k = torch.randn((b, h, lkv, d), generator=g, device=dev).to(dtype)
        v = torch.randn((b, h, lkv, d), generator=g, device=dev).to(dtype)
        ref_out = torch.empty((b, h, d), dtype=dtype, device=dev)
        ref_den = torch.empty((b, h), dtype=torch.float32, device=dev)
        out = torch.full((b, h, d), float("nan"), dtype=dtype, device=dev)
        den = torch.full((b, h), float("nan"), dtype=torch.float32, device=dev)
        _decode_with_workspace(lib, q, k, v, ref_out, ref_den, code)
        _decode_noalloc(lib, q, k, v, out, den, code)
        torch.cuda.synchronize(dev)
        assert torch.isfinite(out.float()).all(), f"call {call}: non-finite output"
        assert torch.equal(out, ref_out), f"call {call}"
        assert torch.equal(den, ref_den), f"call {call}"
        want, _ = orc.decode(q.double().cpu().numpy(), k.double().cpu().numpy(), v.double().cpu().numpy(), sink=0.5)
        assert orc.rel_err(out.double().cpu().numpy(), want) <= tol, f"call {call}"
    assert _lib.device_status(dev) == 0


def test_noalloc_shape_without_scratch():
    """Shapes that already fill the GPU need no scratch; the entry point still works."""
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    b, h, lkv, d = 32, 32, 1024, 128
    assert lib.afa_decode_workspace_bytes(b, h, lkv, d) == 0
    g = torch.Generator(device=dev).manual_seed(7)
    q = torch.randn((b, h, d), generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn((b, h, lkv, d), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((b, h, lkv, d), generator=g, device=dev).to(torch.bfloat16)
    ref_out, out = (torch.empty((b, h, d), dtype=torch.bfloat16, device=dev) for _ in range(2))
    ref_den, den = (torch.empty((b, h), dtype=torch.float32, device=dev) for _ in range(2))
    _decode_with_workspace(lib, q, k, v, ref_out, ref_den, _lib.AFA_BF16)
    _decode_noalloc(lib, q, k, v, out, den, _lib.AFA_BF16)
    assert torch.equal(out, ref_out) and torch.equal(den, ref_den)


def test_noalloc_shape_on_the_cuda_core_path():
    """float32 with head_dim 256 runs the CUDA-core kernel, which needs no
    scratch, so the entry point accepts it even though the split-KV size
    formula for this shape is above the fixed 1 MiB."""
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    b, h, lkv, d = 1, 520, 1024, 256
    assert lib.afa_decode_workspace_bytes(b, h, lkv, d) > (1 << 20)
    g = torch.Generator(device=dev).manual_seed(11)
    q = torch.randn((b, h, d), generator=g, device=dev)
    k = torch.randn((b, h, lkv, d), generator=g, device=dev)
    v = torch.randn((b, h, lkv, d), generator=g, device=dev)
    ref_out, out = (torch.empty((b, h, d), device=dev) for _ in range(2))
    ref_den, den = (torch.empty((b, h), device=dev) for _ in range(2))
    _decode_with_workspace(lib, q, k, v, ref_out, ref_den, _lib.AFA_F32)
    _decode_noalloc(lib, q, k, v, out, den, _lib.AFA_F32)
    assert torch.equal(out, ref_out) and torch.equal(den, ref_den)


def test_noalloc_rejects_shapes_beyond_its_scratch():
    """A shape whose scratch exceeds the fixed 1 MiB fails with a clear message,
    before touching the GPU."""
    lib = _lib.load()
    b, h, lkv, d = 1, 520, 1 << 20, 256
    assert lib.afa_decode_workspace_bytes(b, h, lkv, d) > (1 << 20)
    rc = lib.afa_decode_noalloc(1, 1, 1, 1, None, b, h, lkv, d, _lib.AFA_BF16, 0.5, None, 0, None)
    assert rc == _lib.AFA_ERR_INVALID
    assert b"scratch" in lib.afa_last_error()
