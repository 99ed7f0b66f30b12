"""The C-ABI library loads and exports every symbol include/afa_b200.h declares;
argument checks answer before any CUDA call (no GPU needed)."""
import ctypes
import re

import pytest

from algebraic_intelligence_b200 import _lib

HEADER = _lib.LIB_PATH.parents[1] / "include" / "afa_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"AFA_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)))


def test_header_declares_the_reference_boundary():
    names = declared_symbols()
    for required in ("afa_fwd", "afa_fwd_hop", "afa_finalize", "afa_decode", "algebraic_softmax_fwd",
                     "afa_octic", "afa_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), f"libafa_b200.so does not export {name}"
    assert set(declared_symbols()) == set(_lib.SIGNATURES), "ctypes signatures and header disagree"


def test_version_and_error_string():
    lib = _lib.load()
    assert b"sm_100a" in lib.afa_version()
    assert isinstance(lib.afa_last_error(), bytes)


def test_fwd_rejects_float16_before_any_cuda_call():
    lib = _lib.load()
    rc = lib.afa_fwd(1, 1, 1, 1, None, 1, 1, 128, 64, _lib.AFA_F16, 0.5, 0, 0, None)
    assert rc == _lib.AFA_ERR_DTYPE
    assert b"float16" in lib.afa_last_error()


@pytest.mark.parametrize("args,needle", [
    ((None, 1, 1, 1, None, 1, 1, 128, 64, _lib.AFA_BF16, 0.5, 0, 0, None), b"non-null"),
    ((1, 1, 1, 1, None, 1, 1, 128, 0, _lib.AFA_BF16, 0.5, 0, 0, None), b"head dimension must be positive"),
    ((1, 1, 1, 1, None, 1, 1, 128, 64, _lib.AFA_BF16, -1.0, 0, 0, None), b"sink_omega"),
    ((1, 1, 1, 1, None, 1, 1, 128, 64, _lib.AFA_BF16, float("inf"), 0, 0, None), b"sink_omega"),
    ((1, 1, 1, 1, None, 1, 1, 128, 64, _lib.AFA_BF16, 0.5, 0, 129, None), b"valid_seq_len"),
])
def test_fwd_argument_checks(args, needle):
    lib = _lib.load()
    assert lib.afa_fwd(*args) == _lib.AFA_ERR_INVALID
    assert needle in lib.afa_last_error()


def test_softmax_argument_checks():
    lib = _lib.load()
    assert lib.algebraic_softmax_fwd(1, 1, 1, 4, _lib.AFA_F32, -1.0, 1e-5, None) == _lib.AFA_ERR_INVALID
    assert b"sink_omega" in lib.afa_last_error()
    assert lib.algebraic_softmax_fwd(1, 1, 1, 4, _lib.AFA_F32, 0.5, 0.0, None) == _lib.AFA_ERR_INVALID
    assert b"eps" in lib.afa_last_error()
    assert lib.algebraic_softmax_fwd(1, 1, 1, 0, _lib.AFA_F32, 0.5, 1e-5, None) == _lib.AFA_ERR_INVALID
    assert b"nonempty" in lib.afa_last_error()
    assert lib.algebraic_softmax_fwd(1, 1, 1, 4, 9, 0.5, 1e-5, None) == _lib.AFA_ERR_DTYPE


def test_hop_argument_checks():
    lib = _lib.load()
    probs = (ctypes.c_int * 20)(0, 128, 0, 1, 0, 128, 0, 0, 0, 0,
                                64, 128, 64, 1, 0, 128, 0, 0, 0, 0)
    rc = lib.afa_fwd_hop(1, 1, 1, 1, 1, None, None, 1, 1, 256, 256, 64, _lib.AFA_BF16, probs, 2, 0,
                         _lib.AFA_HOP_STORE, 0.5, None)
    assert rc == _lib.AFA_ERR_INVALID and b"overlapping" in lib.afa_last_error()
    two = (ctypes.c_int * 10)(0, 128, 0, 2, 0, 128, 0, 128, 64, 128)
    rc = lib.afa_fwd_hop(1, 1, 1, 1, 1, None, None, 1, 1, 128, 256, 64, _lib.AFA_BF16, two, 1, 1,
                         _lib.AFA_HOP_STORE, 0.5, None)
    assert rc == _lib.AFA_ERR_INVALID and b"first key segment" in lib.afa_last_error()
    rc = lib.afa_fwd_hop(1, 1, 1, None, None, None, None, 1, 1, 128, 128, 64, _lib.AFA_BF16, probs, 1, 0,
                         _lib.AFA_HOP_ACCUMULATE, 0.5, None)
    assert rc == _lib.AFA_ERR_INVALID and b"o_acc" in lib.afa_last_error()


def test_hop_shared_query_rows_only_where_pieces_add():
    """Two problems over the same query rows (two ring hops in one launch) are
    accepted only in AFA_HOP_ACCUMULATE on the tensor cores, whose persistent
    kernel adds every piece with reductions; elsewhere the overlap is an
    argument error found before any CUDA call."""
    lib = _lib.load()
    same_rows = (ctypes.c_int * 20)(0, 128, 0, 1, 0, 128, 0, 0, 0, 0,
                                    0, 128, 0, 1, 128, 128, 128, 0, 0, 0)
    for dtype, mode in ((_lib.AFA_F32, _lib.AFA_HOP_ACCUMULATE), (_lib.AFA_BF16, _lib.AFA_HOP_STORE),
                        (_lib.AFA_BF16, _lib.AFA_HOP_FINALIZE)):
        rc = lib.afa_fwd_hop(1, 1, 1, 1, 1, 1, None, 1, 1, 128, 256, 128, dtype, same_rows, 2, 0, mode, 0.5, None)
        assert rc == _lib.AFA_ERR_INVALID and b"overlapping" in lib.afa_last_error()
    # Accepted by the argument checks (the launch itself then needs a GPU).
    rc = lib.afa_fwd_hop(1, 1, 1, 1, 1, None, None, 1, 1, 128, 256, 128, _lib.AFA_BF16, same_rows, 2, 0,
                         _lib.AFA_HOP_ACCUMULATE, 0.5, None)
    assert b"overlapping" not in lib.afa_last_error()


def test_decode_workspace_query():
    lib = _lib.load()
    # batch 64 x 32 heads already fills the GPU: no split, no workspace
    assert lib.afa_decode_workspace_bytes(64, 32, 8192, 128) == 0
    # one head over a long cache splits the keys and needs (D+1) floats per split
    n = lib.afa_decode_workspace_bytes(1, 1, 65536, 128)
    assert n > 0 and n % (129 * 4) == 0
    assert lib.afa_decode_workspace_bytes(0, 1, 1, 1) == 0


def test_ring_exchange_argument_checks():
    """The ring exchange entry points reject null pointers before any CUDA
    call; a zero-byte pull is a no-op."""
    import ctypes
    lib = _lib.load()
    handle = (ctypes.c_ubyte * 64)()
    off = ctypes.c_ulonglong(0)
    base = ctypes.c_void_p()
    assert lib.afa_ring_export(None, handle, ctypes.byref(off)) == _lib.AFA_ERR_INVALID
    assert b"afa_ring_export" in lib.afa_last_error()
    assert lib.afa_ring_open(None, ctypes.byref(base)) == _lib.AFA_ERR_INVALID
    assert lib.afa_ring_open(handle, None) == _lib.AFA_ERR_INVALID
    assert lib.afa_ring_close(None) == _lib.AFA_ERR_INVALID
    assert lib.afa_ring_pull(None, 1, 16, None) == _lib.AFA_ERR_INVALID
    assert b"afa_ring_pull" in lib.afa_last_error()
    assert lib.afa_ring_pull(None, None, 0, None) == _lib.AFA_OK
    assert lib.afa_ring_pull2d(None, 64, 1, 32, 16, 2, None) == _lib.AFA_ERR_INVALID
    assert b"afa_ring_pull2d" in lib.afa_last_error()
    assert lib.afa_ring_pull2d(1, 8, 1, 32, 16, 2, None) == _lib.AFA_ERR_INVALID
    assert b"pitch" in lib.afa_last_error()
    assert lib.afa_ring_pull2d(None, 0, None, 0, 0, 0, None) == _lib.AFA_OK


def test_backward_argument_checks():
    """afa_bwd validates before any CUDA call: dtype, null pointers, shapes,
    and the workspace size it asks for through afa_bwd_workspace_bytes."""
    lib = _lib.load()
    ptrs = [1] * 9
    assert lib.afa_bwd_workspace_bytes(2, 3, 100, 64, _lib.AFA_F32) == 2 * 3 * 100 * 4
    assert lib.afa_bwd_workspace_bytes(2, 3, 100, 64, _lib.AFA_F64) == 2 * 3 * 100 * 8
    assert lib.afa_bwd(*ptrs, 1, 1, 64, 64, _lib.AFA_F16, 0.5, 0, 0, 1, 1 << 20, None) == _lib.AFA_ERR_DTYPE
    assert lib.afa_bwd(None, *ptrs[1:], 1, 1, 64, 64, _lib.AFA_BF16, 0.5, 0, 0, 1, 1 << 20,
                       None) == _lib.AFA_ERR_INVALID
    assert lib.afa_bwd(*ptrs, 1, 1, 64, 512, _lib.AFA_BF16, 0.5, 0, 0, 1, 1 << 20, None) == _lib.AFA_ERR_INVALID
    assert lib.afa_bwd(*ptrs, 1, 1, 64, 64, _lib.AFA_BF16, 0.5, 0, 65, 1, 1 << 20, None) == _lib.AFA_ERR_INVALID
    for bad_sink in (-1.0, float("inf"), float("nan")):
        assert lib.afa_bwd(*ptrs, 1, 1, 64, 64, _lib.AFA_BF16, bad_sink, 0, 0, 1, 1 << 20,
                           None) == _lib.AFA_ERR_INVALID
        assert b"sink_omega" in lib.afa_last_error()
    assert lib.afa_bwd(*ptrs, 1, 1, 64, 64, _lib.AFA_BF16, 0.5, 0, 0, 1, 16, None) == _lib.AFA_ERR_INVALID
    assert b"workspace" in lib.afa_last_error()


def test_ago_argument_checks():
    lib = _lib.load()
    assert lib.afa_ago_table(1, 1, 7, 16, None, 10000.0, _lib.AFA_F32, None) == _lib.AFA_ERR_INVALID
    assert b"even" in lib.afa_last_error()
    assert lib.afa_ago_table(1, 1, 8, 0, None, 10000.0, _lib.AFA_F32, None) == _lib.AFA_ERR_INVALID
    assert lib.afa_ago_table(1, 1, 1026, 4, None, 10000.0, _lib.AFA_F32, None) == _lib.AFA_ERR_INVALID
    assert lib.afa_ago_table(None, 1, 8, 4, None, 10000.0, _lib.AFA_F32, None) == _lib.AFA_ERR_INVALID
    assert lib.afa_ago_table(1, 1, 8, 4, None, -1.0, _lib.AFA_F32, None) == _lib.AFA_ERR_INVALID
    assert lib.afa_ago_table(1, 1, 8, 4, None, 10000.0, _lib.AFA_F16, None) == _lib.AFA_ERR_DTYPE
    assert lib.afa_ago_rotate(None, 1, 1, 1, 1, 1, _lib.AFA_F32, 4, 8, 4, 1, _lib.AFA_F32, None) == _lib.AFA_ERR_INVALID
    assert lib.afa_ago_rotate(1, 1, 1, 1, 1, 1, _lib.AFA_F32, 4, 7, 4, 1, _lib.AFA_F32, None) == _lib.AFA_ERR_INVALID
    assert lib.afa_ago_rotate(1, 1, 1, 1, 1, 1, _lib.AFA_F32, 0, 8, 4, 1, _lib.AFA_F32, None) == _lib.AFA_OK
