"""The C ABI library loads and exports every entry point include/lca.h declares; argument
validation that happens before any device work behaves as documented (no GPU needed)."""
import ctypes
import os
import re

import pytest

from long_context_attention import _native

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    hdr = open(os.path.join(REPO, "include", "lca.h")).read()
    return re.findall(r"LCA_API\s+[\w\s\*]+?\b(lca_\w+)\s*\(", hdr)


def test_library_exports_every_declared_symbol():
    names = declared_functions()
    assert "lca_swa_forward" in names and len(names) >= 7
    lib = ctypes.CDLL(_native.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_abi_version_and_status_strings():
    c = _native.cabi()
    assert c.lib.lca_abi_version() == 2
    for code in range(7):
        assert c.lib.lca_status_string(code)
    assert c.lib.lca_status_string(99) == b"unknown status"


def _fwd(c, **kw):
    args = dict(q_ptr=None, k_ptr=None, v_ptr=None, o_ptr=None, lse_ptr=None, dtype=c.DTYPE_BF16, batch=1,
                heads=1, seq_len=128, head_dim=64, window=4, scale=0.125, tokens=[], ws_ptr=None, ws_bytes=0,
                stream_ptr=None)
    args.update(kw)
    return c.forward(**args)


def test_forward_validation_before_device_work():
    c = _native.cabi()
    assert _fwd(c, dtype=7) == c.ERR_UNSUPPORTED
    assert _fwd(c, head_dim=96) == c.ERR_UNSUPPORTED
    assert _fwd(c, window=-1) == c.ERR_INVALID_ARGUMENT
    assert _fwd(c, tokens=[128]) == c.ERR_INDEX
    assert _fwd(c, tokens=[-129]) == c.ERR_INDEX
    # empty problems succeed without touching a device
    assert _fwd(c, batch=0) == c.OK
    assert _fwd(c, seq_len=0) == c.OK
    # a NULL tensor pointer is rejected before any launch
    assert _fwd(c) == c.ERR_INVALID_ARGUMENT
    assert "non-NULL" in c.last_error()


def test_typed_forward_validation_before_device_work():
    c = _native.cabi()

    def typed(out_dtype, **kw):
        args = dict(q_ptr=None, k_ptr=None, v_ptr=None, o_ptr=None, out_dtype=out_dtype, lse_ptr=None,
                    dtype=c.DTYPE_BF16, batch=1, heads=1, seq_len=128, head_dim=64, window=4, scale=0.125, flags=0,
                    tokens=[], ws_ptr=None, ws_bytes=0, stream_ptr=None)
        args.update(kw)
        return c.forward_ex(**args)

    assert typed(7) == c.ERR_UNSUPPORTED
    assert "out_dtype" in c.last_error()
    assert typed(c.DTYPE_F32, flags=4) == c.ERR_INVALID_ARGUMENT
    assert "flags" in c.last_error()
    for dt in (c.DTYPE_F32, c.DTYPE_F16, c.DTYPE_BF16):
        for flags in (0, c.FLAG_CAUSAL, c.FLAG_TOKEN_MAJOR, c.FLAG_CAUSAL | c.FLAG_TOKEN_MAJOR):
            assert typed(dt, batch=0, flags=flags) == c.OK
            assert typed(dt, flags=flags) == c.ERR_INVALID_ARGUMENT  # NULL tensors, before any launch


def test_head_window_validation_before_device_work():
    c = _native.cabi()

    def ex(head_windows, heads):
        return c.forward_ex(None, None, None, None, c.DTYPE_F32, None, c.DTYPE_BF16, 1, heads, 128, 64, 4, 0.125, 0,
                            [], None, 0, None, head_windows=head_windows)

    assert ex([3, -1], 2) == c.ERR_INVALID_ARGUMENT
    assert "head_window_sizes[1]" in c.last_error()
    assert ex([1] * 257, 257) == c.ERR_UNSUPPORTED
    assert ex([1, 2], 2) == c.ERR_INVALID_ARGUMENT  # NULL tensors, after the radii checked out


def test_varlen_and_dilated_validation_before_device_work():
    import ctypes
    c = _native.cabi()
    i64 = ctypes.c_int64

    def varlen(cu, tokens=()):
        arr = (i64 * len(cu))(*cu)
        tok = (i64 * max(len(tokens), 1))(*tokens)
        return c.lib.lca_swa_forward_varlen(None, None, None, None, c.DTYPE_F32, None, c.DTYPE_BF16, 1, cu[-1], 64, 8,
                                            None, ctypes.c_float(0.1), 0, arr, len(cu) - 1, tok, len(tokens), None, 0,
                                            None)

    assert varlen([0, 10, 5]) == c.ERR_INVALID_ARGUMENT  # decreasing
    assert varlen([1, 10]) == c.ERR_INVALID_ARGUMENT     # not from 0
    assert varlen(list(range(0, 514))) == c.ERR_UNSUPPORTED  # 513 sequences
    assert varlen([0, 100, 150], [60]) == c.ERR_INDEX    # index 60 is outside the second sequence
    assert varlen([0, 100, 150], [40, -50]) == c.ERR_INVALID_ARGUMENT  # valid tokens, NULL tensors

    def dilated(n, dil, flags=0):
        return c.lib.lca_swa_forward_dilated(None, None, None, None, c.DTYPE_F32, None, c.DTYPE_BF16, 1, 1, n, 64, 8,
                                             None, dil, ctypes.c_float(0.1), flags, None, 0, None, 0, None)

    assert dilated(100, 0) == c.ERR_INVALID_ARGUMENT
    assert dilated(100, 3) == c.ERR_UNSUPPORTED          # not a multiple
    assert dilated(99, 3, c.FLAG_CAUSAL) == c.ERR_UNSUPPORTED
    assert dilated(99, 3, c.FLAG_TOKEN_MAJOR) == c.ERR_UNSUPPORTED
    assert dilated(99, 3) == c.ERR_INVALID_ARGUMENT      # NULL tensors
    size = ctypes.c_size_t(0)
    assert c.lib.lca_swa_dilated_workspace_size(1, 2, 96, 64, 8, 3, 0, c.DTYPE_BF16, c.DTYPE_F32,
                                                ctypes.byref(size)) == c.OK
    base = c.workspace_size(1, 2, 96, 64, 8, 0, c.DTYPE_BF16)[1]
    assert size.value >= base + 3 * 2 * 96 * 64 * 2 + 2 * 96 * 64 * 4


def _bwd(c, **kw):
    args = dict(q_ptr=None, k_ptr=None, v_ptr=None, o_ptr=None, lse_ptr=None, dout_ptr=None, dq_ptr=None,
                dk_ptr=None, dv_ptr=None, dtype=c.DTYPE_BF16, batch=1, heads=1, seq_len=128, head_dim=64, window=4,
                scale=0.125, tokens=[], ws_ptr=None, ws_bytes=0, stream_ptr=None)
    args.update(kw)
    return c.backward(**args)


def test_backward_validation_before_device_work():
    c = _native.cabi()
    assert _bwd(c, dtype=7) == c.ERR_UNSUPPORTED
    assert _bwd(c, head_dim=96) == c.ERR_UNSUPPORTED
    assert _bwd(c, window=-1) == c.ERR_INVALID_ARGUMENT
    assert _bwd(c, tokens=[128]) == c.ERR_INDEX
    assert _bwd(c, batch=0) == c.OK
    assert _bwd(c, seq_len=0) == c.OK
    assert _bwd(c) == c.ERR_INVALID_ARGUMENT
    assert "non-NULL" in c.last_error()


def test_backward_workspace_size():
    c = _native.cabi()
    st, none = c.backward_workspace_size(1, 2, 1000, 64, 16, 0, c.DTYPE_BF16)
    assert st == c.OK
    # at least the 16-bit dO and the two per-row statistics
    assert none >= 2 * 1000 * 64 * 2 + 2 * 2 * 1000 * 4
    st, some = c.backward_workspace_size(1, 2, 1000, 64, 16, 3, c.DTYPE_BF16)
    assert st == c.OK and some > none  # compact global rows and split partials
    assert c.backward_workspace_size(1, 2, 1000, 96, 16, 3, c.DTYPE_BF16)[0] == c.ERR_UNSUPPORTED
    assert c.backward_workspace_size(1, 2, 1000, 64, -1, 3, c.DTYPE_BF16)[0] == c.ERR_INVALID_ARGUMENT
