"""Loading of the native build: the torch extension ``long_context_attention_kernels``
(which links ``liblca_b200.so``) and a ctypes handle on the C ABI itself.

There is no fallback: if the native build is missing, every GPU entry point raises with
the command that builds it.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblca_b200.so")
BUILD_HINT = "build it with: python long-context-attention-kernels_b200/build_native.py"

_lock = threading.Lock()
_ext = None
_cabi = None


def extension():
    """The torch extension module (imported once); raises RuntimeError if unavailable."""
    global _ext
    if _ext is None:
        with _lock:
            if _ext is None:
                try:
                    import long_context_attention_kernels as mod  # noqa: PLC0415
                except ImportError as e:  # pragma: no cover - exercised only without a build
                    raise RuntimeError(
                        f"long_context_attention: native extension not available ({e}); {BUILD_HINT}"
                    ) from e
                _ext = mod
    return _ext


def native_error() -> int:
    return extension().device_error()


class ShardDesc(ctypes.Structure):
    """``lca_shard_desc`` of include/lca.h."""

    _fields_ = [("batch", ctypes.c_int64), ("heads", ctypes.c_int64), ("seq_len", ctypes.c_int64),
                ("head_dim", ctypes.c_int64), ("window_size", ctypes.c_int64), ("shard_offset", ctypes.c_int64),
                ("shard_len", ctypes.c_int64), ("world_size", ctypes.c_int64), ("rank", ctypes.c_int64),
                ("dtype", ctypes.c_int),
                ("scale", ctypes.c_float)]


class ShardLayout(ctypes.Structure):
    """``lca_shard_layout`` of include/lca.h."""

    _fields_ = [("total_bytes", ctypes.c_size_t), ("halo_rows", ctypes.c_int64),
                ("globals_offset", ctypes.c_size_t), ("globals_bytes", ctypes.c_size_t),
                ("globals_row_bytes", ctypes.c_size_t),
                ("halo_send_offset", ctypes.c_size_t), ("halo_recv_offset", ctypes.c_size_t),
                ("halo_side_bytes", ctypes.c_size_t), ("rowpart_offset", ctypes.c_size_t),
                ("rowpart_bytes", ctypes.c_size_t), ("rowpart_all_offset", ctypes.c_size_t)]


class CABI:
    """ctypes binding of include/lca.h (the same stub a non-Python caller would write)."""

    OK = 0
    ERR_INVALID_ARGUMENT = 1
    ERR_INDEX = 2
    ERR_UNSUPPORTED = 3
    ERR_WORKSPACE = 4
    ERR_CUDA = 5
    ERR_DEVICE = 6
    DTYPE_F16 = 0
    DTYPE_BF16 = 1
    DTYPE_F32 = 2
    FLAG_CAUSAL = 1
    FLAG_TOKEN_MAJOR = 2

    def __init__(self, path: str = LIB_PATH):
        if not os.path.exists(path):
            raise RuntimeError(f"long_context_attention: {path} not found; {BUILD_HINT}")
        lib = ctypes.CDLL(path)
        i64, vp, sz = ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t
        lib.lca_abi_version.restype = ctypes.c_int
        lib.lca_abi_version.argtypes = []
        lib.lca_status_string.restype = ctypes.c_char_p
        lib.lca_status_string.argtypes = [ctypes.c_int]
        lib.lca_last_error.restype = ctypes.c_char_p
        lib.lca_last_error.argtypes = []
        lib.lca_normalize_global_tokens.restype = ctypes.c_int
        lib.lca_normalize_global_tokens.argtypes = [ctypes.POINTER(i64), i64, i64, ctypes.POINTER(ctypes.c_int32),
                                                    ctypes.POINTER(i64)]
        lib.lca_swa_workspace_size.restype = ctypes.c_int
        lib.lca_swa_workspace_size.argtypes = [i64, i64, i64, i64, i64, i64, ctypes.c_int, ctypes.POINTER(sz)]
        lib.lca_swa_forward.restype = ctypes.c_int
        lib.lca_swa_forward.argtypes = [vp, vp, vp, vp, vp, ctypes.c_int, i64, i64, i64, i64, i64, ctypes.c_float,
                                        ctypes.POINTER(i64), i64, vp, sz, vp]
        lib.lca_swa_forward_ex.restype = ctypes.c_int
        lib.lca_swa_forward_ex.argtypes = [vp, vp, vp, vp, ctypes.c_int, vp, ctypes.c_int, i64, i64, i64, i64, i64,
                                           ctypes.POINTER(i64), ctypes.c_float, ctypes.c_int, ctypes.POINTER(i64), i64,
                                           vp, sz, vp]
        lib.lca_swa_forward_varlen.restype = ctypes.c_int
        lib.lca_swa_forward_varlen.argtypes = [vp, vp, vp, vp, ctypes.c_int, vp, ctypes.c_int, i64, i64, i64, i64,
                                               ctypes.POINTER(i64), ctypes.c_float, ctypes.c_int, ctypes.POINTER(i64),
                                               i64, ctypes.POINTER(i64), i64, vp, sz, vp]
        lib.lca_swa_dilated_workspace_size.restype = ctypes.c_int
        lib.lca_swa_dilated_workspace_size.argtypes = [i64, i64, i64, i64, i64, i64, i64, ctypes.c_int, ctypes.c_int,
                                                       ctypes.POINTER(sz)]
        lib.lca_swa_forward_dilated.restype = ctypes.c_int
        lib.lca_swa_forward_dilated.argtypes = [vp, vp, vp, vp, ctypes.c_int, vp, ctypes.c_int, i64, i64, i64, i64,
                                                i64, ctypes.POINTER(i64), i64, ctypes.c_float, ctypes.c_int,
                                                ctypes.POINTER(i64), i64, vp, sz, vp]
        lib.lca_swa_forward_noalloc.restype = ctypes.c_int
        lib.lca_swa_forward_noalloc.argtypes = [vp, vp, vp, vp, vp, ctypes.c_int, i64, i64, i64, i64, i64,
                                                ctypes.c_float, ctypes.POINTER(i64), i64, vp]
        lib.lca_swa_backward_workspace_size.restype = ctypes.c_int
        lib.lca_swa_backward_workspace_size.argtypes = [i64, i64, i64, i64, i64, i64, ctypes.c_int, ctypes.POINTER(sz)]
        lib.lca_swa_backward.restype = ctypes.c_int
        lib.lca_swa_backward.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, ctypes.c_int, i64, i64, i64, i64, i64,
                                         ctypes.c_float, ctypes.POINTER(i64), i64, vp, sz, vp]
        dp, lp = ctypes.POINTER(ShardDesc), ctypes.POINTER(ShardLayout)
        lib.lca_swa_shard_layout.restype = ctypes.c_int
        lib.lca_swa_shard_layout.argtypes = [dp, i64, lp]
        lib.lca_swa_shard_prepare.restype = ctypes.c_int
        lib.lca_swa_shard_prepare.argtypes = [dp, vp, vp, vp, ctypes.POINTER(i64), i64, vp, sz, vp]
        lib.lca_swa_shard_forward.restype = ctypes.c_int
        lib.lca_swa_shard_forward.argtypes = [dp, vp, vp, vp, vp, vp, ctypes.POINTER(i64), i64, vp, sz, vp]
        lib.lca_swa_shard_finish.restype = ctypes.c_int
        lib.lca_swa_shard_finish.argtypes = [dp, vp, vp, ctypes.POINTER(i64), i64, vp, sz, vp]
        lib.lca_peer_alloc.restype = ctypes.c_int
        lib.lca_peer_alloc.argtypes = [sz, ctypes.POINTER(vp), vp]
        lib.lca_peer_open.restype = ctypes.c_int
        lib.lca_peer_open.argtypes = [vp, ctypes.POINTER(vp)]
        lib.lca_peer_close.restype = ctypes.c_int
        lib.lca_peer_close.argtypes = [vp]
        lib.lca_peer_free.restype = ctypes.c_int
        lib.lca_peer_free.argtypes = [vp]
        pp = ctypes.POINTER(vp)
        lib.lca_swa_shard_exchange_peer.restype = ctypes.c_int
        lib.lca_swa_shard_exchange_peer.argtypes = [dp, ctypes.POINTER(i64), i64, pp, sz, vp]
        lib.lca_swa_shard_finish_peer.restype = ctypes.c_int
        lib.lca_swa_shard_finish_peer.argtypes = [dp, vp, vp, ctypes.POINTER(i64), i64, pp, sz, vp]
        lib.lca_set_timing_events.restype = ctypes.c_int
        lib.lca_set_timing_events.argtypes = [vp, vp]
        lib.lca_device_error.restype = ctypes.c_int
        lib.lca_device_error.argtypes = [ctypes.POINTER(ctypes.c_int)]
        self.lib = lib

    def last_error(self) -> str:
        return self.lib.lca_last_error().decode()

    def normalize(self, tokens, seq_len: int):
        n = len(tokens)
        arr = (ctypes.c_int64 * max(n, 1))(*tokens)
        out = (ctypes.c_int32 * max(n, 1))()
        cnt = ctypes.c_int64(0)
        st = self.lib.lca_normalize_global_tokens(arr, n, seq_len, out, ctypes.byref(cnt))
        return st, [out[i] for i in range(cnt.value)]

    def workspace_size(self, batch, heads, seq_len, head_dim, window, num_unique_global, dtype) -> tuple[int, int]:
        out = ctypes.c_size_t(0)
        st = self.lib.lca_swa_workspace_size(batch, heads, seq_len, head_dim, window, num_unique_global, dtype,
                                             ctypes.byref(out))
        return st, out.value

    def forward(self, q_ptr, k_ptr, v_ptr, o_ptr, lse_ptr, dtype, batch, heads, seq_len, head_dim, window, scale,
                tokens, ws_ptr, ws_bytes, stream_ptr) -> int:
        n = len(tokens)
        arr = (ctypes.c_int64 * max(n, 1))(*tokens)
        return self.lib.lca_swa_forward(q_ptr, k_ptr, v_ptr, o_ptr, lse_ptr, dtype, batch, heads, seq_len, head_dim,
                                        window, ctypes.c_float(scale), arr, n, ws_ptr, ws_bytes, stream_ptr)

    def forward_ex(self, q_ptr, k_ptr, v_ptr, o_ptr, out_dtype, lse_ptr, dtype, batch, heads, seq_len, head_dim,
                   window, scale, flags, tokens, ws_ptr, ws_bytes, stream_ptr, head_windows=None) -> int:
        n = len(tokens)
        arr = (ctypes.c_int64 * max(n, 1))(*tokens)
        hw = None if head_windows is None else (ctypes.c_int64 * max(len(head_windows), 1))(*head_windows)
        return self.lib.lca_swa_forward_ex(q_ptr, k_ptr, v_ptr, o_ptr, out_dtype, lse_ptr, dtype, batch, heads,
                                           seq_len, head_dim, window, hw, ctypes.c_float(scale), flags, arr, n,
                                           ws_ptr, ws_bytes, stream_ptr)

    def forward_noalloc(self, q_ptr, k_ptr, v_ptr, o_ptr, lse_ptr, dtype, batch, heads, seq_len, head_dim, window,
                        scale, tokens, stream_ptr) -> int:
        n = len(tokens)
        arr = (ctypes.c_int64 * max(n, 1))(*tokens)
        return self.lib.lca_swa_forward_noalloc(q_ptr, k_ptr, v_ptr, o_ptr, lse_ptr, dtype, batch, heads, seq_len,
                                                head_dim, window, ctypes.c_float(scale), arr, n, stream_ptr)

    def backward_workspace_size(self, batch, heads, seq_len, head_dim, window, num_unique_global,
                                dtype) -> tuple[int, int]:
        out = ctypes.c_size_t(0)
        st = self.lib.lca_swa_backward_workspace_size(batch, heads, seq_len, head_dim, window, num_unique_global,
                                                      dtype, ctypes.byref(out))
        return st, out.value

    def backward(self, q_ptr, k_ptr, v_ptr, o_ptr, lse_ptr, dout_ptr, dq_ptr, dk_ptr, dv_ptr, dtype, batch, heads,
                 seq_len, head_dim, window, scale, tokens, ws_ptr, ws_bytes, stream_ptr) -> int:
        arr, n = self._tokens(tokens)
        return self.lib.lca_swa_backward(q_ptr, k_ptr, v_ptr, o_ptr, lse_ptr, dout_ptr, dq_ptr, dk_ptr, dv_ptr, dtype,
                                         batch, heads, seq_len, head_dim, window, ctypes.c_float(scale), arr, n,
                                         ws_ptr, ws_bytes, stream_ptr)

    @staticmethod
    def _tokens(tokens):
        n = len(tokens)
        return (ctypes.c_int64 * max(n, 1))(*tokens), n

    def shard_layout(self, desc: ShardDesc, num_unique_global: int) -> tuple[int, ShardLayout]:
        out = ShardLayout()
        st = self.lib.lca_swa_shard_layout(ctypes.byref(desc), num_unique_global, ctypes.byref(out))
        return st, out

    def shard_prepare(self, desc: ShardDesc, q_ptr, k_ptr, v_ptr, tokens, ws_ptr, ws_bytes, stream_ptr) -> int:
        arr, n = self._tokens(tokens)
        return self.lib.lca_swa_shard_prepare(ctypes.byref(desc), q_ptr, k_ptr, v_ptr, arr, n, ws_ptr, ws_bytes,
                                              stream_ptr)

    def shard_forward(self, desc: ShardDesc, q_ptr, k_ptr, v_ptr, o_ptr, lse_ptr, tokens, ws_ptr, ws_bytes,
                      stream_ptr) -> int:
        arr, n = self._tokens(tokens)
        return self.lib.lca_swa_shard_forward(ctypes.byref(desc), q_ptr, k_ptr, v_ptr, o_ptr, lse_ptr, arr, n, ws_ptr,
                                              ws_bytes, stream_ptr)

    def shard_finish(self, desc: ShardDesc, o_ptr, lse_ptr, tokens, ws_ptr, ws_bytes, stream_ptr) -> int:
        arr, n = self._tokens(tokens)
        return self.lib.lca_swa_shard_finish(ctypes.byref(desc), o_ptr, lse_ptr, arr, n, ws_ptr, ws_bytes, stream_ptr)


def cabi() -> CABI:
    global _cabi
    if _cabi is None:
        with _lock:
            if _cabi is None:
                _cabi = CABI()
    return _cabi
