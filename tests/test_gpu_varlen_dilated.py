"""Packed variable-length sequences (`sliding_window_attention_varlen`,
lca_swa_forward_varlen) and the dilated window (`dilation=`, lca_swa_forward_dilated),
against the oracle on every row: sequences of length 0, 1 and not a multiple of the tile,
global tokens indexed within each sequence, causal; dilations 2-4 with global tokens,
radii per head and the 16-bit output."""
import pytest
import torch

import long_context_attention as lca
from long_context_attention import _native
from long_context_attention.workloads import make_inputs
from lca_testutil import LSE_ABS_TOL, assert_parity, max_abs, to_np
from oracle import swa_oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d,lens,w,g,causal", [
    (64, [300, 1, 0, 700, 129], 64, [0, -1], False),
    (128, [256, 513, 40], 100, [5, 0], False),
    (64, [1000, 64, 333], 128, [0, 2], True),
    (64, [400, 400], 1000, [], False),
])
def test_varlen_matches_oracle(dtype, d, lens, w, g, causal):
    cu = [0]
    for x in lens:
        cu.append(cu[-1] + x)
    H = 2
    q, k, v = make_inputs(900 + cu[-1] + d, 1, H, cu[-1], d, dtype)
    out, lse = lca.sliding_window_attention_varlen(q.cuda(), k.cuda(), v.cuda(), cu, w, g, 0.1, causal=causal,
                                                    return_lse=True)
    want, want_lse = swa_oracle.sliding_window_attention_varlen(q.float().numpy(), k.float().numpy(),
                                                                v.float().numpy(), cu, w, g, 0.1, causal=causal)
    assert_parity(to_np(out), want, f"varlen {lens} w={w} d={d} causal={causal} {dtype}")
    assert max_abs(to_np(lse), want_lse) <= LSE_ABS_TOL
    assert lca.device_error() == 0


def test_varlen_one_sequence_is_the_plain_forward_and_bad_tokens_raise():
    q, k, v = (t.cuda() for t in make_inputs(21, 1, 2, 500, 64, torch.bfloat16))
    a = lca.sliding_window_attention(q, k, v, 50, [3, 499], 0.125)
    b = lca.sliding_window_attention_varlen(q, k, v, [0, 500], 50, [3, 499], 0.125)
    assert torch.equal(a, b)
    with pytest.raises(IndexError):  # index 300 is outside the second sequence (length 200)
        lca.sliding_window_attention_varlen(q, k, v, [0, 300, 500], 50, [299], 0.125)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d,n,w,dil,g", [
    (64, 1024, 64, 2, [0, 511, 1023]),
    (128, 768, 40, 3, [7]),
    (64, 2048, 128, 4, [0, 1, 2, 3, 1000]),
    (64, 600, 1000, 2, []),
])
def test_dilated_matches_oracle(dtype, d, n, w, dil, g):
    q, k, v = make_inputs(1100 + n + dil, 1, 2, n, d, dtype)
    out, lse = lca.sliding_window_attention_with_lse(q.cuda(), k.cuda(), v.cuda(), w, g, 0.1, dilation=dil)
    want, want_lse = swa_oracle.sliding_window_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                                         w, g, 0.1, dilation=dil)
    assert_parity(to_np(out), want, f"dilated n={n} w={w} dil={dil} d={d} {dtype}")
    assert max_abs(to_np(lse), want_lse) <= LSE_ABS_TOL
    assert lca.device_error() == 0


def test_dilated_head_windows_16bit_output_and_dense_definition():
    q, k, v = (t.cuda() for t in make_inputs(31, 1, 2, 512, 64, torch.bfloat16))
    o32 = lca.sliding_window_attention(q, k, v, [16, 64], [9], 0.125, dilation=2)
    o16 = lca.sliding_window_attention(q, k, v, [16, 64], [9], 0.125, dilation=2, out_dtype=torch.bfloat16)
    assert torch.equal(o16, o32.to(torch.bfloat16))
    dense = lca.sliding_window_attention(q, k, v, [16, 64], [9], 0.125, dilation=2, force_reference=True)
    assert_parity(to_np(o32), to_np(dense), "dilated kernel vs dense definition")
    with pytest.raises(RuntimeError, match="multiple"):
        lca.sliding_window_attention(q[:, :, :511].contiguous(), k[:, :, :511].contiguous(),
                                     v[:, :, :511].contiguous(), 16, [], 0.125, dilation=2)


def test_dilated_through_c_abi():
    cabi = _native.cabi()
    B, H, n, d, w, dil, g = 1, 2, 384, 64, 20, 3, [4]
    q, k, v = (t.cuda() for t in make_inputs(41, B, H, n, d, torch.float16))
    ref = lca.sliding_window_attention(q, k, v, w, g, 0.125, dilation=dil)
    import ctypes
    nbytes = ctypes.c_size_t(0)
    st = cabi.lib.lca_swa_dilated_workspace_size(B, H, n, d, w, dil, 1, cabi.DTYPE_F16, cabi.DTYPE_F32,
                                                 ctypes.byref(nbytes))
    assert st == cabi.OK
    ws = torch.empty(nbytes.value, device="cuda", dtype=torch.uint8)
    out = torch.empty(B, H, n, d, device="cuda", dtype=torch.float32)
    arr = (ctypes.c_int64 * 1)(*g)
    st = cabi.lib.lca_swa_forward_dilated(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), cabi.DTYPE_F32,
                                          None, cabi.DTYPE_F16, B, H, n, d, w, None, dil, ctypes.c_float(0.125), 0,
                                          arr, 1, ws.data_ptr(), nbytes.value,
                                          torch.cuda.current_stream().cuda_stream)
    assert st == cabi.OK, cabi.last_error()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
