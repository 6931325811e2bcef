"""16-bit output option (`out_dtype`): the kernels write the same fp32-accumulated result
rounded to fp16 or bf16.  Checked bit for bit against the fp32 output rounded by torch
(round to nearest even), and against the oracle within the parity bar plus the rounding
of the output type; the log-sum-exp is unchanged."""
import numpy as np
import pytest
import torch

import long_context_attention as lca
from long_context_attention import _native
from long_context_attention.workloads import make_inputs
from lca_testutil import LSE_ABS_TOL, MAX_ABS_TOL, max_abs, to_np
from oracle import swa_oracle

pytestmark = pytest.mark.gpu

# half an ulp of the output type, relative
ROUNDING = {torch.float16: 2.0 ** -11, torch.bfloat16: 2.0 ** -8}


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("in_dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d,n,w,g", [(64, 1000, 128, [0, 500, -1]), (128, 700, 300, [3, 699]), (64, 384, 5, []),
                                     (128, 129, 0, [128])])
def test_out_dtype_matches_rounded_fp32(out_dtype, in_dtype, d, n, w, g):
    q, k, v = (t.cuda() for t in make_inputs(300 + n + d, 1, 2, n, d, in_dtype))
    o32, l32 = lca.sliding_window_attention_with_lse(q, k, v, w, g, 0.1)
    o16, l16 = lca.sliding_window_attention_with_lse(q, k, v, w, g, 0.1, out_dtype=out_dtype)
    o16b = lca.sliding_window_attention(q, k, v, w, g, 0.1, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert o16.dtype == out_dtype and o16.shape == q.shape
    assert torch.equal(o16, o32.to(out_dtype)), "16-bit output differs from the rounded fp32 output"
    assert torch.equal(o16b, o16)
    assert torch.equal(l16, l32)
    want, want_lse = swa_oracle.sliding_window_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                                         v.float().cpu().numpy(), w, g, 0.1)
    got = to_np(o16)
    assert np.all(np.abs(got - want) <= MAX_ABS_TOL + ROUNDING[out_dtype] * np.abs(want))
    assert max_abs(to_np(l16), want_lse) <= LSE_ABS_TOL
    assert lca.device_error() == 0


def test_out_dtype_through_c_abi():
    """lca_swa_forward_ex with caller-owned buffers gives the same bits as the extension."""
    cabi = _native.cabi()
    B, H, n, d, w, g = 1, 3, 600, 64, 200, [7, 450]
    q, k, v = (t.cuda() for t in make_inputs(9, B, H, n, d, torch.bfloat16))
    ref = lca.sliding_window_attention(q, k, v, w, g, 0.125, out_dtype=torch.bfloat16)
    out = torch.empty(B, H, n, d, device="cuda", dtype=torch.bfloat16)
    st, gl = cabi.normalize(g, n)
    st, ws_bytes = cabi.workspace_size(B, H, n, d, w, len(gl), cabi.DTYPE_BF16)
    ws = torch.empty(max(ws_bytes, 1), device="cuda", dtype=torch.uint8)
    stream = torch.cuda.current_stream().cuda_stream
    st = cabi.forward_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), cabi.DTYPE_BF16, 0,
                         cabi.DTYPE_BF16, B, H, n, d, w, 0.125, 0, g, ws.data_ptr(), ws_bytes, stream)
    assert st == cabi.OK, cabi.last_error()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_out_dtype_rejected_values():
    q = torch.zeros(1, 1, 128, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="out_dtype"):
        lca.sliding_window_attention(q, q, q, 4, [], 0.1, out_dtype=torch.int32)
