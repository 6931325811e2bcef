"""Token-major tensors (`layout="bnhd"`, LCA_FLAG_TOKEN_MAJOR): Q, K, V and O as
[batch, seq_len, heads, head_dim], read and written in place.  The same computation as the
head-major call on the transposed tensors, so the results are compared bit for bit: band
and global rows (gather and merge with token-major strides), the fp16 copy of V for bf16
inputs, 16-bit output, causal, radii per head and packed sequences; one case also against
the oracle."""
import pytest
import torch

import long_context_attention as lca
from long_context_attention.workloads import make_inputs
from lca_testutil import LSE_ABS_TOL, assert_parity, max_abs, to_np
from oracle import swa_oracle

pytestmark = pytest.mark.gpu


def _bnhd(t):
    return t.transpose(1, 2).contiguous()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d,B,H,n,w,g,kw", [
    (64, 2, 3, 700, 64, [0, 350, -1], {}),
    (128, 1, 2, 513, 100, [5], {}),
    (64, 1, 4, 1024, 128, [1, 900], {"out_dtype": torch.bfloat16}),
    (64, 2, 2, 600, 50, [10, 599], {"causal": True}),
    (64, 1, 3, 400, [8, 64, 200], [3], {}),
])
def test_token_major_equals_head_major(dtype, d, B, H, n, w, g, kw):
    q, k, v = (t.cuda() for t in make_inputs(1300 + n + d, B, H, n, d, dtype))
    o_ref, l_ref = lca.sliding_window_attention_with_lse(q, k, v, w, g, 0.1, **kw)
    o_tm, l_tm = lca.sliding_window_attention_with_lse(_bnhd(q), _bnhd(k), _bnhd(v), w, g, 0.1, layout="bnhd", **kw)
    torch.cuda.synchronize()
    assert o_tm.shape == (B, n, H, d)
    assert torch.equal(o_tm, _bnhd(o_ref))
    assert torch.equal(l_tm, l_ref)
    assert lca.device_error() == 0


def test_token_major_against_oracle_and_varlen():
    q, k, v = make_inputs(77, 1, 2, 800, 64, torch.bfloat16)
    out = lca.sliding_window_attention(_bnhd(q).cuda(), _bnhd(k).cuda(), _bnhd(v).cuda(), 96, [0, 400], 0.125,
                                       layout="bnhd")
    want, _ = swa_oracle.sliding_window_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), 96,
                                                  [0, 400], 0.125)
    assert_parity(to_np(out.transpose(1, 2)), want, "token-major vs oracle")
    cu = [0, 300, 301, 800]
    a, la = lca.sliding_window_attention_varlen(q.cuda(), k.cuda(), v.cuda(), cu, 32, [0], 0.125, return_lse=True)
    b, lb = lca.sliding_window_attention_varlen(_bnhd(q).cuda(), _bnhd(k).cuda(), _bnhd(v).cuda(), cu, 32, [0], 0.125,
                                                return_lse=True, layout="bnhd")
    assert torch.equal(b, _bnhd(a)) and torch.equal(lb, la)
    dense = lca.sliding_window_attention(_bnhd(q).cuda(), _bnhd(k).cuda(), _bnhd(v).cuda(), 96, [0, 400], 0.125,
                                         layout="bnhd", force_reference=True)
    assert_parity(to_np(out), to_np(dense), "token-major kernel vs dense definition")
