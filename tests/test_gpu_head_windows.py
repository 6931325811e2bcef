"""A band radius per head (`window_size` given as one radius per head; the C ABI's
head_window_sizes): head h of every batch uses its own radius.  Checked against the
oracle, which takes the same per-head radii, on every row; with global tokens, causal,
both head dims and input dtypes, radii of 0 and radii beyond the sequence."""
import pytest
import torch

import long_context_attention as lca
from long_context_attention import _native
from long_context_attention.workloads import make_inputs
from lca_testutil import LSE_ABS_TOL, assert_parity, max_abs, to_np
from oracle import swa_oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d,n,radii,g,causal", [
    (64, 1000, [0, 32, 256, 2000], [0, 517, -1], False),
    (128, 700, [300, 5, 128], [3, 699], False),
    (64, 900, [64, 200, 1], [450], True),
    (128, 384, [1000, 0], [], True),
])
def test_head_windows_match_oracle(dtype, d, n, radii, g, causal):
    B, H = 2, len(radii)
    q, k, v = make_inputs(700 + n + d, B, H, n, d, dtype)
    out, lse = lca.sliding_window_attention_with_lse(q.cuda(), k.cuda(), v.cuda(), radii, g, 0.1, causal=causal)
    want, want_lse = swa_oracle.sliding_window_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                                         radii, g, 0.1, causal=causal)
    assert_parity(to_np(out), want, f"radii={radii} n={n} d={d} causal={causal} {dtype}")
    assert max_abs(to_np(lse), want_lse) <= LSE_ABS_TOL
    assert lca.device_error() == 0


def test_equal_head_windows_are_one_window_and_dense_definition_agrees():
    q, k, v = (t.cuda() for t in make_inputs(11, 1, 3, 512, 64, torch.bfloat16))
    a = lca.sliding_window_attention(q, k, v, 96, [5], 0.125)
    b = lca.sliding_window_attention(q, k, v, [96, 96, 96], [5], 0.125)
    assert torch.equal(a, b)
    c = lca.sliding_window_attention(q, k, v, [0, 96, 300], [5], 0.125)
    dense = lca.sliding_window_attention(q, k, v, [0, 96, 300], [5], 0.125, force_reference=True)
    assert_parity(to_np(c), to_np(dense), "per-head radii vs dense definition")


def test_head_windows_through_c_abi():
    cabi = _native.cabi()
    B, H, n, d, g = 1, 2, 400, 64, [9]
    q, k, v = (t.cuda() for t in make_inputs(12, B, H, n, d, torch.float16))
    ref = lca.sliding_window_attention(q, k, v, [17, 150], g, 0.125)
    out = torch.empty(B, H, n, d, device="cuda", dtype=torch.float32)
    st, ws_bytes = cabi.workspace_size(B, H, n, d, 150, 1, cabi.DTYPE_F16)
    ws = torch.empty(max(ws_bytes, 1), device="cuda", dtype=torch.uint8)
    stream = torch.cuda.current_stream().cuda_stream
    st = cabi.forward_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), cabi.DTYPE_F32, 0, cabi.DTYPE_F16,
                         B, H, n, d, 0, 0.125, 0, g, ws.data_ptr(), ws_bytes, stream, head_windows=[17, 150])
    assert st == cabi.OK, cabi.last_error()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
