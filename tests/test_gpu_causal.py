"""Causal (one-sided) variant, `causal=True` / LCA_FLAG_CAUSAL: the reference's mask
intersected with j <= i.  Checked against the oracle (`swa_oracle.sliding_window_attention(
..., causal=True)`) at the parity bar, on every row: band-only problems, global tokens at
both ends and inside bands, windows wider than the sequence, ragged lengths, both head
dims and input dtypes, and with the 16-bit output."""
import pytest
import torch

import long_context_attention as lca
from long_context_attention.workloads import make_inputs
from lca_testutil import LSE_ABS_TOL, assert_parity, max_abs, to_np
from oracle import swa_oracle

pytestmark = pytest.mark.gpu

CASES = [
    (64, 1000, 128, []),
    (64, 1000, 128, [0, 500, -1]),
    (128, 700, 300, [3, 699, 350]),
    (64, 384, 5, list(range(0, 384, 3))),
    (128, 129, 0, [128]),
    (64, 300, 1000, [7]),
    (64, 1, 0, []),
]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d,n,w,g", CASES)
def test_causal_matches_oracle(dtype, d, n, w, g):
    q, k, v = make_inputs(500 + n + d, 1, 2, n, d, dtype)
    out, lse = lca.sliding_window_attention_with_lse(q.cuda(), k.cuda(), v.cuda(), w, g, 0.1, causal=True)
    want, want_lse = swa_oracle.sliding_window_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                                         w, g, 0.1, causal=True)
    assert_parity(to_np(out), want, f"causal n={n} w={w} d={d} G={len(g)} {dtype}")
    assert max_abs(to_np(lse), want_lse) <= LSE_ABS_TOL
    assert lca.device_error() == 0


def test_causal_bf16_output_and_dense_definition():
    """The 16-bit output of the causal variant is its fp32 output rounded; the dense torch
    definition (force_reference=True) agrees with the kernel at the parity bar."""
    q, k, v = (t.cuda() for t in make_inputs(8, 1, 2, 512, 64, torch.bfloat16))
    o32 = lca.sliding_window_attention(q, k, v, 64, [1, 300], 0.125, causal=True)
    o16 = lca.sliding_window_attention(q, k, v, 64, [1, 300], 0.125, causal=True, out_dtype=torch.bfloat16)
    assert torch.equal(o16, o32.to(torch.bfloat16))
    dense = lca.sliding_window_attention(q, k, v, 64, [1, 300], 0.125, causal=True, force_reference=True)
    assert_parity(to_np(o32), to_np(dense), "causal kernel vs dense definition")


def test_causal_first_rows_see_only_their_past():
    """Row 0 sees only key 0, so its output is v[0] exactly (up to fp32 rounding)."""
    q, k, v = (t.cuda() for t in make_inputs(3, 1, 1, 256, 64, torch.float16))
    out = lca.sliding_window_attention(q, k, v, 32, [], 0.125, causal=True)
    assert torch.allclose(out[0, 0, 0], v[0, 0, 0].float(), atol=1e-6, rtol=0)
