"""GPU parity of the backward pass (lca_swa_backward, sliding_window_attention_backward and
autograd through sliding_window_attention) against the oracle's fp64 gradient of the same
16-bit inputs.

Tolerance: dO, P and the score gradient dS enter the tensor-core products rounded to the
inputs' 16-bit type (fp32 accumulation), so the gradients carry a relative error of about
that type's unit roundoff: measured rel-L2 3e-4 for fp16 (unit roundoff 2^-11 = 4.9e-4) and
2.4e-3 for bf16 (2^-8 = 3.9e-3) on every case below.  The bound is about 3x that: rel-L2
<= 1e-3 (fp16) and <= 8e-3 (bf16), per gradient, against the fp64 oracle.
"""
import numpy as np
import pytest
import torch

from lca_testutil import rel_l2
from oracle import swa_oracle

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 1e-3, torch.bfloat16: 8e-3}

CASES = [
    # (B, H, n, d, window, global tokens, dtype)
    (1, 2, 512, 64, 32, [0, 100, 300], torch.float16),
    (1, 1, 300, 64, 17, [5, -1, 5], torch.bfloat16),            # ragged n, duplicate, negative
    (2, 2, 1024, 128, 100, [0, 511, 512, 1023], torch.bfloat16),
    (1, 1, 256, 64, 0, [], torch.float16),                      # window 0, no globals
    (1, 1, 200, 128, 500, [3], torch.float16),                  # window >= n
    (1, 1, 640, 64, 40, list(range(0, 640, 4)), torch.bfloat16),  # G = 160: two global tiles
    (1, 2, 777, 128, 64, [776, 1, 400], torch.float16),         # ragged n, d = 128
    (1, 4, 4096, 64, 256, [0, 17, 2048, 4095], torch.bfloat16),
]


def _inputs(B, H, n, d, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    Q, K, V = (torch.randn(B, H, n, d, generator=g).to(dtype).cuda() for _ in range(3))
    dO = torch.randn(B, H, n, d, generator=g).cuda()
    return Q, K, V, dO


def _oracle(Q, K, V, dO, w, tokens, scale):
    args = [t.double().cpu().numpy() for t in (Q, K, V, dO)]
    return swa_oracle.sliding_window_attention_backward(*args, w, tokens, scale)


@pytest.mark.parametrize("B,H,n,d,w,tokens,dtype", CASES)
def test_backward_matches_oracle(B, H, n, d, w, tokens, dtype):
    import long_context_attention as lca
    Q, K, V, dO = _inputs(B, H, n, d, dtype, seed=n * 7 + d + H)
    scale = d ** -0.5
    O, LSE = lca.sliding_window_attention_with_lse(Q, K, V, w, tokens, scale)
    dq, dk, dv = lca.sliding_window_attention_backward(Q, K, V, O, LSE, dO, w, tokens, scale)
    torch.cuda.synchronize()
    assert lca.device_error() == 0
    want = _oracle(Q, K, V, dO, w, tokens, scale)
    for name, got, ref in zip(("dQ", "dK", "dV"), (dq, dk, dv), want):
        got = got.double().cpu().numpy()
        assert np.isfinite(got).all(), name
        if np.abs(ref).max() < 1e-9:
            # window 0 without globals: each row sees only itself, P = 1 and dS = dP - D = 0,
            # so dQ and dK are exactly zero; the kernel's are the 16-bit rounding of dP - D
            assert np.abs(got).max() < 2e-2, name
            continue
        err = rel_l2(got, ref)
        assert err <= TOL[dtype], f"{name}: rel-L2 {err:.2e}"


def test_backward_negative_and_zero_scale():
    import long_context_attention as lca
    Q, K, V, dO = _inputs(1, 1, 384, 64, torch.float16, seed=3)
    for scale in (-0.2, 0.0):
        O, LSE = lca.sliding_window_attention_with_lse(Q, K, V, 20, [7], scale)
        got = lca.sliding_window_attention_backward(Q, K, V, O, LSE, dO, 20, [7], scale)
        want = _oracle(Q, K, V, dO, 20, [7], scale)
        for g, r in zip(got, want):
            # with scale 0, dQ and dK are exactly zero in both
            if np.abs(r).max() == 0:
                assert float(g.abs().max()) == 0.0
            else:
                assert rel_l2(g.double().cpu().numpy(), r) <= TOL[torch.float16]


def test_autograd_through_sliding_window_attention():
    import long_context_attention as lca
    Q, K, V, dO = _inputs(1, 2, 640, 64, torch.bfloat16, seed=11)
    tokens = [0, 320]
    Qr, Kr, Vr = (t.clone().requires_grad_() for t in (Q, K, V))
    out = lca.sliding_window_attention(Qr, Kr, Vr, 48, tokens)
    out.backward(dO)
    O, LSE = lca.sliding_window_attention_with_lse(Q, K, V, 48, tokens)
    direct = lca.sliding_window_attention_backward(Q, K, V, O, LSE, dO, 48, tokens)
    for t, g in zip((Qr, Kr, Vr), direct):
        assert t.grad.dtype == torch.bfloat16
        assert torch.equal(t.grad, g.to(torch.bfloat16))
    # options outside the backward's coverage are refused while gradients are wanted
    with pytest.raises(NotImplementedError):
        lca.sliding_window_attention(Qr, Kr, Vr, 48, tokens, causal=True)


def test_backward_is_deterministic():
    import long_context_attention as lca
    Q, K, V, dO = _inputs(1, 2, 1024, 128, torch.bfloat16, seed=5)
    O, LSE = lca.sliding_window_attention_with_lse(Q, K, V, 128, [0, 600])
    a = lca.sliding_window_attention_backward(Q, K, V, O, LSE, dO, 128, [0, 600])
    b = lca.sliding_window_attention_backward(Q, K, V, O, LSE, dO, 128, [0, 600])
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_backward_through_the_c_abi():
    """The raw C entry point on a side stream, with a caller-sized workspace."""
    from long_context_attention._native import cabi
    import long_context_attention as lca
    c = cabi()
    Q, K, V, dO = _inputs(1, 1, 512, 64, torch.float16, seed=9)
    O, LSE = lca.sliding_window_attention_with_lse(Q, K, V, 30, [2, 300])
    st, nbytes = c.backward_workspace_size(1, 1, 512, 64, 30, 2, c.DTYPE_F16)
    assert st == c.OK
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    dq, dk, dv = (torch.empty_like(dO) for _ in range(3))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        st = c.backward(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), LSE.data_ptr(), dO.data_ptr(),
                        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), c.DTYPE_F16, 1, 1, 512, 64, 30, 0.125,
                        [2, 300], ws.data_ptr(), nbytes, s.cuda_stream)
    assert st == c.OK, c.last_error()
    s.synchronize()
    want = _oracle(Q, K, V, dO, 30, [2, 300], 0.125)
    for g, r in zip((dq, dk, dv), want):
        assert rel_l2(g.double().cpu().numpy(), r) <= TOL[torch.float16]
    # a workspace one byte short is refused
    assert c.backward(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), LSE.data_ptr(), dO.data_ptr(),
                      dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), c.DTYPE_F16, 1, 1, 512, 64, 30, 0.125,
                      [2, 300], ws.data_ptr(), nbytes - 1, None) == c.ERR_WORKSPACE


def test_backward_full_size_against_the_banded_oracle():
    """One head of the 64K bf16 problem the benchmark times (w = 256, 65 global tokens), every
    row of dQ, dK and dV against the banded fp64 oracle, with the tolerance of the small
    cases; the global tokens' rows (split partials summed by the reduce) are also checked on
    their own, since they are 0.1 % of the rows."""
    import long_context_attention as lca
    from long_context_attention.workloads import WORKLOADS
    wl = WORKLOADS["many_globals_64k"]
    Q, K, V = (t.cuda() for t in wl.inputs(heads_slice=slice(0, 1)))
    tokens = wl.global_tokens()
    dO = torch.randn(Q.shape, generator=torch.Generator().manual_seed(64)).cuda()
    O, LSE = lca.sliding_window_attention_with_lse(Q, K, V, wl.window, tokens, wl.scale)
    got = lca.sliding_window_attention_backward(Q, K, V, O, LSE, dO, wl.window, tokens, wl.scale)
    torch.cuda.synchronize()
    assert lca.device_error() == 0
    args = [t.double().cpu().numpy() for t in (Q, K, V, dO)]
    want = swa_oracle.sliding_window_attention_backward_banded(*args, wl.window, tokens, wl.scale)
    grows = np.asarray(sorted(set(tokens)))
    for name, g, ref in zip(("dQ", "dK", "dV"), got, want):
        g = g.double().cpu().numpy()
        assert np.isfinite(g).all(), name
        err = rel_l2(g, ref)
        assert err <= TOL[torch.bfloat16], f"{name}: rel-L2 {err:.2e}"
        err = rel_l2(g[:, :, grows], ref[:, :, grows])
        assert err <= TOL[torch.bfloat16], f"{name} (global rows): rel-L2 {err:.2e}"
