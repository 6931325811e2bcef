"""The CPU oracle, pinned against outputs of the reference implementation itself
(tests/golden/*.npz, made by tests/golden/make_golden.py) and against the reference's
own known-answer tests (tests/test_correctness.py:26-62 of the reference)."""
import math

import numpy as np
import pytest
import torch

from lca_testutil import golden_names, load_golden, max_abs, rel_l2
from oracle import swa_oracle


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference_fixture(name):
    c = load_golden(name)
    out, lse = swa_oracle.sliding_window_attention(
        c["q"].float().numpy(), c["k"].float().numpy(), c["v"].float().numpy(), c["window"], c["globals"],
        c["scale"], rows=c["rows"])
    # the reference computes in fp32, the oracle in fp64: agreement to fp32 rounding
    assert max_abs(out, c["out"]) < 2e-6, name
    assert rel_l2(out, c["out"]) < 1e-6, name
    assert np.all(np.isfinite(lse))


def _full_attention(q, k, v, scale):
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * scale
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, v)


def test_unmasked_window_equals_full_attention():
    # reference tests/test_correctness.py:26-40
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, 2, 32, 16)) for _ in range(3))
    out, _ = swa_oracle.sliding_window_attention(q, k, v, 32, [], 1 / math.sqrt(16))
    np.testing.assert_allclose(out, _full_attention(q, k, v, 1 / math.sqrt(16)), atol=1e-12)


def test_global_row_gets_full_context():
    # reference tests/test_correctness.py:43-62
    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((1, 1, 64, 16)) for _ in range(3))
    out, _ = swa_oracle.sliding_window_attention(q, k, v, 1, [0], 0.25)
    full = _full_attention(q, k, v, 0.25)
    np.testing.assert_allclose(out[:, :, 0], full[:, :, 0], atol=1e-12)
    assert not np.allclose(out[:, :, 32], full[:, :, 32], atol=1e-3)


def test_duplicates_and_negative_indices():
    rng = np.random.default_rng(2)
    q, k, v = (rng.standard_normal((1, 1, 40, 8)) for _ in range(3))
    a, la = swa_oracle.sliding_window_attention(q, k, v, 3, [0, 0, 5], 0.3)
    b, lb = swa_oracle.sliding_window_attention(q, k, v, 3, [5, 0], 0.3)
    c, _ = swa_oracle.sliding_window_attention(q, k, v, 3, [-40, -35], 0.3)
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(la, lb)
    np.testing.assert_array_equal(a, c)


def test_out_of_range_index_raises():
    q = np.zeros((1, 1, 10, 4))
    with pytest.raises(IndexError):
        swa_oracle.sliding_window_attention(q, q, q, 1, [10], 1.0)
    with pytest.raises(IndexError):
        swa_oracle.sliding_window_attention(q, q, q, 1, [-11], 1.0)


def test_lse_matches_torch_logsumexp():
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, 2, 70, 8, generator=g, dtype=torch.float64) for _ in range(3))
    out, lse = swa_oracle.sliding_window_attention(q.numpy(), k.numpy(), v.numpy(), 5, [3, 60], 0.4)
    mask = torch.from_numpy(swa_oracle.visible_rows(np.arange(70), 70, 5, np.array([3, 60])))
    s = torch.einsum("bhqd,bhkd->bhqk", q, k) * 0.4
    s = s.masked_fill(~mask, float("-inf"))
    np.testing.assert_allclose(lse, torch.logsumexp(s, -1).numpy(), atol=1e-12)
    np.testing.assert_allclose(out, torch.einsum("bhqk,bhkd->bhqd", torch.softmax(s, -1), v).numpy(),
                               atol=1e-12)


def test_row_subset_equals_full():
    rng = np.random.default_rng(4)
    q, k, v = (rng.standard_normal((2, 1, 300, 16)).astype(np.float32) for _ in range(3))
    full, lf = swa_oracle.sliding_window_attention(q, k, v, 20, [7, 299], 0.25, block_rows=64)
    rows = [0, 7, 150, 299]
    sub, ls = swa_oracle.sliding_window_attention(q, k, v, 20, [7, 299], 0.25, rows=rows)
    np.testing.assert_allclose(sub, full[:, :, rows], atol=1e-12)
    np.testing.assert_allclose(ls, lf[:, :, rows], atol=1e-12)


def test_causal_oracle_is_the_dense_mask_with_the_upper_triangle_removed():
    """The oracle's causal option against the dense torch definition of the package
    (the reference's mask intersected with j <= i), on small shapes with global tokens."""
    import torch

    from long_context_attention import _dense_causal_attention
    for n, w, g in [(64, 4, [0, 63]), (100, 200, [5]), (37, 0, [-1, 10])]:
        gen = torch.Generator().manual_seed(n)
        q, k, v = (torch.randn(1, 2, n, 16, generator=gen) for _ in range(3))
        want = _dense_causal_attention(q, k, v, w, g, 0.3).numpy()
        got, lse = swa_oracle.sliding_window_attention(q.numpy(), k.numpy(), v.numpy(), w, g, 0.3, causal=True)
        assert np.abs(got - want).max() < 2e-6
        # every row keeps at least its own key
        assert np.isfinite(lse).all()



def test_dilated_and_varlen_oracle():
    """The oracle's dilated band against the package's dense torch definition, and its packed
    sequences against running each sequence alone."""
    import torch

    from long_context_attention import _dense_causal_attention
    gen = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, 2, 60, 8, generator=gen) for _ in range(3))
    for w, dil, g in [(3, 2, [0]), (5, 3, [7, 59]), (100, 4, [])]:
        want = _dense_causal_attention(q, k, v, w, g, 0.4, dilation=dil, causal=False).numpy()
        got, _ = swa_oracle.sliding_window_attention(q.numpy(), k.numpy(), v.numpy(), w, g, 0.4, dilation=dil)
        assert np.abs(got - want).max() < 2e-6
    cu = [0, 25, 25, 60]
    got, lse = swa_oracle.sliding_window_attention_varlen(q.numpy(), k.numpy(), v.numpy(), cu, 4, [0, -1], 0.4)
    for a, b in [(0, 25), (25, 60)]:
        want, want_lse = swa_oracle.sliding_window_attention(q[:, :, a:b].numpy(), k[:, :, a:b].numpy(),
                                                             v[:, :, a:b].numpy(), 4, [0, -1], 0.4)
        assert np.array_equal(got[:, :, a:b], want) and np.array_equal(lse[:, :, a:b], want_lse)


@pytest.mark.parametrize("B,H,n,d,w,g", [(1, 2, 37, 8, 3, [0, 5, -1]), (2, 1, 64, 16, 0, []),
                                         (1, 1, 50, 4, 100, [7, 7]), (1, 2, 130, 8, 9, [129, 0, 64])])
def test_backward_oracle_matches_autograd_of_the_reference_definition(B, H, n, d, w, g):
    """The oracle's backward is pinned to torch autograd through the reference's own dense
    definition (python/long_context_attention/__init__.py:24-53, restated under the same
    name in this package), which computes in fp32."""
    import long_context_attention as lca
    gen = torch.Generator().manual_seed(n * 31 + d)
    Q, K, V, dO = (torch.randn(B, H, n, d, generator=gen, dtype=torch.float64) for _ in range(4))
    Qr, Kr, Vr = (x.clone().requires_grad_() for x in (Q, K, V))
    out = lca._reference_sliding_window_attention(Qr, Kr, Vr, w, g, 0.3)
    want = torch.autograd.grad((out * dO).sum(), (Qr, Kr, Vr))
    got = swa_oracle.sliding_window_attention_backward(Q.numpy(), K.numpy(), V.numpy(), dO.numpy(), w, g, 0.3,
                                                       block_rows=16)
    for a, b in zip(got, want):
        assert max_abs(a, b.numpy()) < 2e-6


def test_backward_oracle_matches_finite_differences():
    """fp64 central differences of sum(O * dO) against the oracle's gradient."""
    rng = np.random.default_rng(5)
    B, H, n, d, w, g, scale = 1, 1, 12, 3, 2, [4], 0.7
    Q, K, V, dO = (rng.standard_normal((B, H, n, d)) for _ in range(4))
    dq, dk, dv = swa_oracle.sliding_window_attention_backward(Q, K, V, dO, w, g, scale)

    def loss(q, k, v):
        return float((swa_oracle.sliding_window_attention(q, k, v, w, g, scale)[0] * dO).sum())

    eps = 1e-6
    for which, grad in ((0, dq), (1, dk), (2, dv)):
        for idx in [(0, 0, 0, 0), (0, 0, 4, 1), (0, 0, 11, 2), (0, 0, 7, 0)]:
            args = [Q.copy(), K.copy(), V.copy()]
            args[which][idx] += eps
            up = loss(*args)
            args[which][idx] -= 2 * eps
            down = loss(*args)
            assert abs((up - down) / (2 * eps) - grad[idx]) < 1e-6


@pytest.mark.parametrize("B,H,n,d,w,g,block", [(1, 2, 37, 8, 3, [0, 5, -1], 8), (2, 1, 64, 16, 0, [], 16),
                                               (1, 1, 50, 4, 100, [7, 7], 16), (1, 2, 130, 8, 9, [129, 0, 64], 32),
                                               (1, 1, 300, 8, 20, list(range(0, 300, 3)), 64),
                                               (1, 1, 257, 4, 30, [256], 512)])
def test_banded_backward_oracle_matches_the_dense_one(B, H, n, d, w, g, block):
    """The banded restatement (full-length checks) against the dense-mask backward: row
    blocks that hold global rows, blocks of only global rows, window 0 and >= n."""
    rng = np.random.default_rng(n + w)
    Q, K, V, dO = (rng.standard_normal((B, H, n, d)) for _ in range(4))
    want = swa_oracle.sliding_window_attention_backward(Q, K, V, dO, w, g, 0.45)
    got = swa_oracle.sliding_window_attention_backward_banded(Q, K, V, dO, w, g, 0.45, block_rows=block)
    for a, b in zip(got, want):
        assert max_abs(a, b) < 1e-12
