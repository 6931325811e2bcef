"""Host-side logic that needs no GPU: work accounting, global-token normalisation (Python
and C ABI agree with the reference's indexing rules), workspace sizing and the Python
API's dispatch rules."""
import math
import os
import re

import numpy as np
import pytest
import torch

import long_context_attention as lca
from long_context_attention import _native
from long_context_attention.workloads import WORKLOADS, make_inputs, normalize_global_tokens, useful_scores
from oracle import swa_oracle

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("n,w,g", [(1, 0, []), (5, 2, [4]), (300, 17, [5, 5, -1, 150, 0]), (257, 0, []),
                                   (200, 1000, [3]), (640, 64, list(range(0, 640, 7))), (1024, 128, [512]),
                                   (333, 70, [332, -333])])
def test_useful_scores_counts_the_dense_mask(n, w, g):
    gi = swa_oracle.normalize_global_tokens(g, n)
    dense = int(swa_oracle.visible_rows(np.arange(n), n, w, gi).sum())
    assert useful_scores(n, w, g) == dense


def test_workload_definitions():
    w4 = WORKLOADS["many_globals_64k"]
    g = w4.global_tokens()
    assert g[0] == 0 and g == sorted(set(g)) and 64 <= len(g) <= 65 and max(g) < w4.seq_len
    assert WORKLOADS["context_128k_d128"].global_tokens() == list(range(16))
    assert WORKLOADS["single_head_16k"].useful_scores() == 8435956  # figure quoted for this shape
    assert WORKLOADS["cpu_plumbing_2k"].useful_scores() == 521332


def test_make_inputs_heads_slice_matches_full():
    q, k, v = make_inputs(3, 1, 4, 16, 8, torch.bfloat16)
    qs, ks, vs = make_inputs(3, 1, 4, 16, 8, torch.bfloat16, heads_slice=slice(1, 3))
    assert torch.equal(qs, q[:, 1:3]) and torch.equal(vs, v[:, 1:3])


@pytest.mark.parametrize("tokens,n", [([], 10), ([0, 0, 5], 10), ([-1, 3, -10], 10), ([9, 8, 7, 7], 10)])
def test_normalize_python_and_cabi_agree(tokens, n):
    cabi = _native.cabi()
    st, got = cabi.normalize(tokens, n)
    assert st == cabi.OK
    assert got == normalize_global_tokens(tokens, n) == list(swa_oracle.normalize_global_tokens(tokens, n))


@pytest.mark.parametrize("tokens", [[10], [-11], [3, 100]])
def test_normalize_out_of_range(tokens):
    cabi = _native.cabi()
    st, _ = cabi.normalize(tokens, 10)
    assert st == cabi.ERR_INDEX
    assert "out of bounds" in cabi.last_error()
    with pytest.raises(IndexError):
        normalize_global_tokens(tokens, 10)


def test_workspace_size():
    cabi = _native.cabi()
    st, b0 = cabi.workspace_size(1, 16, 65536, 64, 256, 0, cabi.DTYPE_F16)
    # fp16 without globals: only the optional work-unit counter (one 1024-byte aligned block)
    assert st == cabi.OK and b0 == 1024
    # bf16: the recommended size includes the fp16 copy of V (16 heads x 65536 x 64 x 2B)
    st, b0 = cabi.workspace_size(1, 16, 65536, 64, 256, 0, cabi.DTYPE_BF16)
    assert st == cabi.OK and b0 >= 16 * 65536 * 64 * 2
    st, b1 = cabi.workspace_size(1, 16, 65536, 64, 256, 65, cabi.DTYPE_F16)
    assert st == cabi.OK
    # compact Q/K/V global rows (16 heads x 65 rows x 64 x 2B each) + at least two split partials
    assert b1 >= 3 * 16 * 65 * 64 * 2 + 2 * 16 * 65 * 64 * 4
    assert b1 % 1024 == 0
    st, b2 = cabi.workspace_size(1, 16, 65536, 64, 256, 65, cabi.DTYPE_BF16)
    assert st == cabi.OK and b2 >= b1 + 16 * 65536 * 64 * 2 + 65 * 16 * 64 * 2 and b2 % 1024 == 0
    st, _ = cabi.workspace_size(1, 16, 65536, 96, 256, 65, cabi.DTYPE_BF16)
    assert st == cabi.ERR_UNSUPPORTED


def test_api_cpu_tensors_require_force_reference():
    q, k, v = make_inputs(0, 1, 1, 16, 8, torch.float32)
    with pytest.raises(RuntimeError, match="CUDA"):
        lca.sliding_window_attention(q, k, v, 2, [0])
    out = lca.sliding_window_attention(q, k, v, 2, [0], force_reference=True)
    ref, _ = swa_oracle.sliding_window_attention(q.numpy(), k.numpy(), v.numpy(), 2, [0], 1 / math.sqrt(8))
    np.testing.assert_allclose(out.numpy(), ref, atol=1e-6)
    assert out.dtype == torch.float32


def test_reference_helper_is_importable_under_reference_name():
    from long_context_attention import _reference_sliding_window_attention  # noqa: F401
    assert "sliding_window_attention" in lca.__all__


def test_header_documents_reference_interfaces():
    hdr = open(os.path.join(REPO, "include", "lca.h")).read()
    # the forward entry point cites the reference binding it replaces
    assert "csrc/bindings.cpp:31-73" in hdr


def test_window_per_head_argument_and_oracle():
    """One radius per head: the Python argument checks, and the oracle's per-head radii
    against running it head by head with one radius each."""
    import numpy as np
    import pytest
    import torch

    from long_context_attention import _head_windows
    from oracle import swa_oracle
    assert _head_windows(5, 3) == (5, [])
    assert _head_windows([1, 7, 2], 3) == (7, [1, 7, 2])
    assert _head_windows(torch.tensor([4, 0]), 2) == (4, [4, 0])
    with pytest.raises(ValueError):
        _head_windows([1, 2], 3)
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, 3, 80, 8)) for _ in range(3))
    radii = [0, 9, 100]
    got, lse = swa_oracle.sliding_window_attention(q, k, v, radii, [4, 70], 0.5)
    for h, w in enumerate(radii):
        want, want_lse = swa_oracle.sliding_window_attention(q[:, h:h + 1], k[:, h:h + 1], v[:, h:h + 1], w, [4, 70],
                                                             0.5)
        assert np.array_equal(got[:, h:h + 1], want) and np.array_equal(lse[:, h:h + 1], want_lse)
