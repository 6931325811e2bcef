"""lca_swa_forward_noalloc, the entry point for callers that cannot allocate device memory.

Such callers (a serving loop whose device memory belongs to its own pool allocator, a
plugin inside a runtime that forbids allocation after start-up) cannot provide the
workspace lca_swa_forward needs; this entry point uses a fixed scratch array inside the
library instead.  Its results must equal those of the allocating entry point, call after
call, since every call reuses the same array.  This file is collected last so that a run
stopping at the first failure has already run every other test; it also passes when run
on its own in a fresh process.
"""
import re
import os

import numpy as np
import pytest
import torch

from long_context_attention import _native
from long_context_attention.workloads import make_inputs
from lca_testutil import LSE_ABS_TOL, assert_parity, max_abs, to_np
from oracle import swa_oracle

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# (seed, B, H, n, d, dtype, window, global tokens, scale): different problems one after
# the other, each smaller than the one before in some part of the scratch, so stale
# scratch from an earlier call would show.  The third has no global tokens (nothing of
# the scratch is required; the optional fp16 copy of V and the work-unit counter still
# use it); the last is a bf16 problem whose optional part (16 MiB of fp16 V per head pair
# here, 64 MiB in all) does not fit the array while the required part does, so it runs
# without the optional part.
CASES = [
    (41, 1, 4, 4096, 64, torch.bfloat16, 256, [0, 17, 2048, 4095, -7], 0.125),
    (42, 2, 1, 1000, 128, torch.float16, 100, [3, 999, 500], 1 / 11.3),
    (43, 1, 3, 2000, 64, torch.bfloat16, 64, [], 0.125),
    (44, 1, 4, 65536, 64, torch.bfloat16, 256, [0, 30000, 65535], 0.125),
]


def _dtype_code(cabi, dt):
    return cabi.DTYPE_BF16 if dt == torch.bfloat16 else cabi.DTYPE_F16


def _inputs(case):
    seed, B, H, n, d, dt, w, g, scale = case
    return make_inputs(seed, B, H, n, d, dt, device="cuda")


def _run(cabi, case, noalloc: bool):
    seed, B, H, n, d, dt, w, g, scale = case
    q, k, v = _inputs(case)
    out = torch.full((B, H, n, d), float("nan"), device="cuda", dtype=torch.float32)
    lse = torch.full((B, H, n), float("nan"), device="cuda", dtype=torch.float32)
    stream = torch.cuda.current_stream().cuda_stream
    code = _dtype_code(cabi, dt)
    if noalloc:
        st = cabi.forward_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr(), code, B,
                                  H, n, d, w, scale, g, stream)
    else:
        st, gl = cabi.normalize(g, n)
        assert st == cabi.OK
        st, ws_bytes = cabi.workspace_size(B, H, n, d, w, len(gl), code)
        assert st == cabi.OK
        ws = torch.empty(max(ws_bytes, 1), device="cuda", dtype=torch.uint8)
        st = cabi.forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr(), code, B, H, n,
                          d, w, scale, g, ws.data_ptr(), ws_bytes, stream)
    assert st == cabi.OK, cabi.last_error()
    torch.cuda.synchronize()
    return to_np(out), to_np(lse)


def _oracle_rows(case, rows):
    seed, B, H, n, d, dt, w, g, scale = case
    q, k, v = (t.float().cpu().numpy() for t in _inputs(case))
    return swa_oracle.sliding_window_attention(q, k, v, w, g, scale, rows=rows)


def test_noalloc_matches_allocating_entry_point_on_consecutive_calls():
    cabi = _native.cabi()
    st, need = cabi.workspace_size(1, 4, 65536, 64, 256, 3, cabi.DTYPE_BF16)
    assert st == cabi.OK and need > (32 << 20), "the last case must exceed the array with its optional part"
    for case in CASES:
        first, first_lse = _run(cabi, case, noalloc=True)
        got, got_lse = _run(cabi, case, noalloc=True)  # the same problem again over what the first call left
        want, want_lse = _run(cabi, case, noalloc=False)
        assert np.array_equal(first, got) and np.array_equal(first_lse, got_lse), f"case seed {case[0]}"
        assert_parity(got, want, f"noalloc vs workspace entry point, case seed {case[0]}")
        assert max_abs(got_lse, want_lse) <= LSE_ABS_TOL
        # and directly against the oracle, on every row of the small cases and a sample of the large one
        n = case[3]
        rows = np.arange(n) if n <= 4096 else np.unique(np.r_[0:64, n - 64:n, np.random.default_rng(3).choice(
            n, 100, replace=False), np.asarray(case[7]) % n])
        o_want, o_lse = _oracle_rows(case, rows)
        assert_parity(got[:, :, rows], o_want, f"noalloc vs oracle, case seed {case[0]}")
        assert max_abs(got_lse[:, :, rows], o_lse) <= LSE_ABS_TOL


def test_noalloc_rejects_problems_larger_than_its_scratch():
    cabi = _native.cabi()
    hdr = open(os.path.join(REPO, "include", "lca.h")).read()
    limit = int(re.search(r"#define LCA_NOALLOC_SCRATCH_BYTES \((\d+)u << (\d+)\)", hdr).group(1)) << 20
    B, H, n, d, w, g = 1, 4096, 65536, 64, 256, list(range(0, 65536, 1000))
    st, gl = cabi.normalize(g, n)
    st, need = cabi.workspace_size(B, H, n, d, w, len(gl), cabi.DTYPE_BF16)
    assert need > limit
    # the shape is only described; nothing is launched, so small buffers stand in
    t = torch.zeros(16, device="cuda", dtype=torch.float32)
    st = cabi.forward_noalloc(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), None, cabi.DTYPE_BF16, B, H,
                              n, d, w, 0.125, g, torch.cuda.current_stream().cuda_stream)
    assert st == cabi.ERR_UNSUPPORTED
    assert "scratch" in cabi.last_error()
