"""GPU parity: the sm_100a kernels against the CPU oracle and the reference's own outputs.

Bar (fp16/bf16 inputs, fp32 accumulation): max-abs <= 2e-3, relative L2 <= 1e-3 on O,
max-abs <= 1e-4 on the row log-sum-exp.  Small cases are compared on every stored row;
the full-size workloads on a seeded sample of rows (all global rows, both sequence
ends, random interior rows) plus size-independent properties (determinism, head
independence).
"""
import math

import numpy as np
import pytest
import torch

import long_context_attention as lca
from long_context_attention import _native
from long_context_attention.workloads import WORKLOADS, make_inputs
from lca_testutil import (LSE_ABS_TOL, MAX_ABS_TOL, REL_L2_TOL, assert_parity, golden_names, gpu_capable, load_golden,
                          max_abs, rel_l2, to_np)
from oracle import swa_oracle

pytestmark = pytest.mark.gpu

GPU_CASES = [n for n in golden_names() if gpu_capable(load_golden(n))]


def _oracle(case, rows):
    return swa_oracle.sliding_window_attention(case["q"].float().numpy(), case["k"].float().numpy(),
                                               case["v"].float().numpy(), case["window"], case["globals"],
                                               case["scale"], rows=rows)


@pytest.mark.parametrize("name", GPU_CASES)
def test_golden_case_torch_api(name):
    c = load_golden(name)
    q, k, v = (t.cuda() for t in (c["q"], c["k"], c["v"]))
    out, lse = lca.sliding_window_attention_with_lse(q, k, v, c["window"], c["globals"], c["scale"])
    torch.cuda.synchronize()
    assert out.dtype == torch.float32 and out.shape == q.shape
    rows = c["rows"]
    got = to_np(out)[:, :, rows]
    assert_parity(got, c["out"], f"{name} vs reference output")
    want, want_lse = _oracle(c, rows)
    assert_parity(got, want, f"{name} vs oracle")
    assert max_abs(to_np(lse)[:, :, rows], want_lse) <= LSE_ABS_TOL, name
    # the reference's own signature gives the same bits
    out2 = lca.sliding_window_attention(q, k, v, c["window"], c["globals"], c["scale"])
    assert torch.equal(out2, out)
    assert lca.device_error() == 0


@pytest.mark.parametrize("name", ["ref_gpu_case_bf16", "two_global_tiles", "ragged_n_d128", "tiny_n5"])
def test_golden_case_c_abi(name):
    """Same computation through the raw C ABI (ctypes), with caller-owned workspace."""
    c = load_golden(name)
    cabi = _native.cabi()
    q, k, v = (t.cuda() for t in (c["q"], c["k"], c["v"]))
    B, H, n, d = q.shape
    out = torch.empty(B, H, n, d, device="cuda", dtype=torch.float32)
    lse = torch.empty(B, H, n, device="cuda", dtype=torch.float32)
    dt = cabi.DTYPE_BF16 if q.dtype == torch.bfloat16 else cabi.DTYPE_F16
    st, gl = cabi.normalize(c["globals"], n)
    assert st == cabi.OK
    st, ws_bytes = cabi.workspace_size(B, H, n, d, c["window"], len(gl), dt)
    assert st == cabi.OK
    ws = torch.empty(max(ws_bytes, 1), device="cuda", dtype=torch.uint8)
    stream = torch.cuda.current_stream().cuda_stream
    st = cabi.forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr(), dt, B, H, n, d,
                      c["window"], c["scale"], c["globals"], ws.data_ptr(), ws_bytes, stream)
    assert st == cabi.OK, cabi.last_error()
    torch.cuda.synchronize()
    rows = c["rows"]
    want, want_lse = _oracle(c, rows)
    assert_parity(to_np(out)[:, :, rows], want, f"{name} C ABI vs oracle")
    assert max_abs(to_np(lse)[:, :, rows], want_lse) <= LSE_ABS_TOL
    # One byte short of the reported size: the call runs without the optional part (the
    # work units go round-robin and, for bf16, P*V is split into hi + lo on every tile),
    # with the same results.
    out.zero_()
    st = cabi.forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), 0, dt, B, H, n, d, c["window"],
                      c["scale"], c["globals"], ws.data_ptr(), ws_bytes - 1, stream)
    assert st == cabi.OK, cabi.last_error()
    torch.cuda.synchronize()
    assert_parity(to_np(out)[:, :, rows], want, f"{name} C ABI (no optional workspace part) vs oracle")
    if gl:  # the global rows' buffers are never optional
        assert cabi.forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), 0, dt, B, H, n, d,
                            c["window"], c["scale"], c["globals"], ws.data_ptr(), 0, stream) == cabi.ERR_WORKSPACE


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("n,w,g", [(1, 0, []), (129, 0, [128]), (700, 300, [0, 699, 350]), (384, 5, list(range(0, 384, 3)))])
def test_shapes_and_windows(dtype, d, n, w, g):
    q, k, v = make_inputs(100 + n + d, 1, 2, n, d, dtype)
    out, lse = lca.sliding_window_attention_with_lse(q.cuda(), k.cuda(), v.cuda(), w, g, 0.1)
    want, want_lse = swa_oracle.sliding_window_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                                         w, g, 0.1)
    assert_parity(to_np(out), want, f"n={n} w={w} d={d} {dtype}")
    assert max_abs(to_np(lse), want_lse) <= LSE_ABS_TOL


@pytest.mark.parametrize("d", [64, 128])
def test_bf16_values_beyond_fp16_range(d):
    """bf16 inputs with V values far outside the fp16 range (2^17, 7e4, -1e30) in a few
    key tiles, a band tile and a global-key tile among them: P*V stays in bf16 (P split as
    hi + lo), so every finite bf16 value is handled.  (The fp32 accumulator holds
    sum p*v with p <= 2^8, so |v| far beyond 1e30 can overflow it; that range is not
    covered.)"""
    n, w, g = 1024, 200, [5, 900]
    q, k, v = make_inputs(77 + d, 1, 2, n, d, torch.bfloat16)
    v = v.clone()
    v[0, 0, 130] = 131072.0            # key tile 1 of head 0 (band tiles start at q0 - w)
    v[0, 1, 700, :8] = -1.0e30         # head 1
    v[0, 0, 900] = 70000.0             # a global key row
    out, lse = lca.sliding_window_attention_with_lse(q.cuda(), k.cuda(), v.cuda(), w, g, 0.1)
    want, want_lse = swa_oracle.sliding_window_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                                         w, g, 0.1)
    got = to_np(out)
    scale = np.abs(want).max(axis=-1, keepdims=True).clip(min=1.0)  # per-row magnitude of O
    assert np.isfinite(got).all()
    assert (np.abs(got - want) / scale).max() <= 2e-3
    assert max_abs(to_np(lse), want_lse) <= LSE_ABS_TOL


@pytest.mark.parametrize("d", [64, 128])
def test_bf16_tiny_values_keep_bf16_precision(d):
    """bf16 V values of ~1e-6 (below the fp16 normal range, where an fp16 copy would lose
    bits) in head 0, ordinary values in head 1 of the same call: head 0's tiles keep the
    bf16 P split, head 1's may use the fp16 copy of V, and both match the oracle relative
    to their own output magnitude."""
    n, w, g = 1024, 200, [5, 900]
    q, k, v = make_inputs(91 + d, 1, 2, n, d, torch.bfloat16)
    v = v.clone()
    v[0, 0] = (v[0, 0].float() * 1e-6).to(torch.bfloat16)
    out, lse = lca.sliding_window_attention_with_lse(q.cuda(), k.cuda(), v.cuda(), w, g, 0.1)
    want, want_lse = swa_oracle.sliding_window_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                                         w, g, 0.1)
    got = to_np(out)
    for h in range(2):
        assert rel_l2(got[:, h], want[:, h]) <= REL_L2_TOL, h
        assert np.abs(got[:, h] - want[:, h]).max() <= MAX_ABS_TOL * np.abs(want[:, h]).max(), h
    assert max_abs(to_np(lse), want_lse) <= LSE_ABS_TOL


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d", [64, 128])
def test_rising_scores_rescale_every_tile(d, dtype):
    """Scores that grow along every row (keys scaled by 1 + j/8 with q.k > 0: about
    +10 in log2 units per 128-key tile), so the row max rises by more than the
    lazy-rescale threshold (2^8) from one key tile to the next: the accumulator is
    rescaled on most tiles, and an exponent pass started against the previous reference
    max has to be redone with the new one.  The log-sum-exp reaches ~80 here, so it is
    compared relative to its magnitude (fp32 scores carry ~1e-7 relative error)."""
    n, w, g = 1536, 400, [2, 1000]
    q, k, v = make_inputs(53 + d, 1, 2, n, d, dtype)
    q = q.float().abs() * 0.5 + 0.25
    grow = 1.0 + torch.arange(n, dtype=torch.float32) / 8.0
    k = (k.float().abs() * 0.5 + 0.25) * grow[None, None, :, None]
    q, k = q.to(dtype), k.to(dtype)
    scale = 1.0 / d
    out, lse = lca.sliding_window_attention_with_lse(q.cuda(), k.cuda(), v.cuda(), w, g, scale)
    want, want_lse = swa_oracle.sliding_window_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                                         w, g, scale)
    assert_parity(to_np(out), want, f"rising scores d={d} {dtype}")
    assert (np.abs(to_np(lse) - want_lse) / np.maximum(np.abs(want_lse), 1.0)).max() <= LSE_ABS_TOL


@pytest.mark.parametrize("scale", [-0.2, 0.0, 1e-3])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_scale_edge_cases(scale, dtype):
    q, k, v = make_inputs(31, 1, 2, 300, 64, dtype)
    out, lse = lca.sliding_window_attention_with_lse(q.cuda(), k.cuda(), v.cuda(), 40, [3, 250], scale)
    want, want_lse = swa_oracle.sliding_window_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                                         40, [3, 250], scale)
    assert_parity(to_np(out), want, f"scale={scale} {dtype}")
    assert max_abs(to_np(lse), want_lse) <= LSE_ABS_TOL


def test_reference_gpu_test_restated():
    """tests/test_correctness.py:65-80 of the reference: seeded CUDA inputs, n=512, w=64,
    globals [0,1,2], fp16, compared with the dense definition at atol=rtol=2e-2 (and the
    stricter bar of this package)."""
    torch.manual_seed(2)
    Q, K, V = (torch.randn(1, 2, 512, 64, dtype=torch.float16, device="cuda") for _ in range(3))
    out = lca.sliding_window_attention(Q, K, V, 64, [0, 1, 2], 1.0 / math.sqrt(64))
    ref = lca._reference_sliding_window_attention(Q, K, V, 64, [0, 1, 2], 1.0 / math.sqrt(64))
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
    want, _ = swa_oracle.sliding_window_attention(Q.float().cpu().numpy(), K.float().cpu().numpy(),
                                                  V.float().cpu().numpy(), 64, [0, 1, 2], 0.125)
    assert_parity(to_np(out), want, "reference GPU test inputs")


def _sample_rows(n, globals_, count, seed):
    rng = np.random.default_rng(seed)
    rows = set(range(0, 130)) | set(range(n - 130, n)) | set(int(x) for x in rng.choice(n, count, replace=False))
    rows |= set(int(x) for x in globals_)
    return np.asarray(sorted(rows), dtype=np.int64)


@pytest.mark.parametrize("wname,heads_checked", [("single_head_16k", [0]), ("longformer_base_4k", [0, 57, 95]),
                                                 ("many_globals_64k", [0, 9, 15]), ("context_128k_d128", [0, 7])])
def test_full_size_workload_sampled(wname, heads_checked):
    w = WORKLOADS[wname]
    q, k, v = w.inputs(device="cuda")
    g = w.global_tokens()
    out, lse = lca.sliding_window_attention_with_lse(q, k, v, w.window, g, w.scale)
    out_again = lca.sliding_window_attention(q, k, v, w.window, g, w.scale)
    torch.cuda.synchronize()
    assert torch.equal(out, out_again), "two runs differ (the kernels are deterministic)"
    rows = _sample_rows(w.seq_len, g, 160, 5)
    for h in heads_checked:
        b, hh = divmod(h, w.heads)
        qs, ks, vs = (t[b:b + 1, hh:hh + 1].float().cpu().numpy() for t in (q, k, v))
        want, want_lse = swa_oracle.sliding_window_attention(qs, ks, vs, w.window, g, w.scale, rows=rows)
        got = to_np(out[b:b + 1, hh:hh + 1, rows])
        assert_parity(got, want, f"{wname} head {h}")
        assert max_abs(to_np(lse[b:b + 1, hh:hh + 1, rows]), want_lse) <= LSE_ABS_TOL
    # head independence: recomputing one head alone gives the same non-global rows bit
    # for bit (global rows are merged over a split count that depends on batch*heads, so
    # they agree to the rounding of P only: fp16 P on tiles read from the fp16 copy of V)
    h = heads_checked[-1]
    b, hh = divmod(h, w.heads)
    sl = (slice(b, b + 1), slice(hh, hh + 1))
    one = lca.sliding_window_attention(q[sl].contiguous(), k[sl].contiguous(), v[sl].contiguous(), w.window, g,
                                       w.scale)
    is_g = torch.zeros(w.seq_len, dtype=torch.bool, device=out.device)
    is_g[g] = True
    assert torch.equal(one[:, :, ~is_g], out[sl][:, :, ~is_g])
    torch.testing.assert_close(one[:, :, is_g], out[sl][:, :, is_g], atol=1e-4, rtol=1e-3)
    assert lca.device_error() == 0


def test_api_errors_on_gpu():
    q, k, v = make_inputs(1, 1, 1, 64, 64, torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError):
        lca.sliding_window_attention(q.float(), k.float(), v.float(), 4)
    with pytest.raises(RuntimeError):
        lca.sliding_window_attention(q.transpose(2, 3), k, v, 4)
    with pytest.raises(IndexError):
        lca.sliding_window_attention(q, k, v, 4, [64])
    with pytest.raises(RuntimeError):
        lca.sliding_window_attention(q, k, v, -1)
    q96 = torch.zeros(1, 1, 8, 96, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="head_dim"):
        lca.sliding_window_attention(q96, q96, q96, 4)
    empty = torch.zeros(0, 2, 16, 64, device="cuda", dtype=torch.float16)
    assert lca.sliding_window_attention(empty, empty, empty, 4, [1]).shape == (0, 2, 16, 64)


def test_side_stream_and_duplicate_globals():
    q, k, v = make_inputs(7, 1, 2, 520, 64, torch.float16, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        a = lca.sliding_window_attention(q, k, v, 33, [5, 5, -1, 200])
    s.synchronize()
    b = lca.sliding_window_attention(q, k, v, 33, [519, 200, 5])
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("name", ["ref_gpu_case_fp16", "ref_gpu_case_bf16", "dup_neg_globals", "no_globals_w0",
                                  "ragged_n_d128", "two_global_tiles"])
def test_extension_called_as_the_reference_dispatch_calls_it(name):
    """The reference's dispatch (python/long_context_attention/__init__.py:77-80) turns the
    global-token list into an int32 tensor on Q's device and calls the extension's
    ``sliding_window_attention_forward(Q, K, V, window_size, tensor, scale)``: the same call
    here, with negative and duplicate indices and an empty list among the cases, against the
    oracle and the reference's stored outputs.  (The extension reads that tensor on the host,
    so a CUDA tensor costs one blocking device-to-host copy per call.)"""
    c = load_golden(name)
    ext = _native.extension()
    q, k, v = (t.cuda() for t in (c["q"], c["k"], c["v"]))
    idx = torch.as_tensor(list(c["globals"]), dtype=torch.int32, device=q.device)
    out = ext.sliding_window_attention_forward(q, k, v, c["window"], idx, c["scale"])
    torch.cuda.synchronize()
    assert out.dtype == torch.float32 and out.shape == q.shape
    rows = c["rows"]
    got = to_np(out)[:, :, rows]
    assert_parity(got, c["out"], f"{name} (reference dispatch) vs reference output")
    want, _ = _oracle(c, rows)
    assert_parity(got, want, f"{name} (reference dispatch) vs oracle")
    # the index tensor may also live on the host, as the reference's binding allows
    out_host_idx = ext.sliding_window_attention_forward(q, k, v, c["window"], idx.cpu(), c["scale"])
    assert torch.equal(out_host_idx, out)


def test_extension_index_tensor_out_of_range_raises():
    q, k, v = make_inputs(3, 1, 1, 256, 64, torch.float16, device="cuda")
    with pytest.raises(IndexError):
        _native.extension().sliding_window_attention_forward(
            q, k, v, 16, torch.tensor([0, 256], dtype=torch.int32, device="cuda"), 0.125)
    empty = torch.empty(0, dtype=torch.int32, device="cuda")
    out = _native.extension().sliding_window_attention_forward(q, k, v, 16, empty, 0.125)
    want, _ = swa_oracle.sliding_window_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                                  v.float().cpu().numpy(), 16, [], 0.125)
    assert_parity(to_np(out), want, "empty index tensor")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_many_globals_beyond_shared_index_list(dtype):
    """More global tokens (3000) than the d=64 kernel keeps in shared memory (2048): the
    band rows then search the sorted index list in global memory.  Checked on every global
    row (the global-row units) and a sample of the others against the oracle."""
    n, w = 8192, 128
    rng = np.random.default_rng(11)
    g = sorted(int(x) for x in rng.choice(n, 3000, replace=False))
    q, k, v = make_inputs(12, 1, 1, n, 64, dtype)
    out, lse = lca.sliding_window_attention_with_lse(q.cuda(), k.cuda(), v.cuda(), w, g, 0.125)
    rows = np.asarray(sorted(set(rng.choice(n, 300, replace=False).tolist()) | set(g[::10]) | {0, n - 1}))
    want, want_lse = swa_oracle.sliding_window_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                                         w, g, 0.125, rows=rows)
    assert_parity(to_np(out)[:, :, rows], want, f"3000 globals {dtype}")
    assert max_abs(to_np(lse)[:, :, rows], want_lse) <= LSE_ABS_TOL
    assert lca.device_error() == 0
