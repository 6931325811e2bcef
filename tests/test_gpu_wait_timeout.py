"""A bounded device wait that runs out, on one GPU, without a fault.

Every wait in the kernels has a time limit (LCA_WAIT_TIMEOUT_MS, 2 s by default); one
that runs out records its code in the device error word and the kernel returns, so the
CUDA context stays usable.  Here the peer-exchange kernel of a two-rank sequence shard
runs with both "ranks'" workspaces on this one GPU: rank 0's kernel stores its halos and
global rows into the buffer standing in for rank 1 and bumps the counter there, then
waits for rank 1's counter in its own workspace -- which nothing ever bumps.  The wait
gives up after 50 ms, the host reads LCA_DEVERR_TIMEOUT_PEER, the Python check raises,
and a normal forward in the same process afterwards is still at parity with the oracle.

The limit is read once per process, so the scenario runs in a child process with
LCA_WAIT_TIMEOUT_MS=50.
"""
import json
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)

CHILD = textwrap.dedent(r"""
    import ctypes, json, sys, time
    sys.path[:0] = [__PATHS__]
    import numpy as np
    import torch
    import long_context_attention as lca
    from long_context_attention import _native
    from long_context_attention.distributed import ShardSpec, NativeShardSteps
    from long_context_attention.workloads import make_inputs
    from oracle import swa_oracle

    res = {}
    lib = _native.cabi()
    B, H, n, d, w = 1, 2, 1024, 64, 64
    tokens = [3, 700]
    spec = ShardSpec(B, H, n, d, w, 0, 2, 0, 512, lib.DTYPE_BF16, 0.125)   # rank 0 of 2
    steps = NativeShardSteps()
    lay = steps.layout(spec, len(tokens))
    own = torch.zeros(lay.total_bytes, dtype=torch.uint8, device="cuda")
    stand_in = torch.zeros(lay.total_bytes, dtype=torch.uint8, device="cuda")  # "rank 1": never signals
    q, k, v = make_inputs(5, B, H, n, d, torch.bfloat16, device="cuda")
    qs, ks, vs = (t[:, :, :512].contiguous() for t in (q, k, v))
    steps.prepare(spec, qs, ks, vs, tokens, own)
    peers = (ctypes.c_void_p * 2)(own.data_ptr(), stand_in.data_ptr())
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    steps.exchange_peer(spec, tokens, peers, lay.total_bytes, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    res["wait_s"] = time.perf_counter() - t0
    # the stand-in received rank 0's halo rows (side 1 -> its receive side 0) before the wait
    res["halo_delivered"] = bool(torch.equal(stand_in[lay.halo_recv_offset:lay.halo_recv_offset + lay.halo_side_bytes],
                                             own[lay.halo_send_offset + lay.halo_side_bytes:
                                                 lay.halo_send_offset + 2 * lay.halo_side_bytes]))
    try:
        lca.raise_on_device_error()
        res["raised"] = None
    except RuntimeError as e:
        res["raised"] = str(e)
    res["code_after_check"] = lca.device_error()   # the check cleared the word
    # the context is still usable: a normal forward matches the oracle
    out, lse = lca.sliding_window_attention_with_lse(q, k, v, w, tokens, 0.125)
    want, want_lse = swa_oracle.sliding_window_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                                         v.float().cpu().numpy(), w, tokens, 0.125)
    got = out.cpu().numpy()
    res["max_abs"] = float(np.abs(got - want).max())
    res["rel_l2"] = float(np.linalg.norm(got - want) / np.linalg.norm(want))
    res["lse_err"] = float(np.abs(lse.cpu().numpy() - want_lse).max())
    res["code_end"] = lca.device_error()
    print("RESULT " + json.dumps(res))
""")


def test_peer_wait_runs_out_and_context_survives():
    paths = ", ".join(repr(p) for p in (os.path.join(REPO, "long-context-attention-kernels_b200", "python"), REPO))
    env = dict(os.environ, LCA_WAIT_TIMEOUT_MS="50")
    proc = subprocess.run([sys.executable, "-c", CHILD.replace("__PATHS__", paths)], env=env, capture_output=True,
                          text=True, timeout=300)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-4000:]
    line = [ln for ln in proc.stdout.splitlines() if ln.startswith("RESULT ")][-1]
    res = json.loads(line[len("RESULT "):])
    assert res["raised"] is not None and "device error 5" in res["raised"], res
    assert res["code_after_check"] == 0
    assert 0.04 <= res["wait_s"] < 5.0, res          # ended by the 50 ms limit, not by luck or a hang
    assert res["halo_delivered"], res
    assert res["max_abs"] <= 2e-3 and res["rel_l2"] <= 1e-3 and res["lse_err"] <= 1e-4, res
    assert res["code_end"] == 0
