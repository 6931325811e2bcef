"""Sequence shards on the GPU.

* Emulated ranks on one GPU: every shard's native steps run on cuda:0 and the test
  performs the exchanges itself (each shard's global rows to all others, halo copies,
  gather of the per-shard partials) between the shards' workspaces.  This checks the
  shard kernels (halo tensor maps, shard offsets, per-shard global-row partials and
  their merge) against the oracle and against the unsharded forward.
* Real ranks over NCCL (needs >= 2 GPUs): sliding_window_attention_sharded end to end.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

import long_context_attention as lca
from long_context_attention.distributed import (NativeShardSteps, ShardSpec, _dtype_code, _normalize,
                                                global_row_runs, shard_bounds)
from long_context_attention.workloads import WORKLOADS, make_inputs
from lca_testutil import LSE_ABS_TOL, MAX_ABS_TOL, REL_L2_TOL, max_abs, rel_l2
from oracle import swa_oracle

pytestmark = pytest.mark.gpu

_DT = {"fp16": torch.float16, "bf16": torch.bfloat16}


def run_emulated(q, k, v, window, tokens, scale, world, with_lse=True):
    """All shards of one problem on the current GPU, exchanges done by copies."""
    B, H, N, d = q.shape
    steps = NativeShardSteps()
    toks = _normalize(tokens, N)
    bounds = shard_bounds(N, world)
    specs, lays, wss, outs, lses, parts = [], [], [], [], [], []
    for r, (off, ln) in enumerate(bounds):
        spec = ShardSpec(B, H, N, d, window, r, world, off, ln, _dtype_code(q.dtype), float(scale))
        lay = steps.layout(spec, len(toks))
        ws = steps.workspace(lay.total_bytes, q.device)
        ws.fill_(0xFF)  # stale bytes must never be read: 0xFFFF is a NaN in fp16 / bf16
        parts.append(tuple(t[:, :, off:off + ln].contiguous() for t in (q, k, v)))
        specs.append(spec)
        lays.append(lay)
        wss.append(ws)
        outs.append(torch.empty(B, H, ln, d, dtype=torch.float32, device=q.device))
        lses.append(torch.empty(B, H, ln, dtype=torch.float32, device=q.device) if with_lse else None)
    for r in range(world):
        steps.prepare(specs[r], *parts[r], toks, wss[r])
    lay0 = lays[0]
    if lay0.globals_bytes:
        # each shard's run of global rows goes to every other shard, same offsets
        rb = lay0.globals_row_bytes
        for r, (lo, hi) in enumerate(global_row_runs(toks, bounds)):
            for t in range(world):
                if t != r and hi > lo:
                    a, b = lays[r].globals_offset, lays[t].globals_offset
                    wss[t][b + lo * rb:b + hi * rb].copy_(wss[r][a + lo * rb:a + hi * rb])
    for r in range(world):
        lay, side = lays[r], lays[r].halo_side_bytes
        if lay.halo_rows == 0:
            continue
        recv = lay.halo_recv_offset
        if r > 0:
            sl = lays[r - 1]
            src = wss[r - 1][sl.halo_send_offset + side:sl.halo_send_offset + 2 * side]
            wss[r][recv:recv + side].copy_(src)
        if r < world - 1:
            sl = lays[r + 1]
            src = wss[r + 1][sl.halo_send_offset:sl.halo_send_offset + side]
            wss[r][recv + side:recv + 2 * side].copy_(src)
    for r in range(world):
        steps.forward(specs[r], *parts[r], outs[r], lses[r], toks, wss[r])
    if lay0.rowpart_bytes:
        rp = [w[l.rowpart_offset:l.rowpart_offset + l.rowpart_bytes] for w, l in zip(wss, lays)]
        allp = torch.cat(rp)
        for w, l in zip(wss, lays):
            w[l.rowpart_all_offset:l.rowpart_all_offset + world * l.rowpart_bytes].copy_(allp)
    for r in range(world):
        steps.finish(specs[r], outs[r], lses[r], toks, wss[r])
    torch.cuda.synchronize()
    assert lca.device_error() == 0
    return torch.cat(outs, dim=2), (torch.cat(lses, dim=2) if with_lse else None)


def check_rows(out, lse, q, k, v, window, tokens, scale, rows):
    ref_o, ref_l = swa_oracle.sliding_window_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                                       v.float().cpu().numpy(), window, tokens, scale, rows=rows)
    o = out[:, :, rows].cpu().numpy()
    assert max_abs(o, ref_o) <= MAX_ABS_TOL
    assert rel_l2(o, ref_o) <= REL_L2_TOL
    if lse is not None:
        assert max_abs(lse[:, :, rows].cpu().numpy(), ref_l) <= LSE_ABS_TOL


CASES = [
    # name, world, batch, heads, n, d, w, dtype, globals, scale
    ("two_shards", 2, 1, 2, 1024, 64, 100, "bf16", [0, 5, 511, 512, 1000], 0.125),
    ("four_shards_w_eq_shard", 4, 1, 1, 1024, 128, 256, "fp16", [0], 1 / 128 ** 0.5),
    ("three_ragged", 3, 2, 1, 700, 64, 130, "bf16", [255, 256, 600, 3, -1], 0.1),
    ("unaligned_window", 2, 1, 2, 2048, 64, 200, "bf16", [1023, 1024, 1025], 0.125),
    ("no_globals", 2, 1, 1, 512, 128, 64, "bf16", [], 0.09),
    ("window_zero", 2, 1, 1, 256, 64, 0, "fp16", [7], 0.125),
    ("one_shard", 1, 1, 2, 640, 64, 64, "bf16", [3, 600], 0.125),
    ("many_globals", 2, 1, 1, 1024, 64, 32, "bf16", list(range(0, 1024, 5)), 0.125),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_emulated_shards_match_oracle(case):
    _, world, B, H, n, d, w, dt, g, scale = case
    q, k, v = make_inputs(31 + n + world, B, H, n, d, _DT[dt], device="cuda")
    out, lse = run_emulated(q, k, v, w, g, scale, world)
    check_rows(out, lse, q, k, v, w, g, scale, np.arange(n))
    # the unsharded forward agrees too (different tile boundaries: not bitwise)
    ref, ref_l = lca.sliding_window_attention_with_lse(q, k, v, w, g, scale)
    assert (out - ref).abs().max().item() <= MAX_ABS_TOL
    assert (lse - ref_l).abs().max().item() <= LSE_ABS_TOL


def test_emulated_context_128k_eight_shards():
    """The 128K-token, d=128 workload in 8 shards: sampled rows (shard edges, globals,
    random) against the oracle, every row against the unsharded forward."""
    wl = WORKLOADS["context_128k_d128"]
    q, k, v = wl.inputs(device="cuda")
    g = wl.global_tokens()
    out, lse = run_emulated(q, k, v, wl.window, g, wl.scale, 8)
    n = wl.seq_len
    edges = [b for off, _ in shard_bounds(n, 8) for b in range(max(0, off - 3), min(n, off + 3))]
    rng = np.random.default_rng(5)
    rows = np.unique(np.concatenate([np.asarray(g), np.asarray(edges), rng.integers(0, n, 64), [n - 1]]))
    check_rows(out, lse, q, k, v, wl.window, g, wl.scale, rows)
    ref, ref_l = lca.sliding_window_attention_with_lse(q, k, v, wl.window, g, wl.scale)
    assert (out - ref).abs().max().item() <= MAX_ABS_TOL
    assert (lse - ref_l).abs().max().item() <= LSE_ABS_TOL


# ---------------------------------------------------------------------- NCCL ranks

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, outdir):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from long_context_attention.distributed import sliding_window_attention_sharded

        n, w, g = 4096, 300, [0, 1, 2047, 2048, 4000]
        q, k, v = make_inputs(77, 1, 4, n, 64, torch.bfloat16)
        off, ln = shard_bounds(n, world)[rank]
        sl = slice(off, off + ln)
        dev = torch.device("cuda", rank)
        out, lse = sliding_window_attention_sharded(
            q[:, :, sl].contiguous().to(dev), k[:, :, sl].contiguous().to(dev), v[:, :, sl].contiguous().to(dev),
            w, g, 0.125, seq_len=n, return_lse=True)
        torch.cuda.synchronize()
        np.save(os.path.join(outdir, f"o{rank}.npy"), out.cpu().numpy())
        np.save(os.path.join(outdir, f"l{rank}.npy"), lse.cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nccl_ranks_match_oracle(tmp_path):
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 4)
    mp.spawn(_nccl_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    out = np.concatenate([np.load(tmp_path / f"o{r}.npy") for r in range(world)], axis=2)
    lse = np.concatenate([np.load(tmp_path / f"l{r}.npy") for r in range(world)], axis=2)
    q, k, v = make_inputs(77, 1, 4, 4096, 64, torch.bfloat16)
    ref_o, ref_l = swa_oracle.sliding_window_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                                       300, [0, 1, 2047, 2048, 4000], 0.125)
    assert max_abs(out, ref_o) <= MAX_ABS_TOL
    assert rel_l2(out, ref_o) <= REL_L2_TOL
    assert max_abs(lse, ref_l) <= LSE_ABS_TOL


def _peer_rank(rank, world, port, outdir, cases):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        from long_context_attention.distributed import ShardedAttention

        for ci, (n, d, w, g, seed) in enumerate(cases):
            q, k, v = make_inputs(seed, 1, 2, n, d, torch.bfloat16)
            plan = ShardedAttention(1, 2, n, d, w, g, 0.1, torch.bfloat16, device=dev, return_lse=True,
                                    exchange="peer")
            off, ln = plan.shard
            qs, ks, vs = (t[:, :, off:off + ln].contiguous().to(dev) for t in (q, k, v))
            outs = []
            for _ in range(3):  # eager steps (the step counter advances each time)
                o, l = plan(qs, ks, vs)
                outs.append((o.clone(), l.clone()))
            plan.capture(qs, ks, vs)
            for _ in range(3):
                o, l = plan.replay()
            torch.cuda.synchronize()
            outs.append((o.clone(), l.clone()))
            assert lca.device_error() == 0
            for i, (o, l) in enumerate(outs):
                np.save(os.path.join(outdir, f"c{ci}_s{i}_o{rank}.npy"), o.cpu().numpy())
                np.save(os.path.join(outdir, f"c{ci}_s{i}_l{rank}.npy"), l.cpu().numpy())
            plan.release()
    finally:
        dist.destroy_process_group()


PEER_CASES = [(4096, 64, 300, [0, 1, 2047, 2048, 4000], 77), (2048, 128, 128, [], 78), (1920, 64, 64, [1919], 79)]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_exchange_ranks_match_oracle(tmp_path):
    """The peer-memory exchange (NVLink stores into the other ranks' workspaces, no
    collectives in the step): eager steps and CUDA-graph replays on 2-4 GPUs."""
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 4)
    mp.spawn(_peer_rank, args=(world, _free_port(), str(tmp_path), PEER_CASES), nprocs=world, join=True)
    for ci, (n, d, w, g, seed) in enumerate(PEER_CASES):
        q, k, v = make_inputs(seed, 1, 2, n, d, torch.bfloat16)
        ref_o, ref_l = swa_oracle.sliding_window_attention(q.float().numpy(), k.float().numpy(),
                                                           v.float().numpy(), w, g, 0.1)
        for i in range(4):
            out = np.concatenate([np.load(tmp_path / f"c{ci}_s{i}_o{r}.npy") for r in range(world)], axis=2)
            lse = np.concatenate([np.load(tmp_path / f"c{ci}_s{i}_l{r}.npy") for r in range(world)], axis=2)
            assert max_abs(out, ref_o) <= MAX_ABS_TOL, (ci, i)
            assert rel_l2(out, ref_o) <= REL_L2_TOL, (ci, i)
            assert max_abs(lse, ref_l) <= LSE_ABS_TOL, (ci, i)
