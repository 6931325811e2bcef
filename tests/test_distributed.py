"""Multi-rank host logic without a GPU: shard planning, the shard workspace layout and
validation of the C ABI, and the whole sequence-sharded forward (halo exchange, global
row all-reduce, partial all-gather, merge) on world_size 2 and 3 ``gloo`` ranks, with
the compute steps restated on the CPU (tests/shard_cpu_steps.py) and the result checked
against the oracle over the whole sequence."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from long_context_attention import _native
from long_context_attention.distributed import ShardSpec, head_shard, shard_bounds
from long_context_attention.workloads import make_inputs
from oracle import swa_oracle


def test_shard_bounds():
    assert shard_bounds(131072, 8) == [(r * 16384, 16384) for r in range(8)]
    assert shard_bounds(700, 3) == [(0, 256), (256, 256), (512, 188)]
    assert shard_bounds(5, 1) == [(0, 5)]
    for n, w in [(1000, 2), (4096, 4), (129, 2), (100000, 7)]:
        b = shard_bounds(n, w)
        assert len(b) == w and b[0][0] == 0 and sum(ln for _, ln in b) == n
        assert all(b[i][0] + b[i][1] == b[i + 1][0] for i in range(w - 1))
        assert all(ln % 128 == 0 for _, ln in b[:-1]) and b[-1][1] >= 1
    with pytest.raises(ValueError):
        shard_bounds(200, 4)


def test_head_shard():
    assert [head_shard(16, 8, r) for r in range(8)] == [slice(2 * r, 2 * r + 2) for r in range(8)]
    sl = [head_shard(10, 4, r) for r in range(4)]
    assert [s.stop - s.start for s in sl] == [3, 3, 2, 2] and sl[-1].stop == 10


def _spec(**kw):
    a = dict(batch=1, heads=8, seq_len=131072, head_dim=128, window=512, rank=1, world_size=8, offset=16384,
             length=16384, dtype_code=1, scale=0.088)
    a.update(kw)
    return ShardSpec(**a)


def test_shard_layout_sizes():
    c = _native.cabi()
    st, lay = c.shard_layout(_spec().desc(), 16)
    assert st == c.OK, c.last_error()
    bh, d, G, w = 8, 128, 16, 512
    assert lay.halo_rows == w
    assert lay.globals_bytes == 3 * bh * G * d * 2 and lay.globals_row_bytes == 3 * bh * d * 2
    assert lay.halo_side_bytes == 2 * bh * w * d * 2
    assert lay.rowpart_bytes == bh * G * d * 4 + -(-bh * G * 4 // 16) * 16 and lay.rowpart_bytes % 16 == 0
    st, lay_odd = c.shard_layout(_spec(heads=1).desc(), 5)  # 5 LSE floats pad to 8
    assert st == c.OK and lay_odd.rowpart_bytes == 5 * d * 4 + 32
    regions = sorted([(lay.globals_offset, lay.globals_bytes), (lay.halo_send_offset, 2 * lay.halo_side_bytes),
                      (lay.halo_recv_offset, 2 * lay.halo_side_bytes), (lay.rowpart_offset, lay.rowpart_bytes),
                      (lay.rowpart_all_offset, 8 * lay.rowpart_bytes)])
    for (o0, s0), (o1, _) in zip(regions, regions[1:]):
        assert o0 + s0 <= o1 and o0 % 256 == 0
    assert regions[-1][0] + regions[-1][1] <= lay.total_bytes
    # no globals: no global-row regions; one shard: no halo
    st, lay0 = c.shard_layout(_spec().desc(), 0)
    assert st == c.OK and lay0.globals_bytes == 0 and lay0.rowpart_bytes == 0 and lay0.halo_side_bytes > 0
    st, lay1 = c.shard_layout(_spec(world_size=1, rank=0, offset=0, length=131072).desc(), 16)
    assert st == c.OK and lay1.halo_rows == 0 and lay1.halo_side_bytes == 0


def test_shard_validation():
    c = _native.cabi()
    bad = [
        (_spec(window=20000), c.ERR_UNSUPPORTED),                 # halo wider than a shard
        (_spec(length=16100), c.ERR_UNSUPPORTED),                 # middle shard not a multiple of 128
        (_spec(offset=130000, length=2000), c.ERR_INVALID_ARGUMENT),  # beyond the sequence
        (_spec(world_size=0), c.ERR_INVALID_ARGUMENT),
        (_spec(head_dim=96), c.ERR_UNSUPPORTED),
        (_spec(window=-1), c.ERR_INVALID_ARGUMENT),
        (_spec(rank=8), c.ERR_INVALID_ARGUMENT),                  # rank outside [0, world_size)
    ]
    for spec, code in bad:
        st, _ = c.shard_layout(spec.desc(), 4)
        assert st == code, (spec, st, c.last_error())
    # the last shard may be ragged
    st, _ = c.shard_layout(_spec(offset=131072 - 1000, length=1000, window=500).desc(), 4)
    assert st == c.OK, c.last_error()
    # an out-of-range global token is an index error before any device work
    st = c.shard_prepare(_spec().desc(), None, None, None, [131072], None, 0, None)
    assert st == c.ERR_INDEX


# ---------------------------------------------------------------------- gloo ranks

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, case, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from long_context_attention.distributed import sliding_window_attention_sharded
        from shard_cpu_steps import CpuShardSteps

        q, k, v = make_inputs(case["seed"], case["batch"], case["heads"], case["n"], case["d"], torch.bfloat16)
        off, ln = shard_bounds(case["n"], world)[rank]
        sl = slice(off, off + ln)
        out, lse = sliding_window_attention_sharded(
            q[:, :, sl].contiguous(), k[:, :, sl].contiguous(), v[:, :, sl].contiguous(), case["w"], case["g"],
            case["scale"], seq_len=case["n"], return_lse=True, steps=CpuShardSteps())
        np.save(os.path.join(outdir, f"o{rank}.npy"), out.numpy())
        np.save(os.path.join(outdir, f"l{rank}.npy"), lse.numpy())
    finally:
        dist.destroy_process_group()


CASES = [
    dict(name="two_shards", world=2, seed=11, batch=1, heads=2, n=768, d=64, w=100, g=[0, 5, 383, 384, 700, -1],
         scale=0.125),
    dict(name="three_ragged", world=3, seed=12, batch=2, heads=1, n=700, d=64, w=130, g=[255, 256, 600, 3],
         scale=0.1),
    dict(name="no_globals", world=2, seed=13, batch=1, heads=1, n=512, d=128, w=64, g=[], scale=0.09),
    dict(name="window_zero", world=2, seed=14, batch=1, heads=1, n=256, d=64, w=0, g=[7], scale=0.125),
]


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_sharded_forward_on_gloo_ranks(case, tmp_path):
    world = case["world"]
    mp.spawn(_rank_main, args=(world, _free_port(), case, str(tmp_path)), nprocs=world, join=True)
    out = np.concatenate([np.load(tmp_path / f"o{r}.npy") for r in range(world)], axis=2)
    lse = np.concatenate([np.load(tmp_path / f"l{r}.npy") for r in range(world)], axis=2)
    q, k, v = make_inputs(case["seed"], case["batch"], case["heads"], case["n"], case["d"], torch.bfloat16)
    ref_o, ref_l = swa_oracle.sliding_window_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                                       case["w"], case["g"], case["scale"])
    # float64 arithmetic on both sides: only the fp32 output rounding differs
    assert np.abs(out - ref_o).max() < 1e-5
    assert np.abs(lse - ref_l).max() < 1e-5
