"""Multi-GPU sliding-window + global-token attention over ``torch.distributed``.

Two ways to spread one forward over several GPUs, one process per GPU:

* **Head shards** need no exchange: (batch, head) slices are independent, so each rank
  calls :func:`long_context_attention.sliding_window_attention` on its own heads.
  :func:`head_shard` gives a rank's slice.
* **Sequence shards** (:func:`sliding_window_attention_sharded`) cut one sequence into
  contiguous token shards, one per rank (:func:`shard_bounds`).  A rank's rows need
  `window` keys from each neighbouring shard (the halo) and the global tokens' K / V
  rows, and a global row needs every shard's keys.  The forward runs as

    1. ``lca_swa_shard_prepare``: compact global rows this shard owns (zeros for the
       others) and the halo blocks for the neighbours;
    2. exchange: sum all-reduce of the compact global rows (every rank then holds all
       of them) and point-to-point send / receive of the halos with ranks r-1 and r+1;
    3. ``lca_swa_shard_forward``: every local row, plus this shard's partial result
       (normalised O and log-sum-exp) for each global row over its own keys;
    4. exchange: all-gather of the per-shard global-row partials;
    5. ``lca_swa_shard_finish``: log-sum-exp merge of those partials into the global rows
       this shard owns.

  The exchanges use the process group's backend (NCCL between GPUs).  All ranks take the
  same collective steps in the same order.  The reference has no multi-GPU path; the
  result equals the single-GPU forward of the whole sequence.

The compute steps come from the native library; the ``steps`` argument exists so that
the exchange logic can be driven by another implementation of the same three steps
(the CPU tests run it on ``gloo`` ranks that way).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Sequence

import torch
import torch.distributed as dist

from ._native import CABI, ShardDesc, ShardLayout, cabi

__all__ = ["shard_bounds", "head_shard", "ShardSpec", "NativeShardSteps", "sliding_window_attention_sharded"]

_TILE = 128


def shard_bounds(seq_len: int, world_size: int) -> list[tuple[int, int]]:
    """Contiguous token shards ``(offset, length)`` of a sequence, rank order.

    Every shard but the last holds the same multiple of 128 tokens (the kernels align
    key tiles to shard starts); the last holds the rest.  Raises ValueError when the
    sequence is too short to give every rank at least one token under that rule.
    """
    if world_size < 1:
        raise ValueError("world_size must be >= 1")
    if seq_len < 1:
        raise ValueError("seq_len must be >= 1")
    if world_size == 1:
        return [(0, seq_len)]
    per = -(-seq_len // world_size)
    per = -(-per // _TILE) * _TILE
    if per * (world_size - 1) >= seq_len:
        raise ValueError(f"seq_len {seq_len} is too short for {world_size} shards of a multiple of {_TILE} tokens")
    return [(r * per, per if r < world_size - 1 else seq_len - per * (world_size - 1)) for r in range(world_size)]


def head_shard(num_heads: int, world_size: int, rank: int) -> slice:
    """Heads of `rank` when `num_heads` are split as evenly as possible over the ranks."""
    base, extra = divmod(num_heads, world_size)
    lo = rank * base + min(rank, extra)
    return slice(lo, lo + base + (1 if rank < extra else 0))


@dataclass(frozen=True)
class ShardSpec:
    """One rank's view of a sequence-sharded problem."""

    batch: int
    heads: int
    seq_len: int
    head_dim: int
    window: int
    rank: int
    world_size: int
    offset: int
    length: int
    dtype_code: int
    scale: float

    def desc(self) -> ShardDesc:
        return ShardDesc(self.batch, self.heads, self.seq_len, self.head_dim, self.window, self.offset, self.length,
                         self.world_size, self.dtype_code, self.scale)


def _check(st: int, lib: CABI, what: str) -> None:
    if st == CABI.OK:
        return
    msg = f"{what}: {lib.lib.lca_status_string(st).decode()}: {lib.last_error()}"
    if st == CABI.ERR_INDEX:
        raise IndexError(msg)
    raise RuntimeError(msg)


class NativeShardSteps:
    """The three compute steps of a shard's forward, on the current CUDA stream, through
    the C ABI of ``liblca_b200.so``."""

    def __init__(self):
        self.lib = cabi()

    def layout(self, spec: ShardSpec, num_unique_global: int) -> ShardLayout:
        st, lay = self.lib.shard_layout(spec.desc(), num_unique_global)
        _check(st, self.lib, "lca_swa_shard_layout")
        return lay

    def workspace(self, nbytes: int, device) -> torch.Tensor:
        # 256-byte aligned (the caching allocator aligns to 512 bytes)
        return torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)

    def _stream(self, t: torch.Tensor) -> int:
        return torch.cuda.current_stream(t.device).cuda_stream

    def prepare(self, spec, q, k, v, tokens, ws) -> None:
        st = self.lib.shard_prepare(spec.desc(), q.data_ptr(), k.data_ptr(), v.data_ptr(), tokens, ws.data_ptr(),
                                    ws.numel(), self._stream(q))
        _check(st, self.lib, "lca_swa_shard_prepare")

    def forward(self, spec, q, k, v, out, lse, tokens, ws) -> None:
        st = self.lib.shard_forward(spec.desc(), q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                    lse.data_ptr() if lse is not None else None, tokens, ws.data_ptr(), ws.numel(),
                                    self._stream(q))
        _check(st, self.lib, "lca_swa_shard_forward")

    def finish(self, spec, out, lse, tokens, ws) -> None:
        st = self.lib.shard_finish(spec.desc(), out.data_ptr(), lse.data_ptr() if lse is not None else None, tokens,
                                   ws.data_ptr(), ws.numel(), self._stream(out))
        _check(st, self.lib, "lca_swa_shard_finish")


def _dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float16:
        return CABI.DTYPE_F16
    if dtype == torch.bfloat16:
        return CABI.DTYPE_BF16
    raise RuntimeError(f"long_context_attention: dtype {dtype} is not supported (float16 or bfloat16)")


def _normalize(tokens: Sequence[int], seq_len: int) -> list[int]:
    out = set()
    for t in tokens:
        t = int(t)
        if t < -seq_len or t >= seq_len:
            raise IndexError(f"index {t} is out of bounds for dimension 0 with size {seq_len}")
        out.add(t + seq_len if t < 0 else t)
    return sorted(out)


def exchange_globals(ws: torch.Tensor, lay: ShardLayout, dtype: torch.dtype, group=None) -> None:
    """Sum all-reduce of the compact global rows (each rank holds its own, zeros elsewhere)."""
    if lay.globals_bytes == 0:
        return
    buf = ws[lay.globals_offset:lay.globals_offset + lay.globals_bytes].view(dtype)
    dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)


def exchange_halos(ws: torch.Tensor, lay: ShardLayout, rank: int, world_size: int, group=None) -> None:
    """Halo blocks: side 0 of the send region goes to rank - 1 and side 1 to rank + 1; side
    0 of the receive region comes from rank - 1 and side 1 from rank + 1."""
    side = lay.halo_side_bytes
    if lay.halo_rows == 0 or side == 0 or world_size == 1:
        return
    send, recv = lay.halo_send_offset, lay.halo_recv_offset
    ops = []

    def peer(r):
        return r if group is None else dist.get_global_rank(group, r)

    if rank > 0:
        ops.append(dist.P2POp(dist.isend, ws[send:send + side], peer(rank - 1), group))
        ops.append(dist.P2POp(dist.irecv, ws[recv:recv + side], peer(rank - 1), group))
    if rank < world_size - 1:
        ops.append(dist.P2POp(dist.isend, ws[send + side:send + 2 * side], peer(rank + 1), group))
        ops.append(dist.P2POp(dist.irecv, ws[recv + side:recv + 2 * side], peer(rank + 1), group))
    for req in dist.batch_isend_irecv(ops):
        req.wait()


def exchange_rowparts(ws: torch.Tensor, lay: ShardLayout, world_size: int, group=None) -> None:
    """All-gather of every shard's global-row partial, in rank order."""
    if lay.rowpart_bytes == 0:
        return
    src = ws[lay.rowpart_offset:lay.rowpart_offset + lay.rowpart_bytes]
    dst = ws[lay.rowpart_all_offset:lay.rowpart_all_offset + world_size * lay.rowpart_bytes]
    dist.all_gather_into_tensor(dst, src, group=group)


def sliding_window_attention_sharded(
    Q: torch.Tensor,
    K: torch.Tensor,
    V: torch.Tensor,
    window_size: int,
    global_tokens: Sequence[int] = (),
    scale: float | None = None,
    *,
    seq_len: int | None = None,
    group=None,
    return_lse: bool = False,
    steps=None,
):
    """Sequence-sharded Longformer attention forward; call it on every rank of `group`.

    Q, K, V: this rank's shard ``[batch, heads, shard_len, head_dim]`` (fp16 / bf16,
    contiguous) of a sequence of `seq_len` tokens split as :func:`shard_bounds` gives.
    `seq_len` defaults to ``shard_len * world_size`` (equal shards).  `window_size`,
    `global_tokens` (indices into the whole sequence) and `scale` mean what they mean for
    :func:`long_context_attention.sliding_window_attention`, and are the same on every
    rank.  Returns this shard's fp32 output rows (and their log-sum-exp with
    ``return_lse``).  Limit: ``min(window_size, seq_len)`` must not exceed a shard.
    """
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    B, H, n_loc, d = Q.shape
    if K.shape != Q.shape or V.shape != Q.shape:
        raise RuntimeError("long_context_attention: Q, K and V must have the same shape")
    if not (Q.is_contiguous() and K.is_contiguous() and V.is_contiguous()):
        raise RuntimeError("long_context_attention: Q, K and V must be contiguous")
    if Q.dtype != K.dtype or Q.dtype != V.dtype:
        raise RuntimeError("long_context_attention: Q, K and V must share one dtype")
    if window_size < 0:
        raise RuntimeError("long_context_attention: window_size must be >= 0")
    if seq_len is None:
        seq_len = n_loc * world
    bounds = shard_bounds(seq_len, world)
    offset, length = bounds[rank]
    if length != n_loc:
        raise RuntimeError(f"long_context_attention: rank {rank} holds {n_loc} tokens; shard_bounds({seq_len}, {world}) "
                           f"gives it {length}")
    w = min(window_size, seq_len)
    if world > 1 and w > min(ln for _, ln in bounds):
        raise RuntimeError(f"long_context_attention: window {w} exceeds the shortest shard "
                           f"({min(ln for _, ln in bounds)} tokens); halos come from adjacent shards only")
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    tokens = _normalize(global_tokens, seq_len)
    spec = ShardSpec(B, H, seq_len, d, int(window_size), rank, world, offset, length, _dtype_code(Q.dtype),
                     float(scale))
    steps = steps if steps is not None else NativeShardSteps()
    lay = steps.layout(spec, len(tokens))
    ws = steps.workspace(lay.total_bytes, Q.device)
    out = torch.empty(B, H, n_loc, d, dtype=torch.float32, device=Q.device)
    lse = torch.empty(B, H, n_loc, dtype=torch.float32, device=Q.device) if return_lse else None

    steps.prepare(spec, Q, K, V, tokens, ws)
    exchange_globals(ws, lay, Q.dtype, group)
    exchange_halos(ws, lay, rank, world, group)
    steps.forward(spec, Q, K, V, out, lse, tokens, ws)
    exchange_rowparts(ws, lay, world, group)
    steps.finish(spec, out, lse, tokens, ws)
    return (out, lse) if return_lse else out
