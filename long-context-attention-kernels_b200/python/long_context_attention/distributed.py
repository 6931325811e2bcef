"""Multi-GPU sliding-window + global-token attention over ``torch.distributed``.

Two ways to spread one forward over several GPUs, one process per GPU:

* **Head shards** need no exchange: (batch, head) slices are independent, so each rank
  calls :func:`long_context_attention.sliding_window_attention` on its own heads.
  :func:`head_shard` gives a rank's slice.
* **Sequence shards** (:func:`sliding_window_attention_sharded`) cut one sequence into
  contiguous token shards, one per rank (:func:`shard_bounds`).  A rank's rows need
  `window` keys from each neighbouring shard (the halo) and the global tokens' K / V
  rows, and a global row needs every shard's keys.  The forward runs as

    1. ``lca_swa_shard_prepare``: compact copies of the global rows this shard holds and
       the halo blocks for the neighbours;
    2. exchange, one point-to-point group: each rank sends its global rows to all others
       (every rank then holds all of them) and its halo blocks to ranks r-1 and r+1;
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
(the CPU tests run it on ``gloo`` ranks that way).  :class:`ShardedAttention` sets a
problem up once and can capture the whole step, exchanges included, in a CUDA graph.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Sequence

import torch
import torch.distributed as dist

from ._native import CABI, ShardDesc, ShardLayout, cabi

__all__ = ["shard_bounds", "head_shard", "global_row_runs", "ShardSpec", "NativeShardSteps", "ShardedAttention",
           "sliding_window_attention_sharded"]

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
                         self.world_size, self.rank, self.dtype_code, self.scale)


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

    # ---- peer-memory exchange (no collectives library in the step)
    def exchange_peer(self, spec, tokens, peers, nbytes, stream) -> None:
        arr, n = CABI._tokens(tokens)
        st = self.lib.lib.lca_swa_shard_exchange_peer(ctypes.byref(spec.desc()), arr, n, peers, nbytes, stream)
        _check(st, self.lib, "lca_swa_shard_exchange_peer")

    def finish_peer(self, spec, out, lse, tokens, peers, nbytes, stream) -> None:
        arr, n = CABI._tokens(tokens)
        st = self.lib.lib.lca_swa_shard_finish_peer(ctypes.byref(spec.desc()), out.data_ptr(),
                                                    lse.data_ptr() if lse is not None else None, arr, n, peers,
                                                    nbytes, stream)
        _check(st, self.lib, "lca_swa_shard_finish_peer")


class _PeerBuffer:
    """This rank's workspace from lca_peer_alloc, with the other ranks' mapped (the data
    pointer and size are all the compute steps use)."""

    def __init__(self, lib: CABI, nbytes: int, rank: int, world: int, group, device):
        self.lib, self.nbytes, self.rank = lib, nbytes, rank
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        _check(lib.lib.lca_peer_alloc(nbytes, ctypes.byref(ptr), handle), lib, "lca_peer_alloc")
        self.ptr = ptr.value
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
        allh = torch.empty(world * 64, dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(allh, mine, group=group)
        allh = allh.cpu().numpy().reshape(world, 64)
        self.opened = []
        ptrs = []
        for r in range(world):
            if r == rank:
                ptrs.append(self.ptr)
                continue
            h = (ctypes.c_ubyte * 64)(*allh[r].tolist())
            pr = ctypes.c_void_p()
            _check(lib.lib.lca_peer_open(h, ctypes.byref(pr)), lib, "lca_peer_open")
            self.opened.append(pr.value)
            ptrs.append(pr.value)
        self.peers = (ctypes.c_void_p * world)(*ptrs)

    def data_ptr(self) -> int:
        return self.ptr

    def numel(self) -> int:
        return self.nbytes

    def free(self) -> None:
        for pr in self.opened:
            self.lib.lib.lca_peer_close(ctypes.c_void_p(pr))
        self.opened = []
        if self.ptr:
            self.lib.lib.lca_peer_free(ctypes.c_void_p(self.ptr))
            self.ptr = 0


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


def global_row_runs(tokens: Sequence[int], bounds: Sequence[tuple[int, int]]) -> list[tuple[int, int]]:
    """Per rank, the run [lo, hi) of compact global rows (sorted unique tokens) that fall
    in its shard."""
    import bisect

    return [(bisect.bisect_left(tokens, off), bisect.bisect_left(tokens, off + ln)) for off, ln in bounds]


def exchange_p2p(ws: torch.Tensor, lay: ShardLayout, runs, rank: int, world_size: int, group=None) -> None:
    """One point-to-point group: every rank sends the global rows its shard holds to all
    other ranks (into the same offsets of their compact region), and the halo blocks go
    to the neighbours (side 0 of the send region to rank - 1, side 1 to rank + 1; side 0
    of the receive region comes from rank - 1, side 1 from rank + 1)."""
    if world_size == 1:
        return
    ops = []

    def peer(r):
        return r if group is None else dist.get_global_rank(group, r)

    rb, g0 = lay.globals_row_bytes, lay.globals_offset
    if lay.globals_bytes:
        lo, hi = runs[rank]
        for r in range(world_size):
            if r == rank:
                continue
            if hi > lo:
                ops.append(dist.P2POp(dist.isend, ws[g0 + lo * rb:g0 + hi * rb], peer(r), group))
            rlo, rhi = runs[r]
            if rhi > rlo:
                ops.append(dist.P2POp(dist.irecv, ws[g0 + rlo * rb:g0 + rhi * rb], peer(r), group))
    side = lay.halo_side_bytes
    if lay.halo_rows and side:
        send, recv = lay.halo_send_offset, lay.halo_recv_offset
        if rank > 0:
            ops.append(dist.P2POp(dist.isend, ws[send:send + side], peer(rank - 1), group))
            ops.append(dist.P2POp(dist.irecv, ws[recv:recv + side], peer(rank - 1), group))
        if rank < world_size - 1:
            ops.append(dist.P2POp(dist.isend, ws[send + side:send + 2 * side], peer(rank + 1), group))
            ops.append(dist.P2POp(dist.irecv, ws[recv + side:recv + 2 * side], peer(rank + 1), group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


def exchange_rowparts(ws: torch.Tensor, lay: ShardLayout, world_size: int, group=None) -> None:
    """All-gather of every shard's global-row partial, in rank order."""
    if lay.rowpart_bytes == 0:
        return
    src = ws[lay.rowpart_offset:lay.rowpart_offset + lay.rowpart_bytes]
    dst = ws[lay.rowpart_all_offset:lay.rowpart_all_offset + world_size * lay.rowpart_bytes]
    if world_size == 1:
        dst.copy_(src)
    else:
        dist.all_gather_into_tensor(dst, src, group=group)


class ShardedAttention:
    """A sequence-sharded forward of one problem shape on this rank, set up once.

    Holds the shard geometry, the workspace and the output buffers, so a call does only
    the compute steps and the exchanges.  :meth:`capture` records one whole forward
    (kernels and NCCL exchanges) into a CUDA graph over fixed input tensors, and
    :meth:`replay` re-runs it with a single launch: the way to run a shard whose step is
    short enough for host-side launch work to matter.  Outputs live in :attr:`out` (and
    :attr:`lse`) and are overwritten by every call.  All ranks of `group` must build the
    same plan and call it in the same order.

    ``exchange="peer"`` moves the halos, global rows and row partials by NVLink stores
    from the library's own kernels into the other ranks' workspaces (CUDA IPC mappings
    made at construction; one GPU per rank), with bounded waits on counters there, so a
    step runs no collective at all.  ``"nccl"`` (default) uses the process group.  A rank
    that is late or missing makes the others' waits give up after ``LCA_WAIT_TIMEOUT_MS``
    (2 s by default): their step then runs on stale halos and global rows, and the device
    error word says so.  Steps are asynchronous, so the error surfaces only when the host
    looks: :meth:`raise_on_device_error` (or ``check=True`` on a call) does.
    """

    def __init__(self, batch: int, heads: int, seq_len: int, head_dim: int, window_size: int,
                 global_tokens: Sequence[int] = (), scale: float | None = None, dtype=torch.bfloat16, *,
                 group=None, device=None, return_lse: bool = False, steps=None, exchange: str = "nccl"):
        if dist.is_available() and dist.is_initialized():
            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        else:
            if group is not None:
                raise RuntimeError("long_context_attention: a process group was given but torch.distributed "
                                   "is not initialised")
            self.rank, self.world = 0, 1
        if window_size < 0:
            raise RuntimeError("long_context_attention: window_size must be >= 0")
        self.group = group
        self.bounds = shard_bounds(seq_len, self.world)
        off, ln = self.bounds[self.rank]
        w = min(window_size, seq_len)
        if self.world > 1 and w > min(b for _, b in self.bounds):
            raise RuntimeError(f"long_context_attention: window {w} exceeds the shortest shard "
                               f"({min(b for _, b in self.bounds)} tokens); halos come from adjacent shards only")
        if scale is None:
            scale = 1.0 / math.sqrt(head_dim)
        self.tokens = _normalize(global_tokens, seq_len)
        self.runs = global_row_runs(self.tokens, self.bounds)
        self.dtype = dtype
        self.spec = ShardSpec(batch, heads, seq_len, head_dim, int(window_size), self.rank, self.world, off, ln,
                              _dtype_code(dtype), float(scale))
        self.steps = steps if steps is not None else NativeShardSteps()
        self.layout = self.steps.layout(self.spec, len(self.tokens))
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        if exchange not in ("nccl", "peer"):
            raise ValueError("exchange must be 'nccl' or 'peer'")
        self.exchange = exchange if self.world > 1 else "nccl"
        if self.exchange == "peer":
            if steps is not None:
                raise ValueError("the peer exchange runs the native steps only")
            # the peer steps wait on each other across ranks: one GPU per rank
            ids = [None] * self.world
            dist.all_gather_object(ids, str(torch.cuda.get_device_properties(self.device).uuid), group=group)
            if len(set(ids)) != self.world:
                raise RuntimeError("long_context_attention: the peer exchange needs one GPU per rank")
            self.ws = _PeerBuffer(self.steps.lib, self.layout.total_bytes, self.rank, self.world, group,
                                  self.device)
        else:
            self.ws = self.steps.workspace(self.layout.total_bytes, self.device)
        self.out = torch.empty(batch, heads, ln, head_dim, dtype=torch.float32, device=self.device)
        self.lse = torch.empty(batch, heads, ln, dtype=torch.float32, device=self.device) if return_lse else None
        self.graph = None
        self._graph_inputs = None

    @property
    def shard(self) -> tuple[int, int]:
        """(offset, length) of this rank's tokens."""
        return self.spec.offset, self.spec.length

    def _check(self, Q, K, V):
        shape = (self.spec.batch, self.spec.heads, self.spec.length, self.spec.head_dim)
        for name, t in (("Q", Q), ("K", K), ("V", V)):
            if tuple(t.shape) != shape:
                raise RuntimeError(f"long_context_attention: {name} has shape {tuple(t.shape)}; this rank's shard "
                                   f"is {shape}")
            if t.dtype != self.dtype or not t.is_contiguous():
                raise RuntimeError(f"long_context_attention: {name} must be a contiguous {self.dtype} tensor")

    def _run(self, Q, K, V):
        spec, lay, ws = self.spec, self.layout, self.ws
        if self.exchange == "peer":
            stream = torch.cuda.current_stream(self.device).cuda_stream
            self.steps.prepare(spec, Q, K, V, self.tokens, ws)
            self.steps.exchange_peer(spec, self.tokens, ws.peers, ws.nbytes, stream)
            self.steps.forward(spec, Q, K, V, self.out, self.lse, self.tokens, ws)
            self.steps.finish_peer(spec, self.out, self.lse, self.tokens, ws.peers, ws.nbytes, stream)
            return
        self.steps.prepare(spec, Q, K, V, self.tokens, ws)
        exchange_p2p(ws, lay, self.runs, self.rank, self.world, self.group)
        self.steps.forward(spec, Q, K, V, self.out, self.lse, self.tokens, ws)
        exchange_rowparts(ws, lay, self.world, self.group)
        self.steps.finish(spec, self.out, self.lse, self.tokens, ws)

    def __call__(self, Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, check: bool = False):
        """One forward on the current stream; returns :attr:`out` (and :attr:`lse`).
        With ``check=True`` the call synchronises the device afterwards and raises if a
        bounded wait of its kernels gave up (:meth:`raise_on_device_error`)."""
        self._check(Q, K, V)
        self._run(Q, K, V)
        if check:
            self.raise_on_device_error()
        return (self.out, self.lse) if self.lse is not None else self.out

    def raise_on_device_error(self) -> None:
        """Synchronise this rank's device and raise RuntimeError if a kernel's bounded wait
        gave up since the last check (the device error word, read and cleared): for the
        peer exchange, code 5 means another rank's data did not arrive in time, so the
        outputs of the steps since the last check are invalid."""
        from . import raise_on_device_error

        with torch.cuda.device(self.device):
            raise_on_device_error()

    def capture(self, Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, warmup: int = 2) -> None:
        """Record one forward over these input tensors into a CUDA graph (after `warmup`
        eager runs on the capture stream, which also set up the NCCL communicators).
        Later :meth:`replay` calls read whatever Q, K, V then hold."""
        self._check(Q, K, V)
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._run(Q, K, V)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._run(Q, K, V)
        self.graph = g
        self._graph_inputs = (Q, K, V)

    def replay(self):
        """Run the captured forward; returns :attr:`out` (and :attr:`lse`)."""
        if self.graph is None:
            raise RuntimeError("long_context_attention: capture() has not been called")
        self.graph.replay()
        return (self.out, self.lse) if self.lse is not None else self.out

    def release(self) -> None:
        """Drop the captured graph (it holds NCCL work: release it before destroying the
        process group) and, for the peer exchange, unmap the other ranks' workspaces and
        free this one once every rank is done with them (a collective call)."""
        self.graph = None
        self._graph_inputs = None
        if isinstance(self.ws, _PeerBuffer):
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            self.ws.free()
            self.ws = None


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
    ``return_lse``) in new tensors.  Limit: ``min(window_size, seq_len)`` must not exceed
    a shard.  For repeated calls of one shape, :class:`ShardedAttention` avoids the setup.
    """
    B, H, n_loc, d = Q.shape
    world = dist.get_world_size(group)
    if seq_len is None:
        seq_len = n_loc * world
    plan = ShardedAttention(B, H, seq_len, d, window_size, global_tokens, scale, Q.dtype, group=group,
                            device=Q.device, return_lse=return_lse, steps=steps)
    if plan.spec.length != n_loc:
        raise RuntimeError(f"long_context_attention: rank {plan.rank} holds {n_loc} tokens; "
                           f"shard_bounds({seq_len}, {world}) gives it {plan.spec.length}")
    return plan(Q, K, V)
