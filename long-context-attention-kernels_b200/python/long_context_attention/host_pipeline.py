"""Attention forward for inputs and outputs that live in (pinned) host memory.

A caller whose Q, K, V sit in host memory pays the PCIe transfers on top of the kernels:
for the 16-head 64K workload 402 MB go to the GPU and 268 MB of fp32 output come back,
about 12 ms one after the other, against ~0.5 ms of compute.  Heads are independent,
so :func:`sliding_window_attention_from_host` cuts the flattened batch x heads into
chunks and runs three CUDA streams in a pipeline: the host-to-device copy of chunk i+1
and the device-to-host copy of chunk i-1 overlap the forward of chunk i (PCIe is full
duplex, and the two directions use separate copy engines).  The step is then bounded by
the larger of the two transfer directions.

No counterpart in the reference, whose entry point takes device tensors only
(python/long_context_attention/__init__.py:56-82); the forward of each chunk is the same
C-ABI call the device-tensor entry point makes.
"""
from __future__ import annotations

import math
from typing import Sequence

import torch

from ._native import CABI, cabi

__all__ = ["sliding_window_attention_from_host"]


def _check_host(name: str, t: torch.Tensor, like: torch.Tensor | None) -> None:
    if t.is_cuda:
        raise RuntimeError(f"long_context_attention: {name} must be a host tensor here (got a CUDA tensor)")
    if t.dim() != 4:
        raise RuntimeError(f"long_context_attention: {name} must be [batch, heads, seq_len, head_dim]")
    if not t.is_contiguous():
        raise RuntimeError(f"long_context_attention: {name} must be contiguous")
    if like is not None and (t.shape != like.shape or t.dtype != like.dtype):
        raise RuntimeError("long_context_attention: Q, K and V must have the same shape and dtype")


def sliding_window_attention_from_host(
    Q: torch.Tensor,
    K: torch.Tensor,
    V: torch.Tensor,
    window_size: int,
    global_tokens: Sequence[int] = (),
    scale: float | None = None,
    *,
    out: torch.Tensor | None = None,
    chunks: int | None = None,
    device=None,
) -> torch.Tensor:
    """Forward of host-resident Q, K, V ``[batch, heads, seq_len, head_dim]`` (fp16 or
    bf16, contiguous; pinned memory makes the copies asynchronous and is what the overlap
    needs) on a B200, returning the fp32 output in host memory (`out`, or a new pinned
    tensor).

    `window_size`, `global_tokens` and `scale` mean what they mean for
    :func:`long_context_attention.sliding_window_attention`, and the results match it
    within the same tolerances (each chunk is its own call: the split of the global
    rows' keys and, for bf16, the choice of the fp16 copy of V are made per chunk, so
    the rounding can differ).  `chunks` (default ``min(batch * heads, 8)``) is how many pieces the flattened
    batch x heads is cut into.  The call returns once the output has arrived in host
    memory (it synchronises the streams it uses, not the whole device).
    """
    _check_host("Q", Q, None)
    _check_host("K", K, Q)
    _check_host("V", V, Q)
    if Q.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("long_context_attention: Q, K, V must be fp16 or bf16")
    B, H, n, d = Q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    if window_size < 0:
        raise RuntimeError(f"long_context_attention: window_size must be >= 0 (got {window_size})")
    if out is None:
        out = torch.empty((B, H, n, d), dtype=torch.float32, pin_memory=True)
    elif out.shape != (B, H, n, d) or out.dtype != torch.float32 or out.is_cuda or not out.is_contiguous():
        raise RuntimeError("long_context_attention: out must be a contiguous fp32 host tensor of Q's shape")
    bh = B * H
    if bh == 0 or n == 0:
        return out
    lib = cabi()
    tokens = [int(t) for t in global_tokens]
    st, gl = lib.normalize(tokens, n)
    if st != CABI.OK:
        msg = f"global_tokens: {lib.last_error()}"
        raise IndexError(msg) if st == CABI.ERR_INDEX else RuntimeError(msg)
    dt = CABI.DTYPE_BF16 if Q.dtype == torch.bfloat16 else CABI.DTYPE_F16
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    nchunks = max(1, min(bh, chunks if chunks is not None else 8))
    per = -(-bh // nchunks)
    bounds = [(c * per, min(bh, (c + 1) * per)) for c in range(nchunks) if c * per < bh]

    q3, k3, v3, o3 = (t.view(bh, n, d) for t in (Q, K, V, out))
    ws_bytes = 0
    for m in {hi - lo for lo, hi in bounds}:  # the split of the global rows' keys depends on the head count
        st, need = lib.workspace_size(1, m, n, d, window_size, len(gl), dt)
        if st != CABI.OK:
            raise RuntimeError(f"workspace size: {lib.last_error()}")
        ws_bytes = max(ws_bytes, need)
    with torch.cuda.device(dev):
        main = torch.cuda.current_stream(dev)
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        # two buffer sets: chunk i uses set i % 2
        qd = [torch.empty((per, n, d), dtype=Q.dtype, device=dev) for _ in range(2)]
        kd = [torch.empty_like(qd[0]) for _ in range(2)]
        vd = [torch.empty_like(qd[0]) for _ in range(2)]
        od = [torch.empty((per, n, d), dtype=torch.float32, device=dev) for _ in range(2)]
        ws = [torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev) for _ in range(2)]
        loaded = [torch.cuda.Event() for _ in bounds]
        computed = [torch.cuda.Event() for _ in bounds]
        stored = [torch.cuda.Event() for _ in bounds]
        s_in.wait_stream(main)
        s_out.wait_stream(main)
        for i, (lo, hi) in enumerate(bounds):
            b = i % 2
            m = hi - lo
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(computed[i - 2])  # the forward of chunk i-2 has read set b
                qd[b][:m].copy_(q3[lo:hi], non_blocking=True)
                kd[b][:m].copy_(k3[lo:hi], non_blocking=True)
                vd[b][:m].copy_(v3[lo:hi], non_blocking=True)
                loaded[i].record(s_in)
            main.wait_event(loaded[i])
            if i >= 2:
                main.wait_event(stored[i - 2])  # set b's output has gone back to the host
            st = lib.forward(qd[b].data_ptr(), kd[b].data_ptr(), vd[b].data_ptr(), od[b].data_ptr(), None, dt, 1, m,
                             n, d, window_size, float(scale), tokens, ws[b].data_ptr(), ws_bytes, main.cuda_stream)
            if st != CABI.OK:
                msg = f"sliding_window_attention_from_host: {lib.last_error()}"
                raise IndexError(msg) if st == CABI.ERR_INDEX else RuntimeError(msg)
            computed[i].record(main)
            with torch.cuda.stream(s_out):
                s_out.wait_event(computed[i])
                o3[lo:hi].copy_(od[b][:m], non_blocking=True)
                stored[i].record(s_out)
        main.wait_event(stored[-1])
        for t in qd + kd + vd + od + ws:
            t.record_stream(s_in)
            t.record_stream(s_out)
        stored[-1].synchronize()
    return out
