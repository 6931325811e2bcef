"""Sliding-window + global-token (Longformer-style) attention forward for NVIDIA B200.

Drop-in for the reference package ``long_context_attention``
(python/long_context_attention/__init__.py): same module name, same public function
``sliding_window_attention(Q, K, V, window_size, global_tokens=(), scale=None,
force_reference=False)`` and the same helper name ``_reference_sliding_window_attention``.

Dispatch differs from the reference on purpose: CUDA tensors always go to the sm_100a
kernels (``long_context_attention_kernels`` -> ``liblca_b200.so``), and a missing or
unloadable native build raises instead of silently falling back to the dense O(n^2)
computation.  The dense computation runs only when asked for explicitly
(``force_reference=True``), which is also how CPU tensors are handled.
"""
from __future__ import annotations

import math
from typing import Sequence

import torch

from ._native import extension, native_error

__all__ = ["sliding_window_attention", "sliding_window_attention_with_lse", "sliding_window_attention_varlen",
           "sliding_window_attention_backward"]


def _reference_sliding_window_attention(
    Q: torch.Tensor,
    K: torch.Tensor,
    V: torch.Tensor,
    window_size: int,
    global_tokens: Sequence[int],
    scale: float,
) -> torch.Tensor:
    """Dense Longformer-mask attention (the reference's definition, O(n^2) memory).

    Same mask and arithmetic as python/long_context_attention/__init__.py:24-53: key j
    is visible to query i iff |i - j| <= window_size, or j or i is a global token;
    fp32 scores, masked softmax, fp32 output.  Reached only through
    ``force_reference=True`` or a direct call; never used as a fallback.
    """
    seq_len = Q.shape[2]
    device = Q.device
    idx = torch.arange(seq_len, device=device)
    band = (idx[:, None] - idx[None, :]).abs() <= window_size
    is_global = torch.zeros(seq_len, dtype=torch.bool, device=device)
    if len(global_tokens) > 0:
        is_global[list(global_tokens)] = True
    visible = band | is_global[None, :] | is_global[:, None]
    scores = torch.einsum("bhqd,bhkd->bhqk", Q.float(), K.float()) * scale
    scores = scores.masked_fill(~visible[None, None, :, :], float("-inf"))
    return torch.einsum("bhqk,bhkd->bhqd", torch.softmax(scores, dim=-1), V.float())


def _dense_causal_attention(Q, K, V, window_size, global_tokens, scale, dilation: int = 1, causal: bool = True):
    """The dense definition above intersected with j <= i (``causal=True`` together with
    ``force_reference=True``): the reference's mask, then its upper triangle removed; with
    ``dilation`` > 1 the band keeps the keys i + dilation * t, |t| <= window_size."""
    seq_len = Q.shape[2]
    idx = torch.arange(seq_len, device=Q.device)
    diff = idx[:, None] - idx[None, :]
    band = diff.abs() <= window_size * dilation
    if dilation > 1:
        band &= diff % dilation == 0
    is_global = torch.zeros(seq_len, dtype=torch.bool, device=Q.device)
    if len(global_tokens) > 0:
        is_global[list(global_tokens)] = True
    visible = band | is_global[None, :] | is_global[:, None]
    if causal:
        visible &= idx[None, :] <= idx[:, None]
    scores = torch.einsum("bhqd,bhkd->bhqk", Q.float(), K.float()) * scale
    scores = scores.masked_fill(~visible[None, None, :, :], float("-inf"))
    return torch.einsum("bhqk,bhkd->bhqd", torch.softmax(scores, dim=-1), V.float())


def _head_windows(window_size, heads: int):
    """(radius, per-head radii or []): an int applies to every head; a sequence (or 1-D
    tensor) gives one radius per head."""
    if isinstance(window_size, torch.Tensor):
        window_size = window_size.tolist()
    if isinstance(window_size, (list, tuple)):
        radii = [int(w) for w in window_size]
        if len(radii) != heads:
            raise ValueError(f"window_size per head needs {heads} radii, got {len(radii)}")
        return max(radii, default=0), radii
    return int(window_size), []


def _dense(Q, K, V, window_size, global_tokens, scale, causal: bool, dilation: int = 1):
    """The dense definitions for ``force_reference=True``: the reference's (or its causal or
    dilated form), head by head when the heads have radii of their own."""
    if causal or dilation > 1:
        def dense(q, k, v, w, g, sc):
            return _dense_causal_attention(q, k, v, w, g, sc, dilation=dilation, causal=causal)
    else:
        dense = _reference_sliding_window_attention
    _, radii = _head_windows(window_size, Q.shape[1])
    if not radii:
        return dense(Q, K, V, int(window_size), global_tokens, scale)
    return torch.cat([dense(Q[:, h:h + 1], K[:, h:h + 1], V[:, h:h + 1], radii[h], global_tokens, scale)
                      for h in range(Q.shape[1])], dim=1)


def _token_major(layout: str) -> bool:
    if layout not in ("bhnd", "bnhd"):
        raise ValueError(f"layout must be 'bhnd' or 'bnhd', got {layout!r}")
    return layout == "bnhd"


def _prepare(Q: torch.Tensor, window_size, global_tokens: Sequence[int], scale, token_major: bool = False):
    if scale is None:
        scale = 1.0 / math.sqrt(Q.shape[-1])
    if not Q.is_cuda:
        raise RuntimeError(
            "long_context_attention: Q, K, V must be CUDA tensors on a B200 (sm_100a) GPU; "
            "pass force_reference=True for the dense CPU definition"
        )
    tokens = [int(t) for t in global_tokens]
    window, radii = _head_windows(window_size, Q.shape[2] if token_major else Q.shape[1])
    return float(scale), window, tokens, radii


def sliding_window_attention(
    Q: torch.Tensor,
    K: torch.Tensor,
    V: torch.Tensor,
    window_size: int,
    global_tokens: Sequence[int] = (),
    scale: float | None = None,
    force_reference: bool = False,
    out_dtype: torch.dtype | None = None,
    causal: bool = False,
    dilation: int = 1,
    layout: str = "bhnd",
) -> torch.Tensor:
    """Longformer-style sparse attention forward.

    Q, K, V: [batch, heads, seq_len, head_dim], fp16 or bf16, CUDA, contiguous,
    head_dim 64 or 128.  window_size: band radius (|i - j| <= window_size is visible), or one
    radius per head (a sequence of ``heads`` ints; an addition to the reference's int).
    global_tokens: token indices with full rows and columns (negative indices count from
    the end; duplicates are harmless).  scale defaults to 1/sqrt(head_dim).
    Returns a new fp32 tensor [batch, heads, seq_len, head_dim] on Q's device, computed
    on the current CUDA stream.  ``out_dtype`` (an addition; the reference always returns
    fp32) may be torch.float16 or torch.bfloat16: the same fp32-accumulated result,
    rounded to that type by the kernel, with half the output bytes.  ``causal=True`` (also
    an addition) keeps only keys j <= i: the band becomes [i - window_size, i], a global
    key is seen by the rows at or after it, a global row sees the keys up to itself.
    ``dilation`` > 1 (also an addition) keeps, of the band, the keys i + dilation * t with
    |t| <= window_size (seq_len must be a multiple of the dilation; not with causal).
    ``layout="bnhd"`` (also an addition) takes Q, K, V as [batch, seq_len, heads, head_dim],
    the layout of a fused QKV projection's output, without a transpose, and returns O in the
    same layout (not with dilation).
    """
    tm = _token_major(layout)
    if force_reference:
        if scale is None:
            scale = 1.0 / math.sqrt(Q.shape[-1])
        if tm:
            Q, K, V = (t.transpose(1, 2) for t in (Q, K, V))
        out = _dense(Q, K, V, window_size, global_tokens, scale, causal, int(dilation))
        if tm:
            out = out.transpose(1, 2).contiguous()
        return out if out_dtype in (None, torch.float32) else out.to(out_dtype)
    scale, window_size, tokens, radii = _prepare(Q, window_size, global_tokens, scale, tm)
    base = out_dtype in (None, torch.float32) and not causal and not radii and dilation == 1 and not tm
    if torch.is_grad_enabled() and (Q.requires_grad or K.requires_grad or V.requires_grad):
        if not base:
            raise NotImplementedError(
                "long_context_attention: the backward covers fp32 output, one radius, no causal mask, no "
                "dilation and the [batch, heads, seq_len, head_dim] layout")
        return _SlidingWindowAttentionFn.apply(Q, K, V, window_size, tokens, scale)
    if base:
        return extension().sliding_window_attention_forward_list(Q, K, V, window_size, tokens, scale)
    return extension().sliding_window_attention_forward_ex(Q, K, V, window_size, tokens, scale,
                                                           out_dtype or torch.float32, bool(causal), False,
                                                           radii, int(dilation), [], tm)[0]


class _SlidingWindowAttentionFn(torch.autograd.Function):
    """Forward through the sm_100a kernels keeping O and LSE; backward through
    lca_swa_backward (gradients computed in fp32, returned in the inputs' types)."""

    @staticmethod
    def forward(ctx, Q, K, V, window_size, tokens, scale):
        out, lse = extension().sliding_window_attention_forward_lse(Q, K, V, window_size, tokens, scale)
        ctx.save_for_backward(Q, K, V, out, lse)
        ctx.args = (window_size, tokens, scale)
        return out

    @staticmethod
    def backward(ctx, dO):
        Q, K, V, out, lse = ctx.saved_tensors
        window_size, tokens, scale = ctx.args
        dq, dk, dv = extension().sliding_window_attention_backward(
            Q, K, V, out, lse, dO.to(torch.float32).contiguous(), window_size, tokens, scale)
        return dq.to(Q.dtype), dk.to(K.dtype), dv.to(V.dtype), None, None, None


def sliding_window_attention_backward(
    Q: torch.Tensor,
    K: torch.Tensor,
    V: torch.Tensor,
    O: torch.Tensor,
    LSE: torch.Tensor,
    dO: torch.Tensor,
    window_size: int,
    global_tokens: Sequence[int] = (),
    scale: float | None = None,
):
    """Gradients ``(dQ, dK, dV)`` (fp32, Q's shape) of the attention with respect to Q, K, V.

    O and LSE are what :func:`sliding_window_attention_with_lse` returned for the same
    arguments, dO the gradient of the loss with respect to O.  No counterpart in the
    reference (its roadmap's first open item, README.md:113).  ``sliding_window_attention``
    calls this through autograd when Q, K or V requires grad.
    """
    scale, window_size, tokens, radii = _prepare(Q, window_size, global_tokens, scale)
    if radii:
        raise NotImplementedError("long_context_attention: the backward takes one radius")
    dq, dk, dv = extension().sliding_window_attention_backward(Q, K, V, O, LSE, dO.to(torch.float32).contiguous(),
                                                               window_size, tokens, scale)
    return dq, dk, dv


def sliding_window_attention_with_lse(
    Q: torch.Tensor,
    K: torch.Tensor,
    V: torch.Tensor,
    window_size: int,
    global_tokens: Sequence[int] = (),
    scale: float | None = None,
    out_dtype: torch.dtype | None = None,
    causal: bool = False,
    dilation: int = 1,
    layout: str = "bhnd",
):
    """As :func:`sliding_window_attention`, also returning the per-row log-sum-exp.

    Returns ``(O, LSE)`` with LSE [batch, heads, seq_len] fp32, the natural log of the
    sum of exp(scale * q.k) over each row's visible keys (the quantity a backward pass
    or a cross-shard merge needs).  No counterpart in the reference.
    """
    tm = _token_major(layout)
    scale, window_size, tokens, radii = _prepare(Q, window_size, global_tokens, scale, tm)
    if out_dtype in (None, torch.float32) and not causal and not radii and dilation == 1 and not tm:
        out, lse = extension().sliding_window_attention_forward_lse(Q, K, V, window_size, tokens, scale)
    else:
        out, lse = extension().sliding_window_attention_forward_ex(Q, K, V, window_size, tokens, scale,
                                                                   out_dtype or torch.float32, bool(causal), True,
                                                                   radii, int(dilation), [], tm)
    return out, lse


def sliding_window_attention_varlen(
    Q: torch.Tensor,
    K: torch.Tensor,
    V: torch.Tensor,
    cu_seqlens: Sequence[int],
    window_size,
    global_tokens: Sequence[int] = (),
    scale: float | None = None,
    out_dtype: torch.dtype | None = None,
    causal: bool = False,
    return_lse: bool = False,
    layout: str = "bhnd",
):
    """Packed variable-length sequences (no counterpart in the reference).

    Q, K, V: [1, heads, total_len, head_dim] (or [1, total_len, heads, head_dim] with
    ``layout="bnhd"``) with sequence s in rows ``[cu_seqlens[s], cu_seqlens[s + 1])`` (host
    offsets from 0 to total_len, at most 512 sequences).  Each sequence is attended on its own: its band, global keys and global
    rows stay inside it, and ``global_tokens`` is indexed within each sequence as the
    reference indexes one sequence.  Returns O (and LSE with ``return_lse``).
    """
    tm = _token_major(layout)
    scale, window_size, tokens, radii = _prepare(Q, window_size, global_tokens, scale, tm)
    cu = [int(x) for x in (cu_seqlens.tolist() if isinstance(cu_seqlens, torch.Tensor) else cu_seqlens)]
    res = extension().sliding_window_attention_forward_ex(Q, K, V, window_size, tokens, scale,
                                                          out_dtype or torch.float32, bool(causal), bool(return_lse),
                                                          radii, 1, cu, tm)
    return (res[0], res[1]) if return_lse else res[0]


# Values of the device-side error word (include/lca.h, LCA_DEVERR_*).
DEVICE_ERRORS = {
    1: "main kernel: the TMA producer waited too long for a free slot",
    2: "main kernel: an MMA issuer waited too long for data or P",
    3: "main kernel: a softmax warp waited too long for S or O",
    4: "main kernel: waiting for its own copies at exit took too long",
    5: "peer exchange: another rank's halos, global rows or row partials did not arrive in time",
    6: "backward kernel: waited too long for a tile or an MMA",
}


def device_error() -> int:
    """Read and clear the device-side error word (synchronises the current device)."""
    return native_error()


def raise_on_device_error() -> None:
    """Synchronise the current device, read and clear its device-side error word, and
    raise RuntimeError if a kernel's bounded wait gave up since the last check.  Such a
    kernel stops its own work and returns instead of hanging, so the results of the calls
    since the last check are not to be used."""
    code = native_error()
    if code:
        raise RuntimeError(f"long_context_attention: device error {code} "
                           f"({DEVICE_ERRORS.get(code, 'unknown code')}); results since the last check are invalid")
