"""CPU oracle for the sliding-window + global-token attention forward.

TEST INFRASTRUCTURE ONLY.  This module is the checker: only tests/, the smoke check in
__graft_entry__.py and bench.py's CPU-baseline arm may import it.  The product path
(long_context_attention -> liblca_b200.so) never calls it.

It restates, in numpy, the reference's dense Longformer-mask implementation
``_reference_sliding_window_attention`` (python/long_context_attention/__init__.py:24-53)
row block by row block, so that it also runs at sequence lengths where the dense
[n, n] score matrix would not fit:

* mask (``__init__.py:39-47``): key j visible to query i iff |i - j| <= window_size, or
  j is a global token, or i is a global token;
* global-token list (``__init__.py:42-44``): ``global_mask[list(global_tokens)] = True``,
  i.e. negative indices wrap, duplicates are idempotent, out-of-range raises IndexError;
* arithmetic (``__init__.py:49-53``): scores = (Q K^T) * scale on float inputs,
  masked_fill(-inf), softmax over keys, times V.  The reference does this in fp32; the
  oracle defaults to fp64 so its own rounding sits far below the tolerances it checks.

It additionally returns the natural-log log-sum-exp of each row's visible scaled scores
(the reference computes it implicitly inside softmax), and takes `causal=True` for the
one-sided variant this package adds (no counterpart in the reference): the reference's
mask intersected with j <= i (every row keeps at least its own key).

Parity of this restatement is pinned against outputs of the reference itself: see
tests/golden/make_golden.py (generates fixtures by importing the reference) and
tests/test_oracle.py.
"""
from __future__ import annotations

from typing import Sequence

import numpy as np


def normalize_global_tokens(global_tokens: Sequence[int], seq_len: int) -> np.ndarray:
    """Sorted unique global indices under the reference's indexing rules
    (python/long_context_attention/__init__.py:42-44)."""
    out = set()
    for t in global_tokens:
        t = int(t)
        if t < -seq_len or t >= seq_len:
            raise IndexError(f"index {t} is out of bounds for dimension 0 with size {seq_len}")
        out.add(t + seq_len if t < 0 else t)
    return np.asarray(sorted(out), dtype=np.int64)


def visible_rows(rows: np.ndarray, seq_len: int, window_size: int, global_idx: np.ndarray,
                 causal: bool = False, dilation: int = 1) -> np.ndarray:
    """Boolean [len(rows), seq_len] mask rows (python/long_context_attention/__init__.py:39-47),
    intersected with j <= i when `causal`; with `dilation` > 1 the band keeps the keys
    i + dilation * t, |t| <= window_size."""
    rows = np.asarray(rows, dtype=np.int64)
    keys = np.arange(seq_len, dtype=np.int64)
    diff = rows[:, None] - keys[None, :]
    mask = np.abs(diff) <= window_size * dilation
    if dilation > 1:
        mask &= diff % dilation == 0
    is_global = np.zeros(seq_len, dtype=bool)
    if global_idx.size:
        is_global[global_idx] = True
    mask |= is_global[None, :]
    mask |= is_global[rows][:, None]
    if causal:
        mask &= keys[None, :] <= rows[:, None]
    return mask


def sliding_window_attention(Q, K, V, window_size: int, global_tokens: Sequence[int], scale: float,
                             rows: Sequence[int] | None = None, dtype=np.float64, block_rows: int = 256,
                             causal: bool = False, dilation: int = 1):
    """Dense-mask attention on the CPU.

    Q, K, V: arrays [B, H, n, d] (any float dtype; converted to `dtype`).  window_size: one
    radius, or a sequence of H radii (head h uses window_size[h]; a per-head window has no
    counterpart in the reference).
    rows: query rows to compute (default: all).  Returns (O, LSE) with O [B, H, len(rows), d]
    and LSE [B, H, len(rows)] in `dtype`.
    """
    Q = np.asarray(Q)
    K = np.asarray(K)
    V = np.asarray(V)
    B, H, n, d = Q.shape
    g = normalize_global_tokens(global_tokens, n)
    rows = np.arange(n, dtype=np.int64) if rows is None else np.asarray(rows, dtype=np.int64)
    out = np.empty((B, H, rows.size, d), dtype=dtype)
    lse = np.empty((B, H, rows.size), dtype=dtype)
    windows = [int(window_size)] * H if np.isscalar(window_size) else [int(x) for x in window_size]
    assert len(windows) == H, "one radius per head"
    for b in range(B):
        for h in range(H):
            k = K[b, h].astype(dtype, copy=False)
            v = V[b, h].astype(dtype, copy=False)
            for s in range(0, rows.size, block_rows):
                r = rows[s:s + block_rows]
                q = Q[b, h, r].astype(dtype, copy=False)
                scores = (q @ k.T) * dtype(scale)
                scores = np.where(visible_rows(r, n, windows[h], g, causal, dilation), scores, -np.inf)
                m = scores.max(axis=1, keepdims=True)
                p = np.exp(scores - m)
                l = p.sum(axis=1, keepdims=True)
                out[b, h, s:s + r.size] = (p @ v) / l
                lse[b, h, s:s + r.size] = (m + np.log(l))[:, 0]
    return out, lse


def sliding_window_attention_varlen(Q, K, V, cu_seqlens: Sequence[int], window_size, global_tokens: Sequence[int],
                                    scale: float, causal: bool = False, dtype=np.float64):
    """Packed sequences: Q, K, V [1, H, total, d] with sequence s in rows
    [cu_seqlens[s], cu_seqlens[s + 1]); each sequence is attended on its own by
    :func:`sliding_window_attention`, the global-token list indexed within it.  Returns
    (O [1, H, total, d], LSE [1, H, total])."""
    Q, K, V = np.asarray(Q), np.asarray(K), np.asarray(V)
    out = np.empty(Q.shape, dtype=dtype)
    lse = np.empty(Q.shape[:3], dtype=dtype)
    for s in range(len(cu_seqlens) - 1):
        a, b = int(cu_seqlens[s]), int(cu_seqlens[s + 1])
        if b == a:
            continue
        o, l = sliding_window_attention(Q[:, :, a:b], K[:, :, a:b], V[:, :, a:b], window_size, global_tokens, scale,
                                        dtype=dtype, causal=causal)
        out[:, :, a:b], lse[:, :, a:b] = o, l
    return out, lse


def sliding_window_attention_backward(Q, K, V, dO, window_size: int, global_tokens: Sequence[int], scale: float,
                                      dtype=np.float64, block_rows: int = 256):
    """Gradients (dQ, dK, dV) of sum(O * dO) for O = :func:`sliding_window_attention`.

    The reference is forward only (its roadmap lists the backward first, README.md:113);
    this restates the gradient of its dense-mask definition
    (python/long_context_attention/__init__.py:24-53): with P the row softmax over visible
    keys, D_i = sum_c dO[i][c] O[i][c], dP = dO V^T, dS = P (dP - D) on visible pairs,
    dQ = scale dS K, dK = scale dS^T Q, dV = P^T dO.  Row-blocked like the forward; all
    arrays [B, H, n, d], results in `dtype`.
    """
    Q, K, V, dO = (np.asarray(x) for x in (Q, K, V, dO))
    B, H, n, d = Q.shape
    g = normalize_global_tokens(global_tokens, n)
    dQ = np.zeros((B, H, n, d), dtype=dtype)
    dK = np.zeros((B, H, n, d), dtype=dtype)
    dV = np.zeros((B, H, n, d), dtype=dtype)
    for b in range(B):
        for h in range(H):
            k = K[b, h].astype(dtype, copy=False)
            v = V[b, h].astype(dtype, copy=False)
            for s in range(0, n, block_rows):
                r = np.arange(s, min(n, s + block_rows), dtype=np.int64)
                q = Q[b, h, r].astype(dtype, copy=False)
                do = dO[b, h, r].astype(dtype, copy=False)
                scores = np.where(visible_rows(r, n, int(window_size), g), (q @ k.T) * dtype(scale), -np.inf)
                m = scores.max(axis=1, keepdims=True)
                p = np.exp(scores - m)
                p /= p.sum(axis=1, keepdims=True)
                o = p @ v
                dvec = (do * o).sum(axis=1, keepdims=True)
                ds = p * (do @ v.T - dvec)
                dQ[b, h, r] = dtype(scale) * (ds @ k)
                dK[b, h] += dtype(scale) * (ds.T @ q)
                dV[b, h] += p.T @ do
    return dQ, dK, dV


def sliding_window_attention_backward_banded(Q, K, V, dO, window_size: int, global_tokens: Sequence[int],
                                             scale: float, dtype=np.float64, block_rows: int = 512):
    """The gradients of :func:`sliding_window_attention_backward` in O(n (block + 2w + G) d)
    instead of O(n^2 d), for full-length checks.

    A block of non-global rows [s, e) sees only the band keys [s - w, e + w) and the global
    keys, so its scores are taken over those columns alone.  The global rows see every key
    (python/long_context_attention/__init__.py:46-47) and take one dense pass.  Same
    definition, same arithmetic per visible pair; all arrays [B, H, n, d].
    """
    Q, K, V, dO = (np.asarray(x) for x in (Q, K, V, dO))
    B, H, n, d = Q.shape
    g = normalize_global_tokens(global_tokens, n)
    w = int(window_size)
    is_global = np.zeros(n, dtype=bool)
    is_global[g] = True
    dQ = np.zeros((B, H, n, d), dtype=dtype)
    dK = np.zeros((B, H, n, d), dtype=dtype)
    dV = np.zeros((B, H, n, d), dtype=dtype)

    def rows_pass(b, h, r, cols, mask):
        k = K[b, h, cols].astype(dtype, copy=False)
        v = V[b, h, cols].astype(dtype, copy=False)
        q = Q[b, h, r].astype(dtype, copy=False)
        do = dO[b, h, r].astype(dtype, copy=False)
        scores = np.where(mask, (q @ k.T) * dtype(scale), -np.inf)
        m = scores.max(axis=1, keepdims=True)
        p = np.exp(scores - m)
        p /= p.sum(axis=1, keepdims=True)
        o = p @ v
        dvec = (do * o).sum(axis=1, keepdims=True)
        ds = p * (do @ v.T - dvec)
        dQ[b, h, r] = dtype(scale) * (ds @ k)
        dK[b, h, cols] += dtype(scale) * (ds.T @ q)   # cols are unique
        dV[b, h, cols] += p.T @ do

    for b in range(B):
        for h in range(H):
            for s in range(0, n, block_rows):
                r = np.arange(s, min(n, s + block_rows), dtype=np.int64)
                r = r[~is_global[r]]
                if r.size == 0:
                    continue
                cols = np.union1d(np.arange(max(0, int(r[0]) - w), min(n, int(r[-1]) + w + 1), dtype=np.int64), g)
                mask = (np.abs(r[:, None] - cols[None, :]) <= w) | is_global[cols][None, :]
                rows_pass(b, h, r, cols, mask)
            if g.size:
                rows_pass(b, h, g, np.arange(n, dtype=np.int64), np.ones((g.size, n), dtype=bool))
    return dQ, dK, dV
