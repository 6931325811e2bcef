"""Named synthetic workloads, seeded input generation and exact work accounting.

The workloads are the shapes the reference's path is measured on (seeded N(0, 1)
inputs; there is no dataset).  ``useful_scores`` counts the true entries of the
Longformer mask of python/long_context_attention/__init__.py:39-47 exactly, which is the
unit of useful work (4 * head_dim FLOPs per entry: 2*d for q.k and 2*d for p.v).
"""
from __future__ import annotations

import dataclasses
import math
from typing import Sequence

import numpy as np
import torch

_DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


@dataclasses.dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    heads: int
    seq_len: int
    head_dim: int
    window: int
    dtype: str
    scale: float
    globals_spec: str          # "list:0,1,2" | "random:64+0" | "range:16"
    std: float = 1.0
    seed: int = 0

    def global_tokens(self) -> list[int]:
        kind, _, arg = self.globals_spec.partition(":")
        if kind == "list":
            return [int(x) for x in arg.split(",") if x != ""]
        if kind == "range":
            return list(range(int(arg)))
        if kind == "random":
            # "<count>+0": `count` indices drawn uniformly without replacement from
            # [0, n) by the workload seed, plus index 0 (sorted, unique).
            count = int(arg.split("+")[0])
            g = torch.Generator().manual_seed(self.seed + 7919)
            drawn = torch.randperm(self.seq_len, generator=g)[:count].tolist()
            return sorted(set(drawn) | {0})
        raise ValueError(f"bad globals spec {self.globals_spec!r}")

    @property
    def torch_dtype(self) -> torch.dtype:
        return _DTYPES[self.dtype]

    def inputs(self, device="cpu", heads_slice: slice | None = None):
        """Seeded Q, K, V of this workload (generated on the CPU, then moved)."""
        return make_inputs(self.seed, self.batch, self.heads, self.seq_len, self.head_dim, self.torch_dtype,
                           std=self.std, device=device, heads_slice=heads_slice)

    def useful_scores(self) -> int:
        return self.batch * self.heads * useful_scores(self.seq_len, self.window, self.global_tokens())

    def useful_flops(self) -> int:
        return 4 * self.head_dim * self.useful_scores()

    def io_bytes(self) -> int:
        """Algorithmic HBM bytes: Q, K, V read once, fp32 O written once."""
        esize = torch.empty(0, dtype=self.torch_dtype).element_size()
        elems = self.batch * self.heads * self.seq_len * self.head_dim
        return 3 * elems * esize + elems * 4

    def tokens(self) -> int:
        """Query rows processed (batch * heads * seq_len)."""
        return self.batch * self.heads * self.seq_len


# The five shapes the reference path is quoted on (1: CPU plumbing case; 2: single long
# head; 3: Longformer-base batch; 4: many global tokens at 64K; 5: 128K, d=128).
WORKLOADS = {
    "cpu_plumbing_2k": Workload("cpu_plumbing_2k", 1, 1, 2048, 64, 128, "fp32", 1 / 8, "list:0,1,2"),
    "single_head_16k": Workload("single_head_16k", 1, 1, 16384, 64, 256, "fp16", 1 / math.sqrt(64), "list:0,1,2"),
    "longformer_base_4k": Workload("longformer_base_4k", 1, 96, 4096, 64, 256, "bf16", 1 / 8, "list:0"),
    "many_globals_64k": Workload("many_globals_64k", 1, 16, 65536, 64, 256, "bf16", 1 / 8, "random:64+0"),
    "context_128k_d128": Workload("context_128k_d128", 1, 8, 131072, 128, 512, "bf16", 1 / math.sqrt(128),
                                  "range:16", std=1 / math.sqrt(2)),
}


def make_inputs(seed: int, batch: int, heads: int, seq_len: int, head_dim: int, dtype: torch.dtype,
                std: float = 1.0, device="cpu", heads_slice: slice | None = None):
    """Q, K, V ~ N(0, std^2) drawn in that order from a CPU generator seeded `seed`,
    rounded to `dtype`, then moved to `device`.  With `heads_slice`, only those heads are
    materialised (the values are those of the full tensors)."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(3):
        t = torch.randn(batch, heads, seq_len, head_dim, generator=g, dtype=torch.float32)
        if std != 1.0:
            t = t * std
        if heads_slice is not None:
            t = t[:, heads_slice].contiguous()
        out.append(t.to(dtype).to(device))
    return tuple(out)


def normalize_global_tokens(tokens: Sequence[int], seq_len: int) -> list[int]:
    """Sorted unique indices with the reference's indexing rules (negative wraps, out of
    range raises IndexError), as `global_mask[list(global_tokens)] = True` does
    (python/long_context_attention/__init__.py:44)."""
    out = set()
    for t in tokens:
        t = int(t)
        if t < -seq_len or t >= seq_len:
            raise IndexError(f"index {t} is out of bounds for dimension 0 with size {seq_len}")
        out.add(t + seq_len if t < 0 else t)
    return sorted(out)


def useful_scores(seq_len: int, window: int, global_tokens: Sequence[int]) -> int:
    """Exact number of true entries of the Longformer mask for one head.

    Global rows see all n keys.  A non-global row i sees its band
    [max(0, i-w), min(n-1, i+w)] plus the global keys outside that band.
    """
    n, w = seq_len, window
    g = np.asarray(normalize_global_tokens(global_tokens, n), dtype=np.int64)
    i = np.arange(n, dtype=np.int64)
    lo = np.maximum(0, i - w)
    hi = np.minimum(n - 1, i + w)
    band = hi - lo + 1
    if g.size:
        inside = np.searchsorted(g, hi, side="right") - np.searchsorted(g, lo, side="left")
        extra = g.size - inside
    else:
        extra = np.zeros(n, dtype=np.int64)
    per_row = band + extra
    is_g = np.zeros(n, dtype=bool)
    is_g[g] = True
    per_row = np.where(is_g, n, per_row)
    return int(per_row.sum())


def useful_scores_shard(seq_len: int, window: int, global_tokens: Sequence[int], offset: int, length: int) -> int:
    """True mask entries one sequence shard computes: its non-global rows' entries, plus
    the global rows' entries against its own keys (G * length).  Summed over all shards
    this is :func:`useful_scores`."""
    n, w = seq_len, window
    g = np.asarray(normalize_global_tokens(global_tokens, n), dtype=np.int64)
    i = np.arange(offset, offset + length, dtype=np.int64)
    lo = np.maximum(0, i - w)
    hi = np.minimum(n - 1, i + w)
    per_row = hi - lo + 1
    if g.size:
        inside = np.searchsorted(g, hi, side="right") - np.searchsorted(g, lo, side="left")
        per_row = per_row + (g.size - inside)
        is_g = np.isin(i, g)
        per_row = np.where(is_g, 0, per_row)
    return int(per_row.sum()) + int(g.size) * length
