"""Generate the golden fixtures under tests/golden/ by running the REFERENCE implementation.

Run in a container that has the reference checkout, naming its root directory in
LCA_REFERENCE_DIR (required: the script has no default location):

    LCA_REFERENCE_DIR=<reference checkout> python tests/golden/make_golden.py

For every case it builds seeded inputs, calls the reference's
``_reference_sliding_window_attention`` (python/long_context_attention/__init__.py:24-53,
imported by file path under a private module name so it cannot collide with this
repository's package of the same name), and stores the reference output for the chosen
rows in ``<case>.npz``.  Inputs are not stored for most cases: they are regenerated from
the seed with ``long_context_attention.workloads.make_inputs`` and checked against the
SHA-256 recorded here.  The two reference-test cases store their (tiny) inputs inline,
drawn exactly as tests/test_correctness.py:26-62 draws them.
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "long-context-attention-kernels_b200", "python"))
from long_context_attention.workloads import WORKLOADS, make_inputs  # noqa: E402

_DT = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def load_reference():
    ref_dir = os.environ.get("LCA_REFERENCE_DIR")
    if not ref_dir:
        raise SystemExit("set LCA_REFERENCE_DIR to the root of the reference checkout")
    path = os.path.join(ref_dir, "python", "long_context_attention", "__init__.py")
    spec = importlib.util.spec_from_file_location("_lca_reference_impl", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod._reference_sliding_window_attention


def input_digest(q, k, v) -> str:
    h = hashlib.sha256()
    for t in (q, k, v):
        h.update(t.float().contiguous().numpy().tobytes())
    return h.hexdigest()


def sample_rows(n, g, every):
    rows = set(range(min(n, 48))) | set(range(max(0, n - 48), n)) | set(range(0, n, every))
    rows |= {int(x) % n for x in g}
    return sorted(rows)


# name: (B, H, n, d, dtype, window, globals, scale, seed, row_every or None for all rows)
CASES = {
    # shapes of the reference's own GPU test (tests/test_correctness.py:65-80)
    "ref_gpu_case_fp16": (1, 2, 512, 64, "fp16", 64, [0, 1, 2], 1 / 8, 2, None),
    "ref_gpu_case_bf16": (1, 2, 512, 64, "bf16", 64, [0, 1, 2], 1 / 8, 2, 3),
    # edge cases
    "dup_neg_globals": (1, 2, 300, 64, "bf16", 17, [5, 5, -1, 150, 0], 0.125, 11, None),
    "no_globals_w0": (1, 1, 257, 64, "fp16", 0, [], 0.125, 12, None),
    "window_exceeds_n": (1, 1, 200, 128, "bf16", 1000, [3], 1 / math.sqrt(128), 13, None),
    "tiny_n5": (1, 1, 5, 64, "fp16", 2, [4], 0.125, 14, None),
    "two_global_tiles": (2, 1, 640, 64, "bf16", 64, "rand150", 0.125, 15, 3),
    "d128_multi_head": (1, 3, 384, 128, "fp16", 100, [0, 383], 1 / math.sqrt(128), 16, 5),
    "globals_in_band": (1, 1, 512, 64, "bf16", 256, [10, 20, 30, 300], 0.125, 17, None),
    "batch2_heads2": (2, 2, 320, 64, "fp16", 40, [7, 200], 0.125, 18, 4),
    "ragged_n_d128": (1, 2, 333, 128, "bf16", 70, [332, -333], 1 / math.sqrt(128), 19, 3),
    "band_tile_aligned": (1, 1, 1024, 64, "bf16", 128, [512], 0.125, 20, 4),
}


def case_globals(spec, n, seed):
    if spec == "rand150":
        g = torch.Generator().manual_seed(seed + 1)
        return sorted(torch.randperm(n, generator=g)[:150].tolist())
    return list(spec)


def main():
    ref = load_reference()
    written = []

    # -- the reference's two CPU tests, inputs drawn exactly as the tests draw them
    torch.manual_seed(0)
    q, k, v = (torch.randn(1, 2, 32, 16) for _ in range(3))
    out = ref(q, k, v, window_size=32, global_tokens=[], scale=1 / math.sqrt(16))
    np.savez_compressed(os.path.join(HERE, "reftest_unmasked.npz"),
                        meta=json.dumps(dict(window=32, globals=[], scale=1 / math.sqrt(16), inline=True)),
                        q=q.numpy(), k=k.numpy(), v=v.numpy(), rows=np.arange(32), out=out.numpy())
    written.append("reftest_unmasked")
    torch.manual_seed(1)
    q, k, v = (torch.randn(1, 1, 64, 16) for _ in range(3))
    out = ref(q, k, v, window_size=1, global_tokens=[0], scale=1 / math.sqrt(16))
    np.savez_compressed(os.path.join(HERE, "reftest_global_row.npz"),
                        meta=json.dumps(dict(window=1, globals=[0], scale=1 / math.sqrt(16), inline=True)),
                        q=q.numpy(), k=k.numpy(), v=v.numpy(), rows=np.arange(64), out=out.numpy())
    written.append("reftest_global_row")

    # -- the CPU plumbing workload (fp32), sampled rows
    w = WORKLOADS["cpu_plumbing_2k"]
    q, k, v = w.inputs()
    out = ref(q, k, v, w.window, w.global_tokens(), w.scale)
    rows = sample_rows(w.seq_len, w.global_tokens(), 16)
    meta = dict(batch=w.batch, heads=w.heads, seq_len=w.seq_len, head_dim=w.head_dim, dtype=w.dtype,
                window=w.window, globals=w.global_tokens(), scale=w.scale, seed=w.seed, std=w.std,
                sha256=input_digest(q, k, v), inline=False)
    np.savez_compressed(os.path.join(HERE, "workload_cpu_plumbing_2k.npz"), meta=json.dumps(meta),
                        rows=np.asarray(rows), out=out[:, :, rows].numpy())
    written.append("workload_cpu_plumbing_2k")

    # -- edge / parity cases
    for name, (B, H, n, d, dt, win, gspec, scale, seed, every) in CASES.items():
        g = case_globals(gspec, n, seed)
        q, k, v = make_inputs(seed, B, H, n, d, _DT[dt])
        out = ref(q, k, v, win, g, scale)
        rows = list(range(n)) if every is None else sample_rows(n, g, every)
        meta = dict(batch=B, heads=H, seq_len=n, head_dim=d, dtype=dt, window=win, globals=g, scale=scale,
                    seed=seed, std=1.0, sha256=input_digest(q, k, v), inline=False)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), meta=json.dumps(meta), rows=np.asarray(rows),
                            out=out[:, :, rows].numpy().astype(np.float32))
        written.append(name)
    total = sum(os.path.getsize(os.path.join(HERE, f"{x}.npz")) for x in written)
    print(f"wrote {len(written)} fixtures, {total / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
