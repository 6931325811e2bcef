"""Shared helpers for the tests: golden fixtures, tolerances, comparison metrics."""
from __future__ import annotations

import glob
import hashlib
import json
import os

import numpy as np
import torch

from long_context_attention.workloads import make_inputs

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
_DT = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}

# Parity bar for fp16/bf16 inputs with fp32 accumulation.
MAX_ABS_TOL = 2e-3
REL_L2_TOL = 1e-3
LSE_ABS_TOL = 1e-4


def golden_names() -> list[str]:
    return sorted(os.path.splitext(os.path.basename(p))[0] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def load_golden(name: str) -> dict:
    """Fixture dict: meta fields + q, k, v (torch, CPU, input dtype) + rows + out (np fp32)."""
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    meta = json.loads(str(z["meta"]))
    case = dict(meta)
    case["name"] = name
    case["rows"] = z["rows"].astype(np.int64)
    case["out"] = z["out"].astype(np.float32)
    if meta.get("inline"):
        case["q"], case["k"], case["v"] = (torch.from_numpy(z[x]) for x in ("q", "k", "v"))
        case["dtype"] = "fp32"
        case["batch"], case["heads"], case["seq_len"], case["head_dim"] = z["q"].shape
    else:
        q, k, v = make_inputs(meta["seed"], meta["batch"], meta["heads"], meta["seq_len"], meta["head_dim"],
                              _DT[meta["dtype"]], std=meta.get("std", 1.0))
        h = hashlib.sha256()
        for t in (q, k, v):
            h.update(t.float().contiguous().numpy().tobytes())
        assert h.hexdigest() == meta["sha256"], f"{name}: regenerated inputs differ from the fixture's"
        case["q"], case["k"], case["v"] = q, k, v
    return case


def gpu_capable(case: dict) -> bool:
    return case["dtype"] in ("fp16", "bf16") and case["head_dim"] in (64, 128)


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def max_abs(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.max(np.abs(np.asarray(a, dtype=np.float64) - np.asarray(b, dtype=np.float64))))


def assert_parity(got: np.ndarray, want: np.ndarray, what: str, max_abs_tol=MAX_ABS_TOL, rel_tol=REL_L2_TOL):
    assert np.all(np.isfinite(got)), f"{what}: non-finite values"
    ma, rl = max_abs(got, want), rel_l2(got, want)
    assert ma <= max_abs_tol and rl <= rel_tol, f"{what}: max_abs={ma:.3e} rel_l2={rl:.3e}"


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()
