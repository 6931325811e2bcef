"""The reference arm of bench.py (`--impl reference`) on the CPU: the JSON line the round-end
driver reads, and the behaviour of ranks other than 0 under torchrun."""
import json
import os
import sys

import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

KEYS = ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
        "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e", "gpu_launches")


def _run(capsys, monkeypatch, argv, rank=0, world=1):
    import bench
    monkeypatch.setenv("RANK", str(rank))
    monkeypatch.setenv("WORLD_SIZE", str(world))
    monkeypatch.setenv("LOCAL_RANK", str(rank))
    assert bench.main(argv) == 0
    return [ln for ln in capsys.readouterr().out.splitlines() if ln.strip()]


@pytest.mark.parametrize("workload", ["many_globals_64k", "context_128k_d128"])
def test_reference_arm_prints_one_contract_line(capsys, monkeypatch, workload):
    import bench
    from long_context_attention.workloads import WORKLOADS
    lines = _run(capsys, monkeypatch, ["--impl", "reference", "--workload", workload, "--steps", "2", "--warmup", "1"])
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in KEYS:
        assert key in line, key
    w = WORKLOADS[workload]
    assert line["impl"] == "reference" and line["metric"] == bench.metric_of(w)
    assert line["value"] > 0 and line["steps"] == 2 and line["warmup"] == 1 and line["higher_is_better"] is True
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["e2e"]["value"] == line["value"] and line["e2e"]["unit"] == line["unit"]
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    # the same config keys as the GPU arm's line for this workload
    assert set(line["config"]) == set(bench.config_of(w, 1, "x").keys())
    assert line["config"]["workload"] == workload


def test_reference_arm_other_ranks_print_nothing(capsys, monkeypatch):
    assert _run(capsys, monkeypatch, ["--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0"],
                rank=1, world=2) == []


def test_sequence_workload_has_its_own_metric():
    import bench
    from long_context_attention.workloads import WORKLOADS
    assert bench.metric_of(WORKLOADS["context_128k_d128"]) != bench.metric_of(WORKLOADS["many_globals_64k"])
