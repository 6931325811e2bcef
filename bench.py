#!/usr/bin/env python
"""Throughput of the sliding-window + global-token attention forward on B200.

Default workload: B=1 x 16 heads, n=65536, d=64, w=256, 65 global tokens (64 drawn by
seed + index 0), bf16, scale 1/8 -- the shape the headline metric is quoted on.  One
"step" is one forward over the resident inputs.  With N GPUs (torchrun, one rank per
GPU) the 16 heads are split over the ranks (16/N each; heads are independent, so there
is no collective on the data path) and the whole job stays fixed ("strong").  The same
line also carries `sequence_128k`: the 128K-token, d=128 workload cut into N contiguous
sequence shards (halo and global-row exchange by NVLink peer stores), timed the same way.

Prints one JSON line (rank 0).  `value` is tokens/s (query rows x heads per second,
whole job); `useful_tflops` counts 4*d FLOPs per true mask entry.  `--impl reference`
times the reference's dense-mask algorithm (the CPU oracle port, all host threads) on a
bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "long-context-attention-kernels_b200", "python"))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402
import torch  # noqa: E402

from long_context_attention.workloads import WORKLOADS  # noqa: E402

METRIC = "tokens/s & useful TFLOP/s, n=64K w=256 d=64 bf16, 1/2/4/8 B200 vs roofline"
UNIT = "tokens/s"
SEQUENCE_WORKLOAD = "context_128k_d128"


def metric_of(w) -> str:
    """The headline metric string for the 64K workload; the same form for the others."""
    if w.name == "many_globals_64k":
        return METRIC
    n = f"{w.seq_len // 1024}K" if w.seq_len % 1024 == 0 else str(w.seq_len)
    split = "sequence-sharded over" if w.name == SEQUENCE_WORKLOAD else ""
    return (f"tokens/s & useful TFLOP/s, n={n} w={w.window} d={w.head_dim} {w.dtype}, "
            f"{split + ' ' if split else ''}1/2/4/8 B200 vs roofline")


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="many_globals_64k", choices=sorted(WORKLOADS))
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--cpu-budget-s", type=float, default=10.0, help="CPU baseline sample budget (rank 0, N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--heads", type=int, default=None,
                    help="override heads per GPU (smaller cases for profiling; not the headline config)")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="sequence shards: halos / global rows / row partials by the library's NVLink peer "
                         "stores (default) or through NCCL")
    ap.add_argument("--parallel", choices=["heads", "sequence"], default=None,
                    help="multi-GPU split: independent head shards (default) or contiguous sequence shards "
                         "(default for context_128k_d128)")
    ap.add_argument("--no-graph", action="store_true",
                    help="time eager forward calls instead of replays of one captured forward")
    ap.add_argument("--no-backward", action="store_true",
                    help="skip the one-GPU measurement of the backward pass on the headline workload")
    ap.add_argument("--no-sequence", action="store_true",
                    help="skip the sequence-sharded 128K measurement added to the head-sharded line")
    ap.add_argument("--cpu-dense-all", action="store_true",
                    help="also time the dense reference definition on the 96-head 4K workload (~40 s)")
    return ap.parse_args(argv)


def load_peaks():
    """(bf16 TFLOP/s, HBM GB/s, source): the pool's measured burst figures, else the
    fallback ones."""
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, 6650.0, "fallback"


def roofline(flops: float, io_bytes: float, kernel_ms: float, traffic, kernel: str) -> dict:
    """Roofline of the main kernel: the slower of the tensor-pipe time (useful FLOPs at the
    bf16 peak) and the HBM time (Q/K/V/O bytes at the copy bandwidth) is the bound;
    `frac` is the roofline time over the measured kernel time.  Both pipes' fractions are
    kept as extra fields."""
    peak_tf, peak_gbs, src = load_peaks()
    sec = kernel_ms * 1e-3
    t_tensor = flops / (peak_tf * 1e12)
    t_hbm = io_bytes / (peak_gbs * 1e9)
    tf = flops / sec / 1e12
    gbs = io_bytes / sec / 1e9
    hbm_bound = t_hbm > t_tensor
    return {"bound": "hbm" if hbm_bound else "tensor",
            "achieved": gbs if hbm_bound else tf, "peak": peak_gbs if hbm_bound else peak_tf,
            "unit": "GB/s" if hbm_bound else "TFLOP/s", "frac": max(t_tensor, t_hbm) / sec,
            "traffic": traffic, "kernel": kernel, "kernel_ms": kernel_ms, "peak_source": src + " (burst)",
            "roofline_ms": max(t_tensor, t_hbm) * 1e3,
            "tensor_achieved_tflops": tf, "tensor_peak_tflops": peak_tf, "tensor_frac": tf / peak_tf,
            "hbm_achieved_gbs": gbs, "hbm_peak_gbs": peak_gbs, "hbm_frac": gbs / peak_gbs}


def load_traffic(workload: str):
    path = os.path.join(REPO, "profiles", "traffic.json")
    try:
        with open(path) as f:
            t = json.load(f)
        return t.get(workload, {}).get("dram_bytes_per_launch")
    except (OSError, ValueError):
        return None


class ClockSampler:
    """Polls NVML for SM clock and clock-event reasons while the timed region runs."""

    REASONS = {0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x4: "sw_power_cap", 0x2: "applications_clocks_setting",
               0x1: "gpu_idle", 0x100: "sync_boost", 0x200: "display_clock_setting"}

    def __init__(self, device_index: int):
        self.ok = False
        self.samples = []
        self.reasons = 0
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            props = torch.cuda.get_device_properties(device_index)
            bus = "%08X:%02X:%02X.0" % (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
            try:
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:  # noqa: BLE001
                self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def sample_now(self):
        """One sample from the calling thread (the launch loop can starve the polling thread of
        the interpreter lock; called right after the loop, while queued steps still run)."""
        if not self.ok:
            return
        try:
            self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            self.reasons |= int(self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
        except Exception:  # noqa: BLE001
            pass

    def _run(self):
        while not self._stop.is_set():
            self.sample_now()
            time.sleep(0.002)

    def start(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        if self._t is not None:
            self._stop.set()
            self._t.join()

    def report(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_baseline(w, q, k, v, budget_s: float, dense_all: bool = False):
    """The reference's dense-mask algorithm on the host cores, on a bounded sample: the
    oracle port (fp32 numpy, all host threads) on random query rows of head 0 of `w`,
    plus the dense torch definition of the reference (`_reference_sliding_window_attention`,
    python/long_context_attention/__init__.py:24-53) run whole on the small workloads where
    its n x n scores fit in host memory."""
    from oracle import swa_oracle

    qs, ks, vs = (t[:1, :1].float().cpu().numpy() for t in (q, k, v))
    g = w.global_tokens()
    rng = np.random.default_rng(0)
    probe = np.sort(rng.choice(w.seq_len, 32, replace=False))
    t0 = time.perf_counter()
    swa_oracle.sliding_window_attention(qs, ks, vs, w.window, g, w.scale, rows=probe, dtype=np.float32, block_rows=32)
    per_row = (time.perf_counter() - t0) / probe.size
    nrows = int(max(64, min(w.seq_len, budget_s / max(per_row, 1e-9))))
    rows = np.sort(rng.choice(w.seq_len, nrows, replace=False))
    t0 = time.perf_counter()
    swa_oracle.sliding_window_attention(qs, ks, vs, w.window, g, w.scale, rows=rows, dtype=np.float32, block_rows=128)
    dt = time.perf_counter() - t0
    out = {"value": rows.size / dt, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
           "sample": f"{rows.size} random query rows of head 0 of {w.name} (dense-mask fp32 numpy, "
                     f"{dt:.1f} s); value = rows/s"}
    out["dense_reference"] = dense_reference_small(dense_all)
    return out


def dense_reference_small(include_4k: bool) -> dict:
    """Whole-workload timings of the reference's dense torch definition on the host cores
    (tokens/s): the 2K plumbing case and the single 16K head, and the 96-head 4K batch on
    request."""
    import long_context_attention as lca

    torch.set_num_threads(os.cpu_count() or 1)
    names = ["cpu_plumbing_2k", "single_head_16k"] + (["longformer_base_4k"] if include_4k else [])
    res = {"threads": torch.get_num_threads(), "impl": "_reference_sliding_window_attention (torch, dense mask)"}
    for name in names:
        w = WORKLOADS[name]
        q, k, v = w.inputs()
        t0 = time.perf_counter()
        lca._reference_sliding_window_attention(q, k, v, w.window, w.global_tokens(), w.scale)
        dt = time.perf_counter() - t0
        res[name] = {"tokens_per_s": w.tokens() / dt, "seconds": dt}
    return res


def config_of(w, world: int, parallelism: str) -> dict:
    """The `config` object of a line; both arms print the same keys for one workload."""
    return {"workload": w.name, "batch": w.batch, "heads": w.heads, "seq_len": w.seq_len, "head_dim": w.head_dim,
            "window": w.window, "num_global": len(w.global_tokens()), "dtype": w.dtype,
            "parallelism": parallelism, "n_gpus": world,
            "l2": "inputs larger than L2 (Q/K/V/O: %.0f MB)" % (w.io_bytes() / 1e6)}


def launches_per_forward(w, fast: bool = True) -> int:
    """Kernels of one lca_swa_forward: gather and merge with global tokens, the main
    kernel, and for bf16 the fp16 copy of V."""
    g = len(w.global_tokens()) > 0
    return 1 + (2 if g else 0) + (1 if (w.dtype == "bf16" and fast) else 0)


def run_reference(args):
    world, rank, _ = dist_setup(args)
    if rank != 0:
        return 0
    from oracle import swa_oracle

    w = WORKLOADS[args.workload]
    q, k, v = w.inputs(heads_slice=slice(0, 1))
    qs, ks, vs = (t.float().numpy() for t in (q, k, v))
    g = w.global_tokens()
    rows_per_step = 16
    rng = np.random.default_rng(1)

    def step():
        rows = np.sort(rng.choice(w.seq_len, rows_per_step, replace=False))
        swa_oracle.sliding_window_attention(qs, ks, vs, w.window, g, w.scale, rows=rows, dtype=np.float32,
                                            block_rows=rows_per_step)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = rows_per_step * args.steps / dt
    sample = (f"{rows_per_step} random query rows of one head per step (dense Longformer-mask fp32, "
              f"numpy oracle port of the reference's _reference_sliding_window_attention)")
    parallel = "sequence" if w.name == SEQUENCE_WORKLOAD else "heads"
    line = {"impl": "reference", "metric": metric_of(w), "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": config_of(w, args.gpus, f"{parallel}-sharded x{args.gpus} (reference: host cores)"),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "gpu_launches": 0}
    print(json.dumps(line), flush=True)
    return 0


def _max_over_ranks(pg, dev, values):
    if pg is None:
        return [float(x) for x in values]
    t = torch.tensor([float(x) for x in values], device=dev, dtype=torch.float64)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def run_ours(args):
    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    import dataclasses

    import long_context_attention as lca
    from long_context_attention import _native
    from long_context_attention.distributed import head_shard
    from long_context_attention.host_pipeline import sliding_window_attention_from_host
    from long_context_attention.workloads import useful_scores

    w = WORKLOADS[args.workload]
    if args.heads is not None:
        w = dataclasses.replace(w, heads=args.heads)
    # rank r computes heads head_shard(H, N, r) of the one seeded job
    hs = head_shard(w.heads, world, rank)
    h_loc = hs.stop - hs.start
    q, k, v = w.inputs(device=dev, heads_slice=hs)
    g = w.global_tokens()
    cabi = _native.cabi()

    def fwd():
        return lca.sliding_window_attention(q, k, v, w.window, g, w.scale)

    # warm-up (on a side stream, as CUDA-graph capture wants), then one forward captured as a
    # CUDA graph: a step is one replay, so the host's per-call work (argument checks, tensor
    # maps, five launches) is off the timed path when a rank's share is small
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(max(args.warmup, 3)):
            out = fwd()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = None
    if h_loc and not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = fwd()
        graph.replay()
        torch.cuda.synchronize()
    step = graph.replay if graph is not None else fwd

    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    clocks.start()
    start.record()
    for _ in range(args.steps):
        step()
    stop.record()
    clocks.sample_now()
    torch.cuda.synchronize()
    clocks.stop()
    if pg is not None:
        pg.barrier()
    ms = start.elapsed_time(stop) / args.steps

    # the main kernel alone: events the library records around its launch, in eager calls
    n_main = min(args.steps, 50)
    ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(n_main)]
    ev_a = [torch.cuda.Event(enable_timing=True) for _ in range(n_main)]
    for e in ev_b + ev_a:  # (torch's elapsed_time wants events it has seen recorded once)
        e.record()
    main_ms = 0.0
    if h_loc:
        for i in range(n_main):
            cabi.lib.lca_set_timing_events(ev_b[i].cuda_event, ev_a[i].cuda_event)
            out = fwd()
        cabi.lib.lca_set_timing_events(None, None)
        torch.cuda.synchronize()
        main_ms = statistics.mean(ev_b[i].elapsed_time(ev_a[i]) for i in range(n_main))
    assert lca.device_error() == 0
    del out, graph

    # ---- end to end through the public host-buffer entry point: pinned H2D of the step's
    # inputs, the forward, D2H of the output, pipelined over head chunks
    qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
    oh = torch.empty(q.shape, dtype=torch.float32).pin_memory()

    def e2e_step():
        sliding_window_attention_from_host(qh, kh, vh, w.window, g, w.scale, out=oh)

    e2e_step()
    torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.e2e_steps
    h2d = sum(t.numel() * t.element_size() for t in (q, k, v))
    d2h = oh.numel() * 4
    del qh, kh, vh, oh

    per_head = useful_scores(w.seq_len, w.window, g) * 4 * w.head_dim * w.batch
    flops_rank = per_head * h_loc
    io_rank = w.io_bytes() // w.heads * h_loc
    ms, e2e_ms, main_ms, flops_max, io_max = _max_over_ranks(pg, dev, [ms, e2e_ms, main_ms, flops_rank, io_rank])
    h2d_all, d2h_all = (h2d * world, d2h * world) if pg is None else _sum_over_ranks(pg, dev, [h2d, d2h])
    del q, k, v

    others = None
    if world == 1 and not args.no_sequence and w.name == "many_globals_64k":
        others = {name: measure_one_gpu(WORKLOADS[name], dev, steps=min(args.steps, 100), warmup=args.warmup)
                  for name in ("single_head_16k", "longformer_base_4k")}

    backward = None
    if world == 1 and not args.no_backward:
        backward = measure_backward(w, dev, steps=min(args.steps, 20), warmup=args.warmup)

    sequence = None
    if not args.no_sequence and w.name != SEQUENCE_WORKLOAD:
        sequence = measure_sequence(WORKLOADS[SEQUENCE_WORKLOAD], world, rank, local, dev, pg,
                                    steps=min(args.steps, 200), warmup=max(args.warmup, 3), exchange=args.exchange,
                                    e2e_steps=0, cpu=False)

    tokens = w.tokens()
    traffic = load_traffic(w.name)
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(w, *w.inputs(heads_slice=slice(0, 1)), args.cpu_budget_s, args.cpu_dense_all)
        rf = roofline(flops_max, io_max, main_ms,
                      traffic * io_max / w.io_bytes() if traffic is not None else None, "lca_swa_main")
        rf["note"] = ("largest head shard's useful FLOPs and Q/K/V/O bytes over the max-over-ranks main-kernel "
                      "time" if world > 1 else "useful FLOPs and Q/K/V/O bytes over the main-kernel time")
        line = {
            "metric": metric_of(w), "value": tokens / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": w.dtype, "data": "synthetic",
            "useful_tflops": w.useful_flops() / (ms * 1e-3) / 1e12,
            "config": config_of(w, world, f"head-sharded x{world} ({w.heads // world if world <= w.heads else 1}"
                                          f" heads per GPU)"),
            "step_timing": ("replays of one forward captured as a CUDA graph" if not args.no_graph
                            else "eager forward calls"),
            "roofline": rf,
            "cpu_baseline": cpu,
            "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d_all,
                    "d2h_bytes_per_step": d2h_all, "ms_per_step": e2e_ms,
                    "path": "sliding_window_attention_from_host (pinned host buffers, head chunks pipelined "
                            "over copy and compute streams)"},
            "gpu_launches": args.steps * launches_per_forward(w),
            "clocks": clocks.report(),
        }
        if sequence is not None:
            line["sequence_128k"] = sequence
        if others is not None:
            line["other_configs"] = others
        if backward is not None:
            line["backward"] = backward
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def _sum_over_ranks(pg, dev, values):
    t = torch.tensor([float(x) for x in values], device=dev, dtype=torch.float64)
    pg.all_reduce(t)
    return [int(x) for x in t.tolist()]


def measure_one_gpu(w, dev, steps: int, warmup: int) -> dict:
    """One workload whole on this GPU: a step is one replay of one forward captured as a
    CUDA graph (inputs resident); the main kernel is timed by the library's events in eager
    calls.  For the workloads the headline line does not carry (one 16K head in fp16, the
    96-head 4K batch), so every configuration has a device measurement."""
    import long_context_attention as lca
    from long_context_attention import _native

    cabi = _native.cabi()
    q, k, v = w.inputs(device=dev)
    g = w.global_tokens()

    def fwd():
        return lca.sliding_window_attention(q, k, v, w.window, g, w.scale)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(max(warmup, 3)):
            out = fwd()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = fwd()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        graph.replay()
    stop.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / steps
    n_main = min(steps, 20)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_main)]
    for a, b in ev:
        a.record()
        b.record()
    for a, b in ev:
        cabi.lib.lca_set_timing_events(a.cuda_event, b.cuda_event)
        out = fwd()
    cabi.lib.lca_set_timing_events(None, None)
    torch.cuda.synchronize()
    main_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    assert lca.device_error() == 0
    del out, graph, q, k, v
    rf = roofline(w.useful_flops(), w.io_bytes(), main_ms, None, "lca_swa_main")
    return {"workload": w.name, "metric": metric_of(w), "value": w.tokens() / (ms * 1e-3), "unit": UNIT,
            "ms_per_step": ms, "main_kernel_ms": main_ms, "useful_tflops": w.useful_flops() / (ms * 1e-3) / 1e12,
            "config": config_of(w, 1, "one GPU"), "roofline": rf,
            "step_timing": "replays of one forward captured as a CUDA graph"}


def measure_backward(w, dev, steps: int, warmup: int) -> dict:
    """The backward pass (sliding_window_attention_backward: dQ, dK, dV from the forward's O
    and LSE and a seeded dO) of the whole workload on this GPU, inputs resident, one call
    captured as a CUDA graph and replayed; CUDA events around the replays.  Useful FLOPs are
    2.5x the forward's (five products of 2 d per visible score against two)."""
    import long_context_attention as lca

    q, k, v = w.inputs(device=dev)
    g = w.global_tokens()
    out, lse = lca.sliding_window_attention_with_lse(q, k, v, w.window, g, w.scale)
    gen = torch.Generator(device=dev).manual_seed(7)
    dout = torch.randn(out.shape, device=dev, generator=gen)

    def bwd():
        return lca.sliding_window_attention_backward(q, k, v, out, lse, dout, w.window, g, w.scale)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(max(warmup, 3)):
            grads = bwd()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        grads = bwd()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        graph.replay()
    stop.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / steps
    assert lca.device_error() == 0
    del grads, graph, q, k, v, out, lse, dout
    torch.cuda.empty_cache()
    flops = 2.5 * w.useful_flops()
    # bytes the backward must move: Q, K, V (16-bit) and O, dO (fp32) read, dQ, dK, dV (fp32) written
    elems = w.batch * w.heads * w.seq_len * w.head_dim
    io = elems * (3 * 2 + 2 * 4 + 3 * 4)
    rf = roofline(flops, io, ms, None, "lca_bwd_prep + lca_bwd_main (dQ, dK/dV) + lca_bwd_reduce")
    return {"workload": w.name, "ms_per_step": ms, "useful_tflops": flops / (ms * 1e-3) / 1e12,
            "tokens_per_s": w.tokens() / (ms * 1e-3), "roofline": rf,
            "step_timing": "replays of one backward call captured as a CUDA graph",
            "note": "whole backward call (5 launches); useful FLOPs = 2.5 x the forward's"}


def measure_sequence(w, world, rank, local, dev, pg, steps, warmup, exchange, e2e_steps, cpu, heads=None,
                     cpu_budget_s=10.0):
    """One sequence cut into contiguous shards, one per rank (strong scaling: the whole
    job is fixed).  A step is the full sharded forward on every rank -- prepare, the
    exchange of global rows and halos, the shard kernels, the exchange of the global-row
    partials and their merge -- replayed from one CUDA graph per rank; the step time is
    the max over ranks.  Returns the measurement as a dict (rank 0; None elsewhere)."""
    import dataclasses

    import long_context_attention as lca
    from long_context_attention import _native
    from long_context_attention.distributed import ShardedAttention, shard_bounds
    from long_context_attention.workloads import useful_scores_shard

    if heads is not None:
        w = dataclasses.replace(w, heads=heads)
    g = w.global_tokens()
    off, ln = shard_bounds(w.seq_len, world)[rank]
    qf, kf, vf = w.inputs()
    q, k, v = (t[:, :, off:off + ln].contiguous().to(dev) for t in (qf, kf, vf))
    cpu_inputs = (qf[:, :1], kf[:, :1], vf[:, :1]) if (cpu and rank == 0 and world == 1) else None
    del qf, kf, vf
    cabi = _native.cabi()
    plan = ShardedAttention(w.batch, w.heads, w.seq_len, w.head_dim, w.window, g, w.scale, w.torch_dtype, device=dev,
                            exchange=exchange)
    plan.capture(q, k, v, warmup=warmup)
    for _ in range(warmup):
        plan.replay()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    clocks.start()
    start.record()
    for _ in range(steps):
        plan.replay()
    stop.record()
    clocks.sample_now()
    torch.cuda.synchronize()
    clocks.stop()
    ms = start.elapsed_time(stop) / steps

    # main-kernel time from eager calls of the same plan (events recorded around the launch)
    k_steps = min(steps, 20)
    ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(k_steps)]
    ev_a = [torch.cuda.Event(enable_timing=True) for _ in range(k_steps)]
    for e in ev_b + ev_a:  # torch's events count as recorded only after one record()
        e.record()
    for i in range(k_steps):
        cabi.lib.lca_set_timing_events(ev_b[i].cuda_event, ev_a[i].cuda_event)
        plan(q, k, v)
    cabi.lib.lca_set_timing_events(None, None)
    torch.cuda.synchronize()
    main_ms = statistics.mean(ev_b[i].elapsed_time(ev_a[i]) for i in range(k_steps))
    plan.raise_on_device_error()

    e2e_ms = 0.0
    h2d = d2h = 0
    if e2e_steps > 0:
        # pinned H2D of this rank's shard into the plan's inputs, the graph, D2H of its rows
        qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
        oh = torch.empty(plan.out.shape, dtype=torch.float32).pin_memory()

        def e2e_step():
            q.copy_(qh, non_blocking=True)
            k.copy_(kh, non_blocking=True)
            v.copy_(vh, non_blocking=True)
            oh.copy_(plan.replay(), non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        if pg is not None:
            pg.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(e2e_steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / e2e_steps
        h2d = sum(t.numel() * t.element_size() for t in (q, k, v)) * world
        d2h = oh.numel() * 4 * world

    flops_rank = 4 * w.head_dim * w.batch * w.heads * useful_scores_shard(w.seq_len, w.window, g, off, ln)
    io_rank = w.io_bytes() * ln // w.seq_len
    ms, e2e_ms, main_ms, flops_max, io_max = _max_over_ranks(pg, dev, [ms, e2e_ms, main_ms, flops_rank, io_rank])
    # kernels of one step: gather (global tokens), halo pack (2+ shards), the fp16 copy of V
    # (bf16), the main kernel, the split merge (global tokens), then the peer exchange's two
    # copy kernels and its merge, or the final merge alone
    g1 = 1 if g else 0
    halo = 1 if (world > 1 and w.window > 0) else 0
    main = 2 if w.dtype == "bf16" else 1
    per_step = g1 + halo + main + g1 + (3 if plan.exchange == "peer" else g1)
    exchange_used = plan.exchange
    plan.release()
    del q, k, v
    if rank != 0:
        return None
    full_traffic = load_traffic(w.name)
    res = {
        "workload": w.name, "metric": metric_of(w), "value": w.tokens() / (ms * 1e-3), "unit": UNIT,
        "ms_per_step": ms, "n_gpus": world, "steps": steps, "scaling": "strong",
        "useful_tflops": w.useful_flops() / (ms * 1e-3) / 1e12,
        "config": config_of(w, world, f"sequence-sharded x{world}") | {"cuda_graph": True, "exchange": exchange_used,
                                                                          "tokens_per_gpu_step": ln * w.batch * w.heads},
        "main_kernel_ms": main_ms,
        "roofline": roofline(flops_max, io_max, main_ms,
                             full_traffic * ln / w.seq_len if full_traffic is not None else None, "lca_swa_main")
                    | {"note": "largest shard's useful FLOPs and Q/K/V/O bytes over the max-over-ranks main-kernel "
                               "time"},
        "gpu_launches": steps * per_step,
        "clocks": clocks.report(),
    }
    if e2e_steps > 0:
        res["e2e"] = {"value": w.tokens() / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                      "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms}
    if cpu_inputs is not None:
        res["cpu_baseline"] = cpu_baseline(w, *cpu_inputs, cpu_budget_s)
    return res


def run_sequence(args):
    """The sequence-sharded workload as the line's headline (``--workload context_128k_d128``)."""
    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import datetime

    import torch.distributed as dist

    pg = None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    w = WORKLOADS[args.workload]
    res = measure_sequence(w, world, rank, local, dev, pg, steps=args.steps, warmup=max(args.warmup, 3),
                           exchange=args.exchange, e2e_steps=args.e2e_steps, cpu=not args.no_cpu_baseline,
                           heads=args.heads, cpu_budget_s=args.cpu_budget_s)
    if rank == 0:
        line = {"metric": res.pop("metric"), "value": res.pop("value"), "unit": res.pop("unit"), "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": res.pop("ms_per_step"),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": w.dtype,
                "data": "synthetic"}
        res.pop("n_gpus")
        res.pop("steps")
        res.pop("scaling")
        res.pop("workload")
        line.update(res)
        line.setdefault("cpu_baseline", None)
        print(json.dumps(line), flush=True)
    if pg is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        return run_reference(args)
    parallel = args.parallel or ("sequence" if args.workload == "context_128k_d128" else "heads")
    if parallel == "sequence":
        return run_sequence(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
