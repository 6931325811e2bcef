#!/usr/bin/env python
"""Throughput of the sliding-window + global-token attention forward on B200.

Default workload: B=1 x 16 heads, n=65536, d=64, w=256, 65 global tokens (64 drawn by
seed + index 0), bf16, scale 1/8 -- the shape the headline metric is quoted on.  One
"step" is one forward over the resident inputs.  With N GPUs (torchrun, one rank per
GPU) every rank processes its own 16-head shard of an N*16-head job (heads are
independent: no collective on the data path), so per-GPU work is fixed ("weak").

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
    return ap.parse_args(argv)


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, 6650.0, "fallback"


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


def cpu_baseline(w, q, k, v, budget_s: float):
    """The reference's dense-mask algorithm (oracle port, fp32 like the reference) on a
    bounded sample of query rows of head 0, all host threads."""
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
    return {"value": rows.size / dt, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
            "sample": f"{rows.size} random query rows of head 0 of {w.name} (dense-mask fp32 numpy, "
                      f"{dt:.1f} s); value = rows/s"}


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
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": w.name, "seq_len": w.seq_len, "head_dim": w.head_dim,
                                            "window": w.window, "num_global": len(g)},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "gpu_launches": 0}
    print(json.dumps(line), flush=True)
    return 0


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
    import long_context_attention as lca
    from long_context_attention import _native

    base = WORKLOADS[args.workload]
    # rank r owns heads [r*H, (r+1)*H) of an N*H-head job; its inputs are the workload's
    # seeded tensors with the seed offset by the rank
    import dataclasses
    w = dataclasses.replace(base, seed=base.seed + rank)
    if args.heads is not None:
        w = dataclasses.replace(w, heads=args.heads)
    q, k, v = w.inputs(device=dev)
    g = w.global_tokens()
    cabi = _native.cabi()

    def fwd():
        return lca.sliding_window_attention(q, k, v, w.window, g, w.scale)

    for _ in range(max(args.warmup, 3)):
        out = fwd()
    torch.cuda.synchronize()

    # per-step events around the main kernel (recorded by the library on the launch stream)
    ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ev_a = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for e in ev_b + ev_a:
        e.record()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)

    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    clocks.start()
    start.record()
    for i in range(args.steps):
        cabi.lib.lca_set_timing_events(ev_b[i].cuda_event, ev_a[i].cuda_event)
        out = fwd()
    stop.record()
    clocks.sample_now()
    torch.cuda.synchronize()
    clocks.stop()
    cabi.lib.lca_set_timing_events(None, None)
    if pg is not None:
        pg.barrier()
    ms = start.elapsed_time(stop) / args.steps
    main_ms = statistics.mean(ev_b[i].elapsed_time(ev_a[i]) for i in range(args.steps))
    assert lca.device_error() == 0
    del out

    # ---- end to end through the public API with host buffers: pinned H2D of the step's
    # inputs, the forward, D2H of the output
    qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
    oh = torch.empty(q.shape, dtype=torch.float32).pin_memory()
    qd, kd, vd = (torch.empty_like(t) for t in (q, k, v))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def e2e_step():
        qd.copy_(qh, non_blocking=True)
        kd.copy_(kh, non_blocking=True)
        vd.copy_(vh, non_blocking=True)
        o = lca.sliding_window_attention(qd, kd, vd, w.window, g, w.scale)
        oh.copy_(o, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    e0.record()
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.e2e_steps

    if pg is not None:
        t = torch.tensor([ms, e2e_ms, main_ms], device=dev, dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms, e2e_ms, main_ms = (float(x) for x in t.tolist())

    tokens = w.tokens() * world
    value = tokens / (ms * 1e-3)
    flops_rank = w.useful_flops()
    peak_tf, peak_gbs, peak_src = load_peaks()
    achieved_tf = flops_rank / (main_ms * 1e-3) / 1e12
    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(w, q, k, v, args.cpu_budget_s)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16" if w.dtype == "bf16" else w.dtype, "data": "synthetic",
            "useful_tflops": flops_rank * world / (ms * 1e-3) / 1e12,
            "config": {"workload": w.name, "batch": w.batch, "heads_per_gpu": w.heads, "seq_len": w.seq_len,
                       "head_dim": w.head_dim, "window": w.window, "num_global": len(g),
                       "tokens_per_gpu_step": w.tokens(), "parallelism": f"head-sharded x{world}",
                       "l2": "inputs larger than L2 (Q/K/V/O resident: %.0f MB)" % (w.io_bytes() / 1e6)},
            "roofline": {"bound": "tensor", "achieved": achieved_tf, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": achieved_tf / peak_tf, "traffic": load_traffic(w.name),
                         "kernel": "lca_swa_main", "kernel_ms": main_ms, "peak_source": peak_src,
                         "hbm_achieved_gbs": w.io_bytes() / (main_ms * 1e-3) / 1e9, "hbm_peak_gbs": peak_gbs,
                         "hbm_frac": w.io_bytes() / (main_ms * 1e-3) / 1e9 / peak_gbs},
            "cpu_baseline": cpu,
            "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in (q, k, v)),
                    "d2h_bytes_per_step": oh.numel() * 4, "ms_per_step": e2e_ms},
            # main kernel; gather and merge with global tokens; for bf16 the fp16 copy of V
            # and the second main-kernel variant (one of the two returns at once)
            "gpu_launches": args.steps * (1 + (2 if g else 0) + (2 if w.dtype == "bf16" else 0)),
            "clocks": clocks.report(),
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def run_sequence(args):
    """One sequence cut into contiguous shards, one per rank (strong scaling: the whole
    job is fixed).  A step is the full sharded forward on every rank -- prepare, the
    point-to-point exchange (global rows, halos), the shard kernels, the global-row
    partial all-gather and the merge -- replayed from one CUDA graph per rank; the step
    time is the max over ranks."""
    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import datetime

    import torch.distributed as dist

    import long_context_attention as lca
    from long_context_attention import _native
    from long_context_attention.distributed import ShardedAttention, shard_bounds
    from long_context_attention.workloads import useful_scores_shard

    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    w = WORKLOADS[args.workload]
    if args.heads is not None:
        import dataclasses
        w = dataclasses.replace(w, heads=args.heads)
    g = w.global_tokens()
    off, ln = shard_bounds(w.seq_len, world)[rank]
    qf, kf, vf = w.inputs()
    q, k, v = (t[:, :, off:off + ln].contiguous().to(dev) for t in (qf, kf, vf))
    cpu_inputs = (qf, kf, vf) if (rank == 0 and world == 1) else None
    del qf, kf, vf
    cabi = _native.cabi()
    plan = ShardedAttention(w.batch, w.heads, w.seq_len, w.head_dim, w.window, g, w.scale, w.torch_dtype, device=dev,
                            exchange=args.exchange)
    plan.capture(q, k, v, warmup=max(args.warmup, 3))
    for _ in range(max(args.warmup, 3)):
        plan.replay()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    start.record()
    for _ in range(args.steps):
        plan.replay()
    stop.record()
    clocks.sample_now()
    torch.cuda.synchronize()
    clocks.stop()
    ms = start.elapsed_time(stop) / args.steps

    # main-kernel time from eager calls of the same plan (events recorded around the launch)
    k_steps = min(args.steps, 20)
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
    assert lca.device_error() == 0

    # end to end: pinned H2D of this rank's shard into the plan's inputs, the graph, D2H
    # of its rows
    qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
    oh = torch.empty(plan.out.shape, dtype=torch.float32).pin_memory()

    def e2e_step():
        q.copy_(qh, non_blocking=True)
        k.copy_(kh, non_blocking=True)
        v.copy_(vh, non_blocking=True)
        oh.copy_(plan.replay(), non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.e2e_steps

    flops_rank = 4 * w.head_dim * w.batch * w.heads * useful_scores_shard(w.seq_len, w.window, g, off, ln)
    if world > 1:
        t = torch.tensor([ms, e2e_ms, main_ms, float(flops_rank)], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, main_ms, flops_max = (float(x) for x in t.tolist())
    else:
        flops_max = flops_rank
    tokens = w.tokens()
    # DRAM bytes of one whole-sequence launch (ncu, profiles/traffic.json), split evenly over
    # the shards (the per-shard band work is uniform)
    full_traffic = load_traffic(w.name)
    shard_traffic = full_traffic / world if full_traffic is not None else None
    peak_tf, peak_gbs, peak_src = load_peaks()
    achieved_tf = flops_max / (main_ms * 1e-3) / 1e12
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(w, *cpu_inputs, args.cpu_budget_s)
        shard_io = w.io_bytes() / world
        line = {
            "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": w.dtype, "data": "synthetic",
            "useful_tflops": w.useful_flops() / (ms * 1e-3) / 1e12,
            "config": {"workload": w.name, "batch": w.batch, "heads": w.heads, "seq_len": w.seq_len,
                       "head_dim": w.head_dim, "window": w.window, "num_global": len(g),
                       "tokens_per_gpu_step": ln * w.batch * w.heads,
                       "parallelism": f"sequence-sharded x{world}", "cuda_graph": True,
                       "exchange": plan.exchange,
                       "l2": "inputs larger than L2 (shard Q/K/V/O resident: %.0f MB)" % (shard_io / 1e6)},
            "roofline": {"bound": "tensor", "achieved": achieved_tf, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": achieved_tf / peak_tf, "traffic": shard_traffic, "kernel": "lca_swa_main",
                         "kernel_ms": main_ms, "peak_source": peak_src,
                         "note": "largest shard's useful FLOPs / max-over-ranks main-kernel time"},
            "cpu_baseline": cpu,
            "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in (q, k, v)) * world,
                    "d2h_bytes_per_step": oh.numel() * 4 * world, "ms_per_step": e2e_ms},
            # main, halo pack (2+ shards), the two peer puts and the peer merge (peer exchange);
            # with global tokens also gather, local merge (and the final merge over NCCL); for
            # bf16 the fp16 copy of V and the second main-kernel variant
            "gpu_launches": args.steps * (
                ((5 + (2 if g else 0)) if plan.exchange == "peer" else ((2 if world > 1 else 1) + (3 if g else 0)))
                + (2 if w.dtype == "bf16" else 0)),
            "clocks": clocks.report(),
        }
        print(json.dumps(line), flush=True)
    plan.release()
    if world > 1:
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
