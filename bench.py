"""Benchmark of the B200 AWA layer (SeedVR2 adaptive window attention).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--workload cfg4]

Metric: AWA attention windows/s (and TFLOPS) per B200, against
the reference's ncnn CPU path. A step is one AWA layer forward -- Pack ->
MMRoPE -> WindowAttention -> Unpack, run as the fused chain awa_forward --
over one synthetic batch of the workload's shape, inputs resident in HBM.

* value      windows of all ranks / max-over-ranks device time (CUDA events)
* e2e        same metric through the C ABI with host buffers (awa_forward_host:
             copy of the step's QKV from pinned host memory, the forward, copy
             of the outputs back, every step inside the timed region); steps
             alternate over two streams and device workspaces (copy in of the
             next step and copy out of the previous one overlap the forward)
* roofline   the dominant kernel (fused tcgen05 attention), timed live by the
             library's launch profiler (events on its own stream)
* cpu_baseline  the reference's own awa_layers.cpp CPU forward (oracle/_ref),
             on a bounded sample of cfg4-shaped windows, scaled by sum(L^2)

N > 1 (torchrun, one rank per GPU): one layer split over the N GPUs
(awa_forward_sharded: bands of windows per rank, NCCL all-reduce of the text
partial sums, the video rows pushed to every rank by peer copies, or NCCL
all-gather with --exchange nccl) -- strong scaling; --mode replicas runs an
independent layer per GPU instead (weak scaling).
--impl reference times the reference CPU path on all host cores (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import math
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "seedvr2-ncnn_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "AWA attention TFLOPS & windows/s per B200 (1/2/4/8 GPU) vs ncnn CPU ref"
UNIT = "windows/s"
HEADS, HEAD_DIM, TEXT = 20, 128, 58

WORKLOADS = {
    # name: (grid, num_windows, shifted, precision, description)
    "cfg4": ((21, 64, 64), (6, 8, 8), 0, "bf16",
             "81x1024x1024 video -> 21x64x64 latent grid, 4x8x8 windows (num_windows 6,8,8), unshifted"),
    "cfg4-shifted": ((21, 64, 64), (6, 8, 8), 1, "bf16",
                     "21x64x64 grid, 4x8x8 windows shifted by (2,4,4), partial edge windows"),
    "cfg5": ((9, 45, 80), (3, 6, 10), 0, "bf16", "33x720x1280 video -> 9x45x80 grid, adaptive 3x8x8 windows"),
    "cfg5-fp32": ((9, 45, 80), (3, 6, 10), 0, "fp32", "9x45x80 grid, adaptive 3x8x8 windows, fp32 block"),
    "cfg2": ((6, 16, 16), (2, 8, 8), 0, "bf16", "21x256x256 video -> 6x16x16 grid, 3x8x8 windows"),
    "cfg4b": ((21, 64, 64), (21, 8, 8), 0, "bf16", "21x64x64 grid, 1x8x8 windows (num_windows 21,8,8): 1344 windows"),
    "cfg4-f32qkv": ((21, 64, 64), (6, 8, 8), 0, "bf16",
                    "cfg4 fed fp32 QKV in a bf16 block (the reference's promoted fp32 QKV): converted to bf16 "
                    "in the workspace, then the tensor-core kernel"),
}
INPUT_F32 = {"cfg4-f32qkv"}  # workloads whose QKV rows are fp32 although the block is bf16
WORKLOADS["cfg4-prerotated"] = ((21, 64, 64), (6, 8, 8), 0, "bf16",
                                "cfg4 with Q/K rotated by the QKV projection's epilogue "
                                "(awa_qkv_project_rotated): awa_forward_prerotated, no rotation in the attention")
PREROTATED = {"cfg4-prerotated"}


def window_costs(grid, num, shifted):
    """Windows and their lengths (video tokens + text) from the library's plan
    rule (the B200 arm)."""
    import awa_b200

    wins = awa_b200.make_windows(grid, num, bool(shifted))
    lengths = [(w[1] - w[0]) * (w[3] - w[2]) * (w[5] - w[4]) + TEXT for w in wins]
    return wins, lengths


def reference_windows(grid, num, shifted):
    """The same windows from the reference's own make_awa_windows (oracle/_ref),
    so the reference arm loads nothing of the B200 library."""
    from oracle.oracle import Reference

    return Reference().make_windows(grid, num, bool(shifted))


def attention_flops(lengths, heads=HEADS, head_dim=HEAD_DIM):
    return float(sum(4.0 * L * L * head_dim * heads for L in lengths))


def workload_config(name, world, mode="replicas"):
    """The `config` both arms print for a workload (identical keys and values)."""
    grid, num, shifted, precision, desc = WORKLOADS[name]
    n_v = grid[0] * grid[1] * grid[2]
    esize = 2 if precision == "bf16" and name not in INPUT_F32 else 4
    in_bytes = (n_v + TEXT) * 3 * HEADS * HEAD_DIM * esize
    parallelism = (f"sharded: one layer's windows split over {world} GPU(s), NCCL text all-reduce + video all-gather"
                   if mode == "sharded" else f"replicas: {world} independent layer(s), one per GPU")
    return {"workload": name, "description": desc, "grid": list(grid), "num_windows": list(num),
            "shifted": bool(shifted), "heads": HEADS, "head_dim": HEAD_DIM, "text_tokens": TEXT, "rope_dim": 126,
            "precision": precision, "l2": f"inputs {in_bytes / 1e9:.2f} GB per step > 126 MB L2; no flush",
            "parallelism": parallelism}


# ----------------------------------------------------------------------------- CPU baseline
_REF = None
_REF_INPUTS = {}


def _ref_window_worker(args):
    """The reference's CPU chain (Pack -> MMRoPE -> WindowAttention -> Unpack,
    awa_layers.cpp:419-458, 913-953, 1062-1120, 638-689, compiled unmodified in
    oracle/_ref) on windows of the workload, one at a time. A grid of a window's
    size with num_windows (1,1,1) holds exactly that window: the same video
    tokens, the 58 text tokens, the same window-local RoPE coordinates and the
    same attention. Returns (seconds inside the reference forward, windows)."""
    global _REF
    dims_list, heads = args
    import numpy as np

    from oracle.oracle import LayerConfig, Reference

    if _REF is None:
        _REF = Reference()
    seconds = 0.0
    for dims in dims_list:
        cfg = LayerConfig(*dims, 1, 1, 1, text_tokens=TEXT, shifted=0, heads=heads, head_dim=HEAD_DIM)
        key = (tuple(dims), heads)
        if key not in _REF_INPUTS:
            wins = _REF.make_windows(dims, (1, 1, 1), False)
            assert wins == [(0, dims[0], 0, dims[1], 0, dims[2])], (dims, wins)
            rng = np.random.default_rng(sum(dims) * 131 + heads)
            _REF_INPUTS[key] = (rng.standard_normal((cfg.source_tokens, 3, heads, HEAD_DIM), dtype=np.float32),
                                rng.standard_normal((TEXT, 3, heads, HEAD_DIM), dtype=np.float32))
        v, t = _REF_INPUTS[key]
        start = time.perf_counter()
        _REF.chain(cfg, v, t)
        seconds += time.perf_counter() - start
    return seconds, len(dims_list)


def _window_dims(windows):
    return [(w[1] - w[0], w[3] - w[2], w[5] - w[4]) for w in windows]


def cpu_kind():
    from oracle.oracle import Reference

    return "reference" if Reference.available() else "port"


def cpu_baseline_single(name, budget_s=12.0):
    """The reference CPU forward on 1 core, for ~budget_s, on the workload's own
    windows in plan order (a contiguous run of the window list, which cycles
    through every window shape of the layer); value = windows / seconds."""
    grid, num, shifted, _, _ = WORKLOADS[name]
    dims = _window_dims(reference_windows(grid, num, shifted))
    total_s, done = 0.0, 0
    while total_s < budget_s and done < len(dims):
        s, n = _ref_window_worker(([dims[done]], HEADS))
        total_s += s
        done += n
    return {
        "value": done / total_s,
        "unit": UNIT,
        "cores": 1,
        "kind": cpu_kind(),
        "sample": f"windows 0..{done - 1} of the workload's {len(dims)} (plan order, every window shape), each "
                  f"through the reference's Pack->MMRoPE->WindowAttention->Unpack CPU forward with {HEADS} heads x "
                  f"{HEAD_DIM} and {TEXT} text tokens, {total_s:.1f} s on 1 core",
        "seconds": round(total_s, 3),
    }


def run_reference_arm(args, rank, world):
    """--impl reference: the reference's own CPU forward of the AWA chain on
    every host core (one process per core; the reference code is
    single-threaded), rank 0 only. A step runs a fixed deterministic sample of
    the workload's own windows, split over the processes: the whole layer
    (every window once) when that fits the time budget, else the next run of
    the window list in rotation, so that over the timed steps every window
    shape appears in its share. value = windows processed / elapsed."""
    if rank != 0:
        return None
    name = args.workload
    grid, num, shifted, precision, desc = WORKLOADS[name]
    dims = _window_dims(reference_windows(grid, num, shifted))
    W = len(dims)
    cores = os.cpu_count() or 1
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores) as pool:
        # warm-up: every process loads the reference and runs one window
        per_window = []
        for i in range(args.warmup):
            chunk = [[dims[(i * cores + c) % W]] for c in range(cores)]
            res = pool.map(_ref_window_worker, [(c, HEADS) for c in chunk])
            per_window.append(max(r[0] for r in res))
        t_window = max(per_window[-1], 1e-3)
        budget = 150.0  # seconds of timed work
        per_proc = max(1, int(budget / (args.steps * t_window)))
        per_step = min(W, cores * per_proc)
        cursor = 0
        done = 0
        start = time.perf_counter()
        for _ in range(args.steps):
            picks = [dims[(cursor + j) % W] for j in range(per_step)]
            cursor = (cursor + per_step) % W
            chunks = [picks[c::cores] for c in range(cores) if picks[c::cores]]
            res = pool.map(_ref_window_worker, [(c, HEADS) for c in chunks])
            done += sum(n for _, n in res)
        elapsed = time.perf_counter() - start
    value = done / elapsed
    sample = (f"per step {per_step} of the workload's {W} windows ({'the whole layer' if per_step == W else 'the next run of the window list, in rotation'}), "
              f"split over {cores} processes, each window through the reference's "
              f"Pack->MMRoPE->WindowAttention->Unpack CPU forward ({HEADS} heads x {HEAD_DIM}, {TEXT} text tokens)")
    mode = "sharded" if world > 1 else "replicas"
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed * 1000 / args.steps, "higher_is_better": True,
        "scaling": "strong" if mode == "sharded" else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic N(0,1) QKV, seeded", "config": workload_config(name, world, mode),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": cpu_kind(), "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(device_index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(",") for r in out.strip().splitlines() if r.count(",") >= 8]
        sm, sm_max, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            try:
                sm.append(float(r[1]))
                sm_max = float(r[2])
            except ValueError:
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        loaded = [s for s in sm if sm_max and s > 0.5 * sm_max] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": sm_max,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- B200 arm
def measured_peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, source) from MEASURED_PEAKS.json, else the
    profiling recipe's fallback figures."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
        return float(peaks["hbm_gbs"]), float(peaks["bf16_tflops"]), "measured"
    except (OSError, ValueError, KeyError):
        return 6650.0, 1590.0, "fallback"


def clock_device(local_rank):
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    return int(visible.split(",")[local_rank]) if visible else local_rank


def run_sharded(args, rank, world, local_rank):
    """One layer split over the N ranks (awa_forward_sharded: window ranges of
    near-equal cost, or head ranges when windows are few; NCCL all-reduce of the
    text partial sums and all-gather of the video rows). Strong scaling: the
    whole layer is one step at every N."""
    import torch
    import torch.distributed as dist

    import awa_b200

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    name = args.workload
    grid, num, shifted, precision, desc = WORKLOADS[name]
    prec = awa_b200.AWA_PREC_BF16 if precision == "bf16" else awa_b200.AWA_PREC_FP32
    dtype = torch.bfloat16 if precision == "bf16" else torch.float32
    esize = 2 if precision == "bf16" else 4
    wins, lengths = window_costs(grid, num, shifted)
    W = len(lengths)
    flops = attention_flops(lengths)
    n_v = grid[0] * grid[1] * grid[2]
    plan = awa_b200.AwaPlan(*grid, *num, text_tokens=TEXT, shifted=bool(shifted))
    box = [awa_b200.AwaComm.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    comm = awa_b200.AwaComm(box[0], world, rank)
    comm.set_push({"auto": awa_b200.AWA_PUSH_AUTO, "ce": awa_b200.AWA_PUSH_COPY_ENGINES,
                   "kernel": awa_b200.AWA_PUSH_KERNEL}[args.push])
    by_heads, bounds = plan.shard_split(world, HEADS)

    gen = torch.Generator(device=device).manual_seed(1234)  # the same layer on every rank
    video_qkv = torch.randn(n_v, 3, HEADS, HEAD_DIM, device=device, generator=gen).to(dtype)
    text_qkv = torch.randn(TEXT, 3, HEADS, HEAD_DIM, device=device, generator=gen).to(dtype)
    direct = args.exchange == "p2p"
    # p2p: the video output lives in a buffer shared over the ranks, and the
    # attention kernel stores each row into every rank's copy over NVLink;
    # nccl: each rank keeps its own output and NCCL all-gathers the rows
    video_out = (comm.shared_tensor((n_v, HEADS, HEAD_DIM), dtype) if direct else
                 torch.empty(n_v, HEADS, HEAD_DIM, device=device, dtype=dtype))
    text_out = torch.empty(TEXT, HEADS, HEAD_DIM, device=device, dtype=dtype)
    workspace = torch.empty(plan.sharded_workspace_bytes(world, HEADS, HEAD_DIM, dtype), device=device,
                            dtype=torch.uint8)
    stream = torch.cuda.current_stream(device)

    def step(v=video_qkv, t=text_qkv):
        plan.forward_sharded(comm, v, t, prec, out_dtype=dtype, workspace=workspace, video_out=video_out,
                             text_out=text_out, stream=stream)

    def barrier():
        dist.barrier(device_ids=[local_rank])

    clocks = ClockSampler(clock_device(local_rank))
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    awa_b200.device_status()
    awa_b200.profile_reset()
    awa_b200.profile_enable(True)
    barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        step()
    stop.record(stream)
    torch.cuda.synchronize()
    barrier()
    awa_b200.profile_enable(False)
    prof = awa_b200.profile_collect()
    kernel_ms = sum(v[1] for v in prof.values()) / args.steps  # this rank's library kernels per step
    attn_name = next((k for k in prof if k.startswith("awa_attention")), None)
    # the rank's attention per step: one launch, or one per chunk of its bands
    attn_launches, attn_ms_total = prof.get(attn_name, (0, 0.0))
    attn_ms = attn_ms_total / args.steps
    t = torch.tensor([start.elapsed_time(stop), kernel_ms * args.steps], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t[0].item()) / args.steps
    compute_ms_max = float(t[1].item()) / args.steps
    value = W / (ms_per_step / 1000.0)

    # end to end with host buffers: each rank copies from pinned host memory only
    # the QKV rows its windows read (its bands' token runs, awa_shard_runs, and
    # the text rows), runs the sharded layer, and copies its runs of the video
    # output back; rank 0 also copies the text output. Together the ranks move
    # the whole input in and the whole output out every step.
    e2e_ms, e2e_steps = None, 0
    in_bytes = out_bytes = 0
    if not args.no_e2e:
        e2e_steps = max(3, min(args.steps, args.e2e_steps))
        runs = plan.shard_runs(world, HEADS, rank)
        rows = sum(c for _, c in runs)
        row_bytes = HEADS * HEAD_DIM * esize
        # bytes copied per step, summed over the ranks
        nb = torch.tensor([(rows + TEXT) * 3 * row_bytes, (rows + (TEXT if rank == 0 else 0)) * row_bytes],
                          device=device, dtype=torch.float64)
        dist.all_reduce(nb)
        in_bytes, out_bytes = int(nb[0].item()), int(nb[1].item())
        host_v = torch.empty(rows, 3, HEADS, HEAD_DIM, dtype=dtype, pin_memory=True)
        host_o = torch.empty(rows, HEADS, HEAD_DIM, dtype=dtype, pin_memory=True)
        at = 0
        for first, count in runs:
            host_v[at:at + count].copy_(video_qkv[first:first + count])
            at += count
        host_t = torch.empty(text_qkv.shape, dtype=dtype, pin_memory=True)
        host_t.copy_(text_qkv)
        host_ot = torch.empty(text_out.shape, dtype=dtype, pin_memory=True)
        dev_v = torch.zeros_like(video_qkv)
        dev_t = torch.empty_like(text_qkv)

        def e2e_step():
            at = 0
            for first, count in runs:
                dev_v[first:first + count].copy_(host_v[at:at + count], non_blocking=True)
                at += count
            dev_t.copy_(host_t, non_blocking=True)
            step(dev_v, dev_t)
            at = 0
            for first, count in runs:
                host_o[at:at + count].copy_(video_out[first:first + count], non_blocking=True)
                at += count
            if rank == 0:
                host_ot.copy_(text_out, non_blocking=True)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        te = torch.tensor([e0.elapsed_time(e1)], device=device, dtype=torch.float64)
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = float(te.item()) / e2e_steps
    clock = clocks.stop()
    awa_b200.device_status()
    if direct:
        comm.free_shared(video_out)
    comm.destroy()

    hbm_peak, tensor_peak, peak_src = measured_peaks()
    if by_heads:
        share_rows, share_frac = n_v, (bounds[rank + 1] - bounds[rank]) / HEADS
    else:
        share_rows = plan.range_video_rows(bounds[rank], bounds[rank + 1])
        share_frac = 1.0
    share_heads = HEADS * share_frac
    alg_bytes = int((share_rows + TEXT) * 4 * share_heads * HEAD_DIM * esize)
    achieved = alg_bytes / (attn_ms / 1000.0) / 1e9 if attn_ms > 0 else 0.0
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": precision, "data": "synthetic N(0,1) QKV, seeded",
            "config": workload_config(name, world, "sharded"),
            "windows": W, "attn_tflops": round(flops / (ms_per_step / 1000.0) / 1e12, 2),
            "sharded": {"split": "heads" if by_heads else "windows", "bounds": bounds,
                        "exchange": ("video rows pushed into every rank's output in a buffer shared over the ranks "
                                     f"(push {args.push}: copy engines chunk by chunk behind the attention with one "
                                     "peer, the SM push kernel after it with three or more); NCCL all-reduce of the "
                                     "text partial sums" if direct else
                                     "NCCL all-gather of the video rows, all-reduce of the text partial sums"),
                        "compute_ms_max": round(compute_ms_max, 5),
                        "collective_and_copies_ms": round(ms_per_step - compute_ms_max, 5),
                        "kernel_only_value": round(W / (compute_ms_max / 1000.0), 2)},
            "gpu_launches": sum(v[0] for v in prof.values()),
            "e2e": None if e2e_ms is None else {
                "value": round(W / (e2e_ms / 1000.0), 2), "unit": UNIT, "h2d_bytes_per_step": in_bytes,
                "d2h_bytes_per_step": out_bytes, "steps": e2e_steps, "ms_per_step": round(e2e_ms, 4),
                "how": "each rank copies in the QKV rows of its windows (its token runs + the text rows) and "
                       "copies out its runs of the video output; rank 0 the text output"},
            "roofline": {"bound": "hbm", "kernel": attn_name, "achieved": round(achieved, 1), "peak": hbm_peak,
                         "unit": "GB/s", "frac": round(achieved / hbm_peak, 4), "traffic": None,
                         "peak_source": peak_src, "algorithmic_bytes": alg_bytes, "kernel_ms": round(attn_ms, 5),
                         "launches_per_step": attn_launches // args.steps,
                         "note": "rank 0's share of the layer; kernel_ms = its attention launches of one step"},
            "clocks": clock,
            "profile": {k: {"launches": v[0], "ms": round(v[1], 4)} for k, v in prof.items()},
        }
    return line


def run_b200(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import awa_b200

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    name = args.workload
    grid, num, shifted, precision, desc = WORKLOADS[name]
    prec = awa_b200.AWA_PREC_BF16 if precision == "bf16" else awa_b200.AWA_PREC_FP32
    dtype = torch.bfloat16 if precision == "bf16" else torch.float32
    in_dtype = torch.float32 if name in INPUT_F32 else dtype
    esize = 2 if precision == "bf16" else 4
    in_esize = 4 if in_dtype == torch.float32 else 2
    wins, lengths = window_costs(grid, num, shifted)
    W = len(lengths)
    flops = attention_flops(lengths)
    n_v = grid[0] * grid[1] * grid[2]
    plan = awa_b200.AwaPlan(*grid, *num, text_tokens=TEXT, shifted=bool(shifted))
    kernel_kind = plan.attention_kernel_kind(prec, HEADS, HEAD_DIM, in_dtype)

    gen = torch.Generator(device=device).manual_seed(1234 + rank)
    video_qkv = torch.randn(n_v, 3, HEADS, HEAD_DIM, device=device, generator=gen).to(in_dtype)
    text_qkv = torch.randn(TEXT, 3, HEADS, HEAD_DIM, device=device, generator=gen).to(in_dtype)
    video_out = torch.empty(n_v, HEADS, HEAD_DIM, device=device, dtype=dtype)
    text_out = torch.empty(TEXT, HEADS, HEAD_DIM, device=device, dtype=dtype)
    workspace = torch.empty(plan.workspace_bytes(HEADS, HEAD_DIM, prec, in_dtype), device=device, dtype=torch.uint8)
    stream = torch.cuda.current_stream(device)

    forward = plan.forward_prerotated if name in PREROTATED else plan.forward

    def step():
        forward(video_qkv, text_qkv, prec, out_dtype=dtype, workspace=workspace, video_out=video_out,
                text_out=text_out, stream=stream)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    clocks = ClockSampler(local_rank if "CUDA_VISIBLE_DEVICES" not in os.environ else
                          int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local_rank]))
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    awa_b200.device_status()

    # ---- device-resident timed region (inputs 1.3 GB >> 126 MB L2: no flush needed)
    awa_b200.profile_reset()
    awa_b200.profile_enable(True)
    barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        step()
    stop.record(stream)
    torch.cuda.synchronize()
    barrier()
    awa_b200.profile_enable(False)
    prof = awa_b200.profile_collect()
    elapsed_ms = start.elapsed_time(stop)
    t = torch.tensor([elapsed_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    ms_per_step = max_ms / args.steps
    value = W * world / (ms_per_step / 1000.0)
    launches = sum(v[0] for v in prof.values())

    # ---- end to end through the C ABI with host buffers (skipped by --no-e2e,
    # for profiler captures that should hold little device memory):
    # awa_forward_host takes the pinned host QKV and output buffers and
    # enqueues copy in, forward and copy out on its stream. Steps alternate
    # over two streams and two device workspaces, as a stream of layers would
    # run: the copy in of step i + 1 overlaps the forward of step i and the copy
    # out of step i - 1 (the host link is full duplex). Every step copies its
    # whole input in and its whole output out inside the timed region.
    e2e_ms, e2e_steps = None, 0
    if not args.no_e2e:
        e2e_steps = max(3, min(args.steps, args.e2e_steps))
        host_v = torch.empty(video_qkv.shape, dtype=video_qkv.dtype, pin_memory=True)
        host_t = torch.empty(text_qkv.shape, dtype=text_qkv.dtype, pin_memory=True)
        host_v.copy_(video_qkv)
        host_t.copy_(text_qkv)
        outs = [(torch.empty(video_out.shape, dtype=dtype, pin_memory=True),
                 torch.empty(text_out.shape, dtype=dtype, pin_memory=True)) for _ in range(2)]
        streams = [torch.cuda.Stream(device), torch.cuda.Stream(device)]
        need = plan.host_workspace_bytes(prec, in_dtype, dtype, HEADS, HEAD_DIM)
        spaces = [torch.empty(need, dtype=torch.uint8, device=device) for _ in range(2)]

        def e2e_step(i):
            b = i % 2
            plan.forward_host(host_v, host_t, outs[b][0], outs[b][1], prec, workspace=spaces[b], stream=streams[b])

        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier()
        e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        for st in streams:
            st.wait_event(e_start)
        for i in range(e2e_steps):
            e2e_step(i)
        for st in streams:
            done = torch.cuda.Event()
            done.record(st)
            stream.wait_event(done)
        e_stop.record(stream)
        torch.cuda.synchronize()
        barrier()
        te = torch.tensor([e_start.elapsed_time(e_stop)], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = float(te.item()) / e2e_steps
    clock = clocks.stop()
    awa_b200.device_status()

    # ---- roofline of the dominant kernel
    attn_name = next((k for k in prof if k.startswith("awa_attention")), None)
    attn_launches, attn_ms_total = prof.get(attn_name, (0, 0.0))
    attn_ms = attn_ms_total / max(attn_launches, 1)
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    hbm_peak = peaks.get("hbm_gbs")
    tensor_peak = peaks.get("bf16_tflops")
    peak_src = "measured" if hbm_peak else "fallback"
    hbm_peak = hbm_peak or 6650.0
    tensor_peak = tensor_peak or 1590.0
    in_bytes = (n_v + TEXT) * 3 * HEADS * HEAD_DIM * in_esize
    out_bytes = (n_v + TEXT) * HEADS * HEAD_DIM * esize
    # the attention kernel reads bf16 rows (for fp32 inputs: the converted copy)
    alg_bytes = (n_v + TEXT) * 3 * HEADS * HEAD_DIM * (2 if kernel_kind == 1 else esize) + out_bytes
    achieved_gbs = alg_bytes / (attn_ms / 1000.0) / 1e9
    achieved_tflops = flops / (attn_ms / 1000.0) / 1e12
    traffic = recorded_traffic(f"{name}:{attn_name}")
    roofline = {
        "bound": "hbm", "kernel": attn_name, "achieved": round(achieved_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
        "frac": round(achieved_gbs / hbm_peak, 4), "traffic": traffic, "peak_source": peak_src,
        "algorithmic_bytes": alg_bytes, "kernel_ms": round(attn_ms, 5),
        "tensor": {"achieved_tflops": round(achieved_tflops, 1), "peak_tflops": tensor_peak,
                   "frac": round(achieved_tflops / tensor_peak, 4), "flops": flops},
    }

    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": precision, "data": "synthetic N(0,1) QKV, seeded",
            "config": workload_config(name, world),
            "windows": W, "attention_kernel": "tcgen05" if kernel_kind == 1 else "simt",
            "attn_tflops": round(flops * world / (ms_per_step / 1000.0) / 1e12, 2),
            "gpu_launches": launches,
            "e2e": None if e2e_ms is None else {
                "value": round(W * world / (e2e_ms / 1000.0), 2), "unit": UNIT, "h2d_bytes_per_step": in_bytes,
                "d2h_bytes_per_step": out_bytes, "steps": e2e_steps, "ms_per_step": round(e2e_ms, 4)},
            "roofline": roofline,
            "clocks": clock,
            "profile": {k: {"launches": v[0], "ms": round(v[1], 4)} for k, v in prof.items()},
        }
    return line


MODEL_DIM = 2560  # vid_dim of the 3B DiT: proj_qkv is 2560 -> 3 x 20 x 128


def recorded_traffic(key):
    """DRAM bytes (read + write) of one launch, from the ncu capture recorded
    in profiles/traffic.json under "<workload>:<kernel>", or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(key)
    except (OSError, ValueError):
        return None


def run_qkv_proj(args, rank, world, local_rank):
    """--stage qkv-proj: the producer of the AWA input (awa_qkv_project) on the
    workload's video rows: x [N_v, 2560] W^T -> [N_v, 7680] with the per-head
    RMSNorm of Q and K. --stage out-proj: the consumer of the AWA output
    (awa_out_project): the AWA output [N_v, 2560] W_out^T + bias, times the Ada
    gate, plus the residual [N_v, 2560]. A step is one GEMM, inputs resident in
    HBM."""
    import torch
    import torch.distributed as dist

    import awa_b200

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    grid = WORKLOADS[args.workload][0]
    n_v = grid[0] * grid[1] * grid[2]
    producer = args.stage in ("qkv-proj", "qkv-proj-rope")
    rotated = args.stage == "qkv-proj-rope"
    n_out = 3 * HEADS * HEAD_DIM if producer else MODEL_DIM
    gen = torch.Generator(device=device).manual_seed(4321 + rank)
    x = torch.randn(n_v, MODEL_DIM, device=device, generator=gen).bfloat16()
    w = (torch.randn(n_out, MODEL_DIM, device=device, generator=gen) / math.sqrt(MODEL_DIM)).bfloat16()
    stream = torch.cuda.current_stream(device)
    if producer:
        gq = 1.0 + 0.25 * torch.randn(HEAD_DIM, device=device, generator=gen)
        gk = 1.0 + 0.25 * torch.randn(HEAD_DIM, device=device, generator=gen)
        out = torch.empty(n_v, 3, HEADS, HEAD_DIM, device=device, dtype=torch.bfloat16)

        if rotated:
            _, num, shifted, _, _ = WORKLOADS[args.workload]
            plan = awa_b200.AwaPlan(*grid, *num, text_tokens=TEXT, shifted=bool(shifted))

            def step():
                awa_b200.qkv_project_rotated(x, w, gq, gk, 1e-5, HEADS, plan, awa_b200.AWA_BRANCH_VIDEO, out=out,
                                             stream=stream)
        else:
            def step():
                awa_b200.qkv_project(x, w, gq, gk, 1e-5, HEADS, out=out, stream=stream)
    else:
        bias = 0.1 * torch.randn(n_out, device=device, generator=gen)
        gate = 0.2 * torch.randn(n_out, device=device, generator=gen)
        resid = torch.randn(n_v, n_out, device=device, generator=gen).bfloat16()
        out = torch.empty(n_v, n_out, device=device, dtype=torch.bfloat16)

        def step():
            awa_b200.out_project(x, w, bias, gate, resid, out=out, stream=stream)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    clocks = ClockSampler(local_rank if "CUDA_VISIBLE_DEVICES" not in os.environ else
                          int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local_rank]))
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    awa_b200.device_status()
    awa_b200.profile_reset()
    awa_b200.profile_enable(True)
    barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        step()
    stop.record(stream)
    torch.cuda.synchronize()
    barrier()
    clock = clocks.stop()
    awa_b200.profile_enable(False)
    prof = awa_b200.profile_collect()
    t = torch.tensor([start.elapsed_time(stop)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item()) / args.steps
    awa_b200.device_status()
    flops = 2.0 * n_v * MODEL_DIM * n_out
    kernel_name = ("awa_qkv_project_rotated" if rotated else "awa_qkv_project") if producer else "awa_out_project"
    launches, kernel_total = prof.get(kernel_name, (0, 0.0))
    kernel_ms = kernel_total / max(launches, 1)
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    # a seconds-long loop of a dense GEMM runs under the power cap: the sustained peak
    tensor_peak = peaks.get("bf16_tflops_sustained")
    peak_src = "measured sustained" if tensor_peak else "fallback sustained"
    tensor_peak = tensor_peak or 1400.0
    achieved = flops / (kernel_ms / 1000.0) / 1e12
    # context: the library GEMM alone (cuBLAS through torch.mm, no RMSNorm) on the same operands
    gemm_out = torch.empty(n_v, n_out, device=device, dtype=torch.bfloat16)
    for _ in range(args.warmup):
        torch.mm(x, w.t(), out=gemm_out)
    torch.cuda.synchronize()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    for _ in range(args.steps):
        torch.mm(x, w.t(), out=gemm_out)
    g1.record(stream)
    torch.cuda.synchronize()
    gemm_ms = g0.elapsed_time(g1) / args.steps
    return {
        "metric": (("QKV projection + per-head RMSNorm + MMRoPE (producer of the pre-rotated AWA input)" if rotated
                    else "QKV projection + per-head RMSNorm (producer of the AWA input)") if producer else
                   "proj_out + Ada gate + residual (consumer of the AWA output)") + " TFLOP/s per B200",
        "value": round(flops * world / (ms_per_step / 1000.0) / 1e12, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1) x, W ~ N(0, 1/2560)",
        "config": {"workload": f"{args.workload}-{args.stage}", "tokens": n_v, "in_features": MODEL_DIM,
                   "out_features": n_out, "heads": HEADS, "head_dim": HEAD_DIM,
                   "l2": f"x {n_v * MODEL_DIM * 2 / 1e9:.2f} GB + out {n_v * n_out * 2 / 1e9:.2f} GB per step > 126 MB L2"},
        "gpu_launches": sum(v[0] for v in prof.values()),
        "roofline": {"bound": "tensor", "kernel": kernel_name, "achieved": round(achieved, 1),
                     "peak": tensor_peak, "unit": "TFLOP/s", "frac": round(achieved / tensor_peak, 4),
                     "traffic": recorded_traffic(f"{args.workload}-{args.stage}:{kernel_name}"),
                     "peak_source": peak_src, "kernel_ms": round(kernel_ms, 5),
                     "flops": flops},
        "library_gemm": {"what": "cuBLAS GEMM alone via torch.mm (no epilogue), same operands", "ms": round(gemm_ms, 5),
                         "tflops": round(flops / (gemm_ms / 1000.0) / 1e12, 1)},
        "clocks": clock,
    }


def run_layers(args, rank, world, local_rank):
    """--stage layers: the reference's four-layer chain as separate passes
    (Pack -> MMRoPE -> WindowAttention -> Unpack, the path an ncnn graph with the
    four layer classes takes) on the workload, each kernel timed by the
    library's launch profiler and set against the HBM peak with its algorithmic
    bytes: the gather (Pack), the rotation (MMRoPE), the packed attention, the
    video scatter and the text mean. A step is one pass of the chain; inputs
    resident in HBM."""
    import torch
    import torch.distributed as dist

    import awa_b200

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    grid, num, shifted, precision, _ = WORKLOADS[args.workload]
    bf16 = precision == "bf16"
    dtype = torch.bfloat16 if bf16 else torch.float32
    esize = 2 if bf16 else 4
    prec = awa_b200.AWA_PREC_BF16 if bf16 else awa_b200.AWA_PREC_FP32
    n_v = grid[0] * grid[1] * grid[2]
    plan = awa_b200.AwaPlan(*grid, *num, TEXT, bool(shifted))
    info = plan.info
    gen = torch.Generator(device=device).manual_seed(777 + rank)
    video = torch.randn(n_v, 3, HEADS, HEAD_DIM, device=device, generator=gen).to(dtype)
    text = torch.randn(TEXT, 3, HEADS, HEAD_DIM, device=device, generator=gen).to(dtype)
    stream = torch.cuda.current_stream(device)

    def step():
        packed, _ = plan.pack(video, text, stream=stream)
        roped = plan.mmrope(packed, stream=stream)
        attended = plan.window_attention(roped, prec, stream=stream)
        return plan.unpack(attended, stream=stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    awa_b200.device_status()
    awa_b200.profile_reset()
    awa_b200.profile_enable(True)
    clocks = ClockSampler(local_rank if "CUDA_VISIBLE_DEVICES" not in os.environ else
                          int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local_rank]))
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        step()
    stop.record(stream)
    torch.cuda.synchronize()
    clock = clocks.stop()
    awa_b200.profile_enable(False)
    prof = awa_b200.profile_collect()
    awa_b200.device_status()
    ms_per_step = start.elapsed_time(stop) / args.steps
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            hbm_peak, peak_src = float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        hbm_peak, peak_src = 6650.0, "fallback"
    s_rows, w, row = info.sequence_tokens, info.window_count, HEADS * HEAD_DIM
    attn_name = "awa_attention_tc_packed" if bf16 else "awa_attention_simt_packed"
    # algorithmic bytes per launch: each source row read once, each output row written once
    alg = {
        "awa_pack": (n_v + TEXT) * 3 * row * esize + s_rows * 3 * row * esize + (w + 1) * 4,
        "awa_mmrope": 2 * s_rows * 3 * row * esize,
        attn_name: s_rows * 3 * row * esize + s_rows * row * esize,
        "awa_unpack_video": 2 * n_v * row * esize,
        "awa_text_reduce": w * TEXT * row * esize + TEXT * row * esize,
    }
    kernels = {}
    for name, nbytes in alg.items():
        launches, total = prof.get(name, (0, 0.0))
        if not launches:
            continue
        kms = total / launches
        gbs = nbytes / (kms / 1000.0) / 1e9
        kernels[name] = {"ms": round(kms, 5), "bytes": nbytes, "gbs": round(gbs, 1), "frac": round(gbs / hbm_peak, 4)}
    return {
        "metric": "AWA layer chain as separate passes (Pack, MMRoPE, WindowAttention, Unpack) windows/s per B200",
        "value": round(info.window_count * world / (ms_per_step / 1000.0), 2), "unit": "windows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if bf16 else "f32", "data": "synthetic N(0,1) QKV",
        "config": {"workload": f"{args.workload}-layers", "grid": list(grid), "num_windows": list(num),
                   "shifted": bool(shifted), "windows": info.window_count, "sequence_rows": s_rows},
        "gpu_launches": sum(v[0] for v in prof.values()),
        "kernels": kernels, "hbm_peak_gbs": hbm_peak, "peak_source": peak_src, "clocks": clock,
    }


STACK_BLOCKS, STACK_FP32_BLOCKS = 32, 9


def run_stack(args, rank, world, local_rank):
    """--stage stack: the attention path of a 32-block DiT step through the
    block-stack driver (awa_stack): per block the QKV projection with Q/K
    RMSNorm, the AWA chain (fp32 in the first 9 blocks, bf16 after, odd blocks
    shifted) and proj_out + gate + residual, the residual stream carried from
    block to block. Timed three ways: with a host wait after every block (the
    reference's submit-and-wait per block), on one stream with no wait, and as
    one CUDA graph. A step is one 32-block pass; inputs resident in HBM."""
    import torch
    import torch.distributed as dist

    import awa_b200

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    grid, num, _, _, _ = WORKLOADS[args.workload]
    n_v = grid[0] * grid[1] * grid[2]
    lib = awa_b200.library()
    gen = torch.Generator(device=device).manual_seed(99 + rank)

    def rnd(*shape, scale=1.0):
        return torch.randn(*shape, device=device, generator=gen) * scale

    sets = [{"wqkv": rnd(3 * MODEL_DIM, MODEL_DIM, scale=MODEL_DIM ** -0.5).bfloat16(),
             "wout": rnd(MODEL_DIM, MODEL_DIM, scale=MODEL_DIM ** -0.5).bfloat16(),
             "gq": 1.0 + 0.2 * rnd(HEAD_DIM), "gk": 1.0 + 0.2 * rnd(HEAD_DIM),
             "bias": 0.02 * rnd(MODEL_DIM), "gate": 0.1 * rnd(MODEL_DIM)} for _ in range(4)]
    x0, t0 = rnd(n_v, MODEL_DIM).bfloat16(), rnd(TEXT, MODEL_DIM).bfloat16()
    xv = [torch.empty_like(x0) for _ in range(2)]
    xt = [torch.empty_like(t0) for _ in range(2)]
    qkv = {dt: (torch.empty(n_v, 3, HEADS, HEAD_DIM, device=device, dtype=dt),
                torch.empty(TEXT, 3, HEADS, HEAD_DIM, device=device, dtype=dt))
           for dt in (torch.float32, torch.bfloat16)}
    attn_v = torch.empty(n_v, MODEL_DIM, device=device, dtype=torch.bfloat16)
    attn_t = torch.empty(TEXT, MODEL_DIM, device=device, dtype=torch.bfloat16)
    state = {"cur": 0, "sync": False}
    dim = MODEL_DIM

    def hook(stage, io, handle):
        w, cur = sets[io.block % 4], state["cur"]
        if stage == awa_b200.AWA_STACK_BEFORE:
            fp32 = io.precision == awa_b200.AWA_PREC_FP32
            qv, qt = qkv[torch.float32 if fp32 else torch.bfloat16]
            code = awa_b200.AWA_F32 if fp32 else awa_b200.AWA_BF16
            for x, q, rows in ((xv[cur], qv, n_v), (xt[cur], qt, TEXT)):
                if lib.awa_qkv_project(rows, dim, HEADS, HEAD_DIM, x.data_ptr(), dim, w["wqkv"].data_ptr(), dim,
                                       w["gq"].data_ptr(), w["gk"].data_ptr(), 1e-5, code, q.data_ptr(), 3 * dim,
                                       handle):
                    return 1
            io.in_dtype = code
            io.video_qkv, io.video_token_stride, io.video_qkv_stride = qv.data_ptr(), 3 * dim, dim
            io.text_qkv, io.text_token_stride, io.text_qkv_stride = qt.data_ptr(), 3 * dim, dim
            io.out_dtype = awa_b200.AWA_BF16
            io.video_out, io.video_out_stride = attn_v.data_ptr(), dim
            io.text_out, io.text_out_stride = attn_t.data_ptr(), dim
            return 0
        nxt = 1 - cur
        for a, x, y, rows in ((attn_v, xv[cur], xv[nxt], n_v), (attn_t, xt[cur], xt[nxt], TEXT)):
            if lib.awa_out_project(rows, dim, dim, a.data_ptr(), dim, w["wout"].data_ptr(), dim, w["bias"].data_ptr(),
                                   w["gate"].data_ptr(), x.data_ptr(), dim, awa_b200.AWA_BF16, awa_b200.AWA_BF16,
                                   y.data_ptr(), dim, handle):
                return 1
        state["cur"] = nxt
        if state["sync"]:
            stream.synchronize()  # the reference waits for every block on the host
        return 0

    params = [{"source_t": -1, "source_h": -1, "source_w": -1, "windows_t": num[0], "windows_h": num[1],
               "windows_w": num[2], "text_tokens": TEXT, "shifted": b % 2, "rope_dim": 126}
              for b in range(STACK_BLOCKS)]
    stack = awa_b200.AwaStack(params, runtime_spec=grid, fp32_blocks=STACK_FP32_BLOCKS, heads=HEADS,
                              head_dim=HEAD_DIM)
    stream = torch.cuda.Stream(device)

    def reset():
        xv[0].copy_(x0)
        xt[0].copy_(t0)
        state["cur"] = 0

    with torch.cuda.stream(stream):
        reset()
        stack.run(hook, stream)
        reset()
        graph = stack.capture(hook, stream)
    stream.synchronize()
    awa_b200.device_status()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def timed(mode):
        state["sync"] = mode == "host_sync"
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                reset()
                graph.launch(stream) if mode == "graph" else stack.run(hook, stream)
        stream.synchronize()
        barrier()
        total = 0.0
        for _ in range(args.steps):
            with torch.cuda.stream(stream):
                reset()
                start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record(stream)
                graph.launch(stream) if mode == "graph" else stack.run(hook, stream)
                stop.record(stream)
            stop.synchronize()
            total += start.elapsed_time(stop)
        barrier()
        state["sync"] = False
        return total / args.steps

    clocks = ClockSampler(local_rank if "CUDA_VISIBLE_DEVICES" not in os.environ else
                          int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local_rank]))
    ms = {mode: timed(mode) for mode in ("host_sync", "stream", "graph")}
    clock = clocks.stop()
    awa_b200.device_status()
    if world > 1:
        t = torch.tensor([ms["graph"]], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms["graph"] = float(t.item())
    del graph
    plans, ws = stack.info()
    return {
        "metric": "DiT step attention path (32 blocks: QKV proj + RMSNorm, AWA, proj_out + gate + residual) ms",
        "value": round(ms["graph"], 4), "unit": "ms", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms["graph"], 4), "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 (fp32 in blocks 0-8)", "data": "synthetic residual stream, random weights",
        "config": {"workload": f"{args.workload}-stack", "grid": list(grid), "num_windows": list(num),
                   "blocks": STACK_BLOCKS, "fp32_blocks": STACK_FP32_BLOCKS, "plans": plans,
                   "workspace_bytes": ws},
        "modes_ms": {k: round(v, 4) for k, v in ms.items()},
        # per block: 2 QKV projections, attention + text mean, 2 output projections; 3 timed modes
        "gpu_launches": STACK_BLOCKS * 6 * args.steps * 3,
        "clocks": clock,
    }


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=200)
    parser.add_argument("--warmup", type=int, default=10)
    parser.add_argument("--impl", default="b200", choices=["b200", "reference"])
    parser.add_argument("--workload", default="cfg4", choices=sorted(WORKLOADS))
    parser.add_argument("--e2e-steps", type=int, default=20)
    parser.add_argument("--push", default="auto", choices=["auto", "ce", "kernel"],
                        help="p2p exchange: copy engines (ce), the SM push kernel, or auto (ce with one peer)")
    parser.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                        help="sharded mode: p2p = the attention kernel stores video rows into every rank's output "
                             "(shared buffer); nccl = NCCL all-gather of the rows")
    parser.add_argument("--mode", default=None, choices=["sharded", "replicas"],
                        help="N > 1: sharded (default) splits one layer over the N GPUs with NCCL (strong scaling); "
                             "replicas runs an independent layer per GPU (weak scaling)")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg (profiler captures)")
    parser.add_argument("--stage", default="awa",
                        choices=["awa", "qkv-proj", "qkv-proj-rope", "out-proj", "stack", "layers"],
                        help="awa: the AWA layer (the headline); qkv-proj / out-proj: its input's producer / "
                             "its output's consumer; stack: the attention path of 32 blocks via the stack driver; layers: "
                             "the four layers as separate passes, per-kernel HBM throughput")
    args = parser.parse_args()
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        line = run_reference_arm(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist

    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.stage in ("qkv-proj", "qkv-proj-rope", "out-proj", "stack", "layers"):
            runner = {"stack": run_stack, "layers": run_layers}.get(args.stage, run_qkv_proj)
            line = runner(args, rank, world, local_rank)
            if rank == 0:
                print(json.dumps(line), flush=True)
            return
        mode = args.mode or ("sharded" if world > 1 else "replicas")
        line = (run_sharded if mode == "sharded" else run_b200)(args, rank, world, local_rank)
        if rank == 0:
            if world == 1 and not args.no_cpu_baseline:
                line["cpu_baseline"] = cpu_baseline_single(args.workload)
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
