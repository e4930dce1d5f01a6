"""Benchmark of the firepit_b200 hot path (one JSON line on rank 0).

Default workload ("gemv"): NVFP4 decode GEMV, W [4096 x
4096] from N(0, 0.02) quantized to NVFP4 (one global per matrix), x bf16
[1, 4096] from N(0, 1) seed 0, y bf16.  One step is one decode-style sweep
over 64*g distinct weight matrices (g = number of GPUs): each matrix is split
along N (rows) over the g ranks, every rank computes its row slice of all
64*g GEMVs and the slices are all-gathered once per step (NCCL).  Each rank
therefore streams 64 * 9.45 MB = 605 MB of weights per step at every g
(inputs larger than L2: nothing is re-read from L2 across steps); per-GPU work
is fixed as g grows ("weak").

  value  device-resident GB/s (algorithmic bytes of all ranks / max step time),
         the step replayed as one CUDA graph per rank;
  e2e    the same metric through the public Python API (firepit_b200.gemv,
         ctypes C ABI) with x copied from pinned host memory each step and y
         copied back, no graph.

--impl reference times the reference's host path (the CPU restatement of
kernels src/gemv/nvfp4.rs:34-59 in oracle/, OpenMP over all host cores) on a
bounded sample of the same workload, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

ROWS = COLS = 4096
MATS_PER_GPU = 64
# Algorithmic bytes of one 4096x4096 GEMV (config 0): packed + scales + global + x + y.
GEMV_BYTES = ROWS * COLS // 2 + ROWS * COLS // 16 + 4 + COLS * 2 + ROWS * 2


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", choices=["gemv"], default="gemv")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the cpu_baseline sample")
    return p.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def emit(obj):
    print(json.dumps(obj), flush=True)


# ---- clocks -------------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = []
        for line in (self.out or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                try:
                    rows.append((float(f[1]), float(f[2]), float(f[3]), f[5:9]))
                except ValueError:
                    pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        loaded = [r for r in rows if r[2] > 200.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(loaded)}


# ---- reference arm -------------------------------------------------------------------------
def reference_arm(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import numpy as np

    from oracle import oracle as O
    w = O.synth_normal(ROWS * COLS, seed=0, stream=1, std=0.02).reshape(ROWS, COLS)
    packed, scales, g = O.nvfp4_quantize(w)
    x = O.bf16_to_f32(O.bf16_bits(O.synth_normal(COLS, seed=0, stream=0)))
    # Size the per-step sample (rows of the matrix) so that warmup + steps
    # take about a minute on this host.
    t0 = time.perf_counter()
    O.nvfp4_gemv_f32(packed, scales, g, ROWS, COLS, x)
    full = max(time.perf_counter() - t0, 1e-4)
    budget = 60.0 / max(args.steps + args.warmup, 1)
    rows = int(min(ROWS, max(16, ROWS * budget / full))) // 16 * 16 or 16
    p, s, gg = packed[: rows * COLS // 2], scales[: rows * COLS // 16], g[:rows]
    for _ in range(args.warmup):
        O.nvfp4_gemv_f32(p, s, gg, rows, COLS, x)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.nvfp4_gemv_f32(p, s, gg, rows, COLS, x)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    bytes_ = rows * COLS // 2 + rows * COLS // 16 + 4 + COLS * 2 + rows * 2
    gbs = bytes_ / dt / 1e9
    cores = O.num_threads()
    sample = f"{rows} of {ROWS} rows of one {ROWS}x{COLS} NVFP4 GEMV per step (oracle f32 kernel order, OpenMP)"
    emit({"impl": "reference", "metric": "NVFP4 GEMV HBM GB/s", "value": gbs, "unit": "GB/s", "n_gpus": args.gpus,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
          "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Philox N(0,1)/N(0,0.02))",
          "config": {"workload": "config0 NVFP4 GEMV 4096x4096, x bf16 [1,4096] N(0,1) seed 0, W N(0,0.02)",
                     "sample_rows": rows},
          "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
          "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})


def cpu_baseline(seconds: float):
    """The reference's host path (oracle port) on this box's cores: full
    config-0 GEMVs repeated for about `seconds`."""
    from oracle import oracle as O
    w = O.synth_normal(ROWS * COLS, seed=0, stream=1, std=0.02).reshape(ROWS, COLS)
    packed, scales, g = O.nvfp4_quantize(w)
    x = O.bf16_to_f32(O.bf16_bits(O.synth_normal(COLS, seed=0, stream=0)))
    O.nvfp4_gemv_f32(packed, scales, g, ROWS, COLS, x)
    n, t0 = 0, time.perf_counter()
    while n < 3 or time.perf_counter() - t0 < seconds:
        O.nvfp4_gemv_f32(packed, scales, g, ROWS, COLS, x)
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": GEMV_BYTES / dt / 1e9, "unit": "GB/s", "cores": O.num_threads(), "kind": "port",
            "sample": f"{n} full 4096x4096 NVFP4 GEMVs (oracle f32 kernel order, OpenMP), {dt * 1e3:.2f} ms each"}


# ---- our arm ---------------------------------------------------------------------------------
def load_traffic():
    f = ROOT / "profiles" / "gemv_nvfp4_config0.json"
    if f.exists():
        try:
            return json.loads(f.read_text()).get("dram_bytes_per_launch")
        except Exception:
            return None
    return None


def measured_peak():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        try:
            return float(json.loads(f.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def ours_arm(args):
    import torch
    import torch.distributed as dist

    import firepit_b200 as F

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    g = world
    mats = MATS_PER_GPU * g
    rows_per_rank = ROWS // g
    r0 = rank * rows_per_rank

    # ---- weights: every rank quantizes each full matrix (one global per
    # matrix, as the unsharded reference would) and keeps its row slice.
    slices = []
    for c in range(mats):
        w = F.synth_normal((ROWS, COLS), seed=0, stream_id=1 + c, std=0.02, device=dev)
        packed, scales, globals_ = F.quantize_nvfp4(w)
        del w
        slices.append(F.Nvfp4Matrix.from_device(packed[r0:r0 + rows_per_rank].contiguous(),
                                                scales[r0:r0 + rows_per_rank].contiguous(),
                                                globals_[r0:r0 + rows_per_rank].contiguous(), rows_per_rank, COLS))
        del packed, scales, globals_
    torch.cuda.synchronize()
    x = F.synth_normal((1, COLS), seed=0, stream_id=0, dtype=torch.bfloat16, device=dev)
    y_local = torch.empty(mats, rows_per_rank, dtype=torch.bfloat16, device=dev)
    y_all = torch.empty(g, mats, rows_per_rank, dtype=torch.bfloat16, device=dev)

    def gemvs(stream_handle):
        for c in range(mats):
            F._native.call("fpb_nvfp4_gemv", slices[c].handle, 0, 0, x.data_ptr(), F._native.FPB_BF16,
                           y_local[c].data_ptr(), F._native.FPB_BF16, 1, stream_handle)

    # warm every code path once outside capture
    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        gemvs(s.cuda_stream)
    torch.cuda.synchronize()
    launches_before = F.launch_count()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        gemvs(torch.cuda.current_stream().cuda_stream)
    launches_per_step = F.launch_count() - launches_before

    def step(timing=None):
        if timing is not None:
            timing[0].record()
        graph.replay()
        if timing is not None:
            timing[1].record()
        if g > 1:
            dist.all_gather_into_tensor(y_all, y_local)
        if timing is not None:
            timing[2].record()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    if g > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for i in range(args.steps):
            step(evs[i])
        end.record()
        torch.cuda.synchronize()
    total_ms = start.elapsed_time(end)
    gemv_ms = sum(e[0].elapsed_time(e[1]) for e in evs)
    gather_ms = sum(e[1].elapsed_time(e[2]) for e in evs)
    t = torch.tensor([total_ms, gemv_ms, gather_ms], device=dev, dtype=torch.float64)
    if g > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, gemv_ms, gather_ms = t.tolist()
    ms_per_step = total_ms / args.steps
    total_bytes = mats * GEMV_BYTES  # all ranks together, per step
    value = total_bytes / (ms_per_step * 1e-3) / 1e9

    # ---- end to end through the public API, host buffers, no graph ------------
    xh = torch.empty(1, COLS, dtype=torch.bfloat16, pin_memory=True)
    xh.copy_(x.cpu())
    yh = torch.empty(g, mats, rows_per_rank, dtype=torch.bfloat16, pin_memory=True)
    sink = F.Async()
    xd = torch.empty_like(x)

    def e2e_step():
        xd.copy_(xh, non_blocking=True)
        for c in range(mats):
            F.gemv(slices[c], xd, y_local[c:c + 1], F.DEFAULT_GEMV_TILE).submit(sink)
        if g > 1:
            dist.all_gather_into_tensor(y_all, y_local)
        else:
            y_all[0].copy_(y_local)
        yh.copy_(y_all, non_blocking=True)

    e2e_steps = max(1, min(args.steps, 50))
    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    if g > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if g > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = total_bytes / (te.item() / e2e_steps * 1e-3) / 1e9

    per_launch_ms = gemv_ms / (args.steps * mats)
    launch_bytes = rows_per_rank * COLS // 2 + rows_per_rank * COLS // 16 + 4 + COLS * 2 + rows_per_rank * 2
    peak, peak_kind = measured_peak()
    achieved = launch_bytes / (per_launch_ms * 1e-3) / 1e9
    traffic = load_traffic() if g == 1 else None
    if rank == 0:
        out = {
            "metric": "NVFP4 GEMV HBM GB/s", "value": value, "unit": "GB/s", "n_gpus": g, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "e2m1xe4m3 weights, bf16 x/y, f32 accumulate",
            "data": "synthetic (seeded Philox: W N(0,0.02), x N(0,1) seed 0)",
            "config": {"workload": "config0 NVFP4 GEMV 4096x4096 (x bf16 [1,4096], y bf16)",
                       "matrices_per_step": mats, "rows_per_rank": rows_per_rank,
                       "parallelism": f"N-split x{g} + NCCL all-gather" if g > 1 else "single GPU",
                       "l2": "inputs larger than L2: 605 MB of distinct weights per rank per step",
                       "timing": "CUDA graph replay per step, CUDA events, max over ranks"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "peak_kind": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured"
                         else "fallback 6650 GB/s",
                         "per_launch_us": per_launch_ms * 1e3,
                         "note": "per-launch time = GEMV region / launches (inter-kernel gaps included)"},
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": COLS * 2,
                    "d2h_bytes_per_step": g * mats * rows_per_rank * 2},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
            "breakdown_ms": {"gemv": gemv_ms / args.steps, "all_gather": gather_ms / args.steps},
        }
        if g == 1:
            out["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
        emit(out)
    del graph
    if g > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse_args()
    if args.impl == "reference":
        reference_arm(args)
    else:
        ours_arm(args)


if __name__ == "__main__":
    main()
