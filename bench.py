"""Benchmark of the firepit_b200 hot path (one JSON line on rank 0).

Default workload ("gemv"): NVFP4 decode GEMV, W [4096 x
4096] from N(0, 0.02) quantized to NVFP4 (one global per matrix), x bf16
rows from N(0, 1) seed 0, y bf16.  One step is one decode-style sweep over
64*g distinct weight matrices (g = number of GPUs), each with its own x row:
every matrix is split along N (rows) over the g ranks; each rank computes its
row slices of all 64*g GEMVs as one prepared tensor-core batch
(fpb_nvfp4_gemv_batch_run: each x row as 8 NVFP4 digit planes, the weights
through tcgen05 mxf4nvf4, up to 512 matrices' slices per batch).  At g > 1
the batch's epilogue also stores each slice into every rank's gathered
output (NVLink peer stores into buffers mapped with CUDA IPC) and a
peer-memory barrier (fpb_peer_barrier) ends the step, which is one CUDA
graph; `--all-gather nccl` uses fpb_comm_all_gather instead.  Each rank
streams 64 * 9.45 MB = 605 MB of weights per step at every g (inputs larger
than L2); per-GPU work is fixed as g grows ("weak").

  value  device-resident GB/s (algorithmic bytes of all ranks / max step time),
         the launches replayed as CUDA graphs;
  e2e    the same metric through the public Python API
         (firepit_b200.gemv_batch_planes(...).submit(Graph sink)) with x copied from
         pinned host memory each step and y copied back.

The default line also carries "sub_records" for the other BASELINE configs
(config 1 FP8 GEMM; config 2 NVFP4 GEMM at M = 1, 16, 128, 2048; config 3 MoE
layer at T = 64 and 4096 on one GPU, expert-parallel over the ranks when g >
1; config 4 decode tokens/s of the hybrid MoE decoder, replicas over the
ranks), each with its own roofline, cpu_baseline (rank 0, one GPU), e2e and clocks;
--no-sub leaves them out, --config runs one of them as the main line.

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
    p.add_argument("--config", choices=["gemv", "nvfp4_gemm_m1", "nvfp4_gemm_m16", "nvfp4_gemm_m128",
                                        "nvfp4_gemm_m2048", "fp8_gemm", "moe_t4096", "moe_t64", "moe_ep",
                                        "decode"],
                   default="gemv",
                   help="gemv: config 0 (default); nvfp4_gemm_m*: config 2 at M=1 / 16 (decode GEMV entry) and "
                        "M=128 / 2048 (tcgen05 GEMM); fp8_gemm: config 1; moe_t*: config 3 MoE layer at T=4096 / "
                        "T=64; moe_ep: config 3 expert-parallel over the ranks (NCCL all-to-all), T=4096 per rank; "
                        "decode: config 4, the hybrid MoE decoder's decode tokens/s")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="budget of the cpu_baseline sample")
    p.add_argument("--no-sub", action="store_true", help="default line without the other configs' sub-records")
    p.add_argument("--all-gather", choices=["peer", "nccl"], default="peer",
                   help="config 0 at N > 1: the GEMV epilogue's NVLink peer stores + peer barrier (peer), or "
                        "NCCL all-gathers overlapping the next batch (nccl)")
    p.add_argument("--sub-steps", type=int, default=20, help="timed steps of each sub-record")
    p.add_argument("--sub-cpu-seconds", type=float, default=3.0, help="cpu_baseline budget of each sub-record")
    p.add_argument("--dec-prompt", type=int, default=2048, help="config 4 prompt tokens per session (2048)")
    p.add_argument("--dec-steps", type=int, default=256, help="config 4 greedy tokens per session (256)")
    return p.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def emit(obj):
    print(json.dumps(obj), flush=True)


_DIST = {}


def dist_init():
    """(rank, world, local_rank, device) with the NCCL process group set up
    once per process (short timeout, so ranks that wait on each other end
    with an error instead of hanging)."""
    import torch
    import torch.distributed as dist
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1 and not _DIST:
        from datetime import timedelta
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        _DIST["up"] = True
    return rank, world, local, dev


def comm():
    """The library's NCCL communicator (fpb_comm_*) for this process, made
    once after the torch.distributed group (which only hands out rank 0's
    unique id); None on one GPU."""
    if not _DIST:
        return None
    if "comm" not in _DIST:
        from firepit_b200.comm import Comm
        _DIST["comm"] = Comm.from_torch()
    return _DIST["comm"]


def dist_sync():
    import torch.distributed as dist
    if _DIST:
        dist.barrier()


def dist_finish():
    import torch.distributed as dist
    if _DIST:
        dist.barrier()
        if "comm" in _DIST:
            _DIST["comm"].destroy()
        dist.destroy_process_group()
        _DIST.clear()


def use_all_cores():
    """The CPU legs use every host core: under torch.distributed.run the
    launcher sets OMP_NUM_THREADS=1 for each rank."""
    n = os.cpu_count() or 1
    from oracle import oracle as O
    O.set_num_threads(n)
    return n


def peaks_json():
    f = ROOT / "MEASURED_PEAKS.json"
    return json.loads(f.read_text()) if f.exists() else {}


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


# ---- config 0 -----------------------------------------------------------------------------
MAX_SEGS = 128  # fpb_nvfp4_gemv_batched's segments per launch
MAX_PLANES_SEGS = 512  # members of one tensor-core batch here (the library takes up to 1024)


def gemv_config(g: int) -> dict:
    return {"workload": "config0 NVFP4 GEMV 4096x4096 (x bf16 [1,4096] N(0,1), y bf16)",
            "matrices_per_step": MATS_PER_GPU * g, "rows_per_rank": ROWS // g,
            "launch": f"each rank's slices of the {MATS_PER_GPU * g} matrices in one prepared batch per "
                      f"{MAX_PLANES_SEGS} (fpb_nvfp4_gemv_batch_run: x as NVFP4 digit planes, tcgen05), every matrix "
                      "with its own x row",
            "parallelism": f"N-split x{g}; the GEMV launch stores each rank's slices into every rank's gathered "
                           "output (NVLink peer stores), one peer-memory barrier per step" if g > 1 else "single GPU",
            "l2": "inputs larger than L2: 605 MB of distinct weights per rank per step",
            "timing": "CUDA graph replay per launch, CUDA events, max over ranks"}


def reference_arm(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    cores = use_all_cores()
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
    sample = (f"{rows} of {ROWS} rows of one {ROWS}x{COLS} NVFP4 GEMV per step (oracle f32 kernel order, OpenMP "
              f"on {cores} threads)")
    emit({"impl": "reference", "metric": "NVFP4 GEMV HBM GB/s", "value": gbs, "unit": "GB/s", "n_gpus": args.gpus,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
          "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Philox N(0,1)/N(0,0.02))",
          "config": gemv_config(args.gpus),
          "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
          "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})


def cpu_baseline(seconds: float):
    """The reference's host path (oracle port) on this box's cores: full
    config-0 GEMVs repeated for about `seconds`."""
    cores = use_all_cores()
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
    return {"value": GEMV_BYTES / dt / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{n} full 4096x4096 NVFP4 GEMVs (oracle f32 kernel order, OpenMP), {dt * 1e3:.2f} ms each"}


def load_traffic(name: str):
    """DRAM bytes per launch from a committed ncu summary (first line:
    `dram_bytes_per_launch <bytes>`), or None."""
    f = ROOT / "profiles" / name
    if f.exists():
        try:
            key, val = f.read_text().split("\n", 1)[0].split()
            return int(val) if key == "dram_bytes_per_launch" else None
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


def graph_of(torch, fn, stream):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn(torch.cuda.current_stream().cuda_stream)
    return g


def ours_arm(args):
    import torch
    import torch.distributed as dist

    import firepit_b200 as F
    N_ = F._native
    BF = N_.FPB_BF16

    rank, world, local, dev = dist_init()
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
    # x row c (of one seed-0 N(0,1) stream) is matrix c's input; row 0 is config 0's x.
    x = F.synth_normal((mats, COLS), seed=0, stream_id=0, dtype=torch.bfloat16, device=dev)
    y_local = torch.empty(mats, rows_per_rank, dtype=torch.bfloat16, device=dev)
    # the tensor-core batch (cols % 256 == 0, <= 4096: config 0) takes every
    # rank's slices at N <= 8 in one launch, so the tiles of all matrices share
    # one tail; the streaming kernel takes at most MAX_SEGS per launch
    gsize = MAX_PLANES_SEGS if COLS % 256 == 0 and COLS <= 4096 else MAX_SEGS
    groups = [range(i, min(i + gsize, mats)) for i in range(0, mats, gsize)]
    # On more than one GPU the gathered outputs are buffers every rank maps
    # (CUDA IPC): the GEMV's epilogue stores this rank's slices into all of
    # them over NVLink, so the all-gather is part of the GEMV launch.
    peer_bufs, barrier = [], None
    if g > 1:
        from firepit_b200.comm import PeerBarrier, PeerBuffer
        peer_bufs = [PeerBuffer(g * len(gr) * rows_per_rank * 2) for gr in groups]
        barrier = PeerBarrier()
        y_all = [pb.local.view(torch.bfloat16).view(g, len(gr), rows_per_rank) for pb, gr in zip(peer_bufs, groups)]
    else:
        y_all = [torch.empty(g, len(gr), rows_per_rank, dtype=torch.bfloat16, device=dev) for gr in groups]

    def peers_of(i):
        gr = groups[i]
        return [[peer_bufs[i].ptrs[p] + (rank * len(gr) + j) * rows_per_rank * 2 for p in range(g)]
                for j in range(len(gr))]

    def batched(xsrc, tensor_cores=True, peers=False):
        """The step's GEMVs, one batch per group of matrices: on the tensor
        cores (x as NVFP4 digit planes, tcgen05) where the shapes allow, else
        the streaming kernel; with `peers` the batch also does the all-gather."""
        if tensor_cores:
            return [F.gemv_batch_planes([(slices[c], xsrc[c:c + 1], y_local[c:c + 1]) for c in gr],
                                        y_peers=peers_of(i) if peers else None) for i, gr in enumerate(groups)]
        # streaming: each group in launches of at most MAX_SEGS matrices
        return [[F.gemv_batched([(slices[c], xsrc[c:c + 1], y_local[c:c + 1]) for c in gr[j:j + MAX_SEGS]])
                 for j in range(0, len(gr), MAX_SEGS)] for gr in groups]

    use_peers = g > 1 and getattr(args, "all_gather", "peer") == "peer"
    try:
        launches_b = batched(x, peers=use_peers)
        tensor_cores = True
    except F.ShapeError:
        launches_b = batched(x, tensor_cores=False)
        tensor_cores = False
    fused = use_peers and tensor_cores

    def launch(i, sh):
        if tensor_cores:
            N_.call("fpb_nvfp4_gemv_batch_run", launches_b[i]._batch, sh)
        else:
            for sub in launches_b[i]:
                N_.call("fpb_nvfp4_gemv_batched", sub._segs, len(sub.gemvs), BF, BF, 1, sh)

    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):  # every code path initialised outside capture
        for i in range(len(groups)):
            launch(i, s.cuda_stream)
    torch.cuda.synchronize()
    before = F.launch_count()
    graphs = [graph_of(torch, lambda sh, i=i: launch(i, sh), s) for i in range(len(groups))]
    launches_per_step = F.launch_count() - before
    ng = len(groups)
    overlap = g > 1
    if overlap:
        # One graph per step: the groups' GEMVs, which store every rank's
        # gathered output themselves (peer stores), then a one-word all-reduce
        # as the barrier; on the streaming fallback each group's NCCL
        # all-gather runs on a second stream, overlapping the next group's GEMV.
        cs = torch.cuda.Stream(device=dev)

        def whole(sh):
            cur = torch.cuda.current_stream()
            for i in range(ng):
                launch(i, sh)
                if not fused:
                    cs.wait_stream(cur)
                    with torch.cuda.stream(cs):
                        comm().all_gather_into(y_all[i], y_local[groups[i].start:groups[i].stop])
            if fused:
                barrier()  # every rank's peer stores have landed (fpb_peer_barrier)
            else:
                cur.wait_stream(cs)

        with torch.cuda.stream(s):  # eager once: the collectives set up outside capture
            whole(s.cuda_stream)
        torch.cuda.synchronize()
        step_graph = graph_of(torch, whole, s)

    def step(ev=None):
        if overlap:
            step_graph.replay()
            return
        for i, gr in enumerate(graphs):
            if ev is not None:
                ev[2 * i].record()
            gr.replay()
            if ev is not None:
                ev[2 * i + 1].record()
            if g > 1:
                comm().all_gather_into(y_all[i], y_local[groups[i].start:groups[i].stop])

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2 * ng)] for _ in range(args.steps)]
    dist_sync()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for i in range(args.steps):
            step(evs[i])
        end.record()
        torch.cuda.synchronize()
    total_ms = start.elapsed_time(end)
    if overlap:
        # the GEMVs alone (the same graphs without the collectives), scaled to
        # the timed steps: per-launch time for the roofline, and the exposed
        # all-gather time as the rest of the step
        gsteps = max(1, min(args.steps, 200))
        for i in range(gsteps):
            for j, gr in enumerate(graphs):
                evs[i][2 * j].record()
                gr.replay()
                evs[i][2 * j + 1].record()
        torch.cuda.synchronize()
        gemv_ms = sum(e[2 * i].elapsed_time(e[2 * i + 1]) for e in evs[:gsteps] for i in range(ng))
        gemv_ms *= args.steps / gsteps
    else:
        gemv_ms = sum(e[2 * i].elapsed_time(e[2 * i + 1]) for e in evs for i in range(ng))
    t = torch.tensor([total_ms, gemv_ms], device=dev, dtype=torch.float64)
    if g > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, gemv_ms = t.tolist()
    ms_per_step = total_ms / args.steps
    total_bytes = mats * GEMV_BYTES  # all ranks together, per step
    value = total_bytes / (ms_per_step * 1e-3) / 1e9

    # ---- one launch per GEMV (the single-matrix entry fpb_nvfp4_gemv) --------
    single_n = min(mats, MATS_PER_GPU)

    def singles(sh):
        for c in range(single_n):
            N_.call("fpb_nvfp4_gemv", slices[c].handle, 0, 0, x[c].data_ptr(), BF, y_local[c].data_ptr(), BF, 1, sh)

    with torch.cuda.stream(s):
        singles(s.cuda_stream)
    torch.cuda.synchronize()
    gs = graph_of(torch, singles, s)
    for _ in range(3):
        gs.replay()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    single_steps = max(1, min(args.steps, 200))
    s0.record()
    for _ in range(single_steps):
        gs.replay()
    s1.record()
    torch.cuda.synchronize()
    ts = torch.tensor([s0.elapsed_time(s1)], device=dev, dtype=torch.float64)
    if g > 1:
        dist.all_reduce(ts, op=dist.ReduceOp.MAX)
    single_launch_ms = ts.item() / (single_steps * single_n)
    del gs

    # ---- the same batch on the streaming CUDA-core kernel (fpb_nvfp4_gemv_batched) --
    stream_b = batched(x, tensor_cores=False)

    def streaming(sh):
        for subs in stream_b:
            for sub in subs:
                N_.call("fpb_nvfp4_gemv_batched", sub._segs, len(sub.gemvs), BF, BF, 1, sh)

    with torch.cuda.stream(s):
        streaming(s.cuda_stream)
    torch.cuda.synchronize()
    gsb = graph_of(torch, streaming, s)
    for _ in range(3):
        gsb.replay()
    torch.cuda.synchronize()
    s0.record()
    for _ in range(single_steps):
        gsb.replay()
    s1.record()
    torch.cuda.synchronize()
    tsb = torch.tensor([s0.elapsed_time(s1)], device=dev, dtype=torch.float64)
    if g > 1:
        dist.all_reduce(tsb, op=dist.ReduceOp.MAX)
    streaming_step_ms = tsb.item() / single_steps
    del gsb

    # ---- end to end through the public API, host buffers ----------------------
    # The reference's Graph sink (sink.rs:94-105): one CUDA graph holds the
    # copy of x from pinned host memory, the batched GEMV submits and (one
    # GPU) the copy of y back to pinned host memory.
    xh = torch.empty(mats, COLS, dtype=torch.bfloat16, pin_memory=True)
    xh.copy_(x.cpu())
    yh = torch.empty(g, mats, rows_per_rank, dtype=torch.bfloat16, pin_memory=True)
    # per group, the gathered [g, group, rows] block in one contiguous pinned buffer
    # (a strided slice of yh is no pinned copy target inside a graph)
    yh_g = [torch.empty(g, len(gr), rows_per_rank, dtype=torch.bfloat16, pin_memory=True) for gr in groups]
    xd = torch.empty_like(x)
    e2e_b = batched(xd, tensor_cores, peers=fused)
    if not tensor_cores:
        e2e_b = [sub for subs in e2e_b for sub in subs]
    for b in e2e_b:  # eager once: every code path initialised outside capture
        b.submit(F.Async())
    torch.cuda.synchronize()
    gsink = F.Graph()
    with gsink:
        xd.copy_(xh, non_blocking=True)
        for b in e2e_b:
            b.submit(gsink)
        if g == 1:
            yh[0].copy_(y_local, non_blocking=True)
        elif fused:
            barrier()
            for i in range(len(groups)):
                yh_g[i].copy_(y_all[i], non_blocking=True)

    def e2e_step():
        gsink.replay()
        if g > 1 and not fused:
            for i, gr in enumerate(groups):
                comm().all_gather_into(y_all[i], y_local[gr.start:gr.stop])
                yh_g[i].copy_(y_all[i], non_blocking=True)

    e2e_steps = max(1, min(args.steps, 50))
    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    dist_sync()
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

    slice_bytes = rows_per_rank * COLS // 2 + rows_per_rank * COLS // 16 + 4 + COLS * 2 + rows_per_rank * 2
    launch_bytes = len(groups[0]) * slice_bytes
    per_launch_ms = gemv_ms / (args.steps * ng)
    peak, peak_kind = measured_peak()
    achieved = launch_bytes / (per_launch_ms * 1e-3) / 1e9
    single_achieved = slice_bytes / (single_launch_ms * 1e-3) / 1e9
    traffic = None
    if g == 1:
        per_matrix = load_traffic("gemv_nvfp4_planes_config0_traffic.txt" if tensor_cores
                                  else "gemv_nvfp4_batched_config0_traffic.txt")
        traffic = per_matrix * len(groups[0]) if per_matrix else None
    out = None
    if rank == 0:
        out = {
            "metric": "NVFP4 GEMV HBM GB/s", "value": value, "unit": "GB/s", "n_gpus": g, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "e2m1xe4m3 weights, bf16 x/y, f32 accumulate",
            "data": "synthetic (seeded Philox: W N(0,0.02), x N(0,1) seed 0)",
            "config": gemv_config(g),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "peak_kind": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured"
                         else "fallback 6650 GB/s",
                         "per_launch_us": per_launch_ms * 1e3, "algorithmic_bytes_per_launch": launch_bytes,
                         "note": ("dominant kernel nvfp4_gemm_kernel in planes mode (x as 8 NVFP4 digit planes, "
                                  "tcgen05 mxf4nvf4), after planes_encode_kernel" if tensor_cores else
                                  "dominant kernel gemv_nvfp4_stream_kernel") +
                                 f"; one launch = the rank's slices of {len(groups[0])} matrices; the time per "
                                 "launch includes the plane encode; traffic = ncu DRAM bytes per matrix x matrices"},
            "single_gemv": {"per_launch_us": single_launch_ms * 1e3, "achieved_gbs": single_achieved,
                            "frac": single_achieved / peak,
                            "note": f"{single_n} fpb_nvfp4_gemv launches (one matrix slice each) in one CUDA graph"},
            "streaming_batched": {"ms_per_step": streaming_step_ms,
                                  "achieved_gbs": launch_bytes * len(groups) / (streaming_step_ms * 1e-3) / 1e9,
                                  "frac": launch_bytes * len(groups) / (streaming_step_ms * 1e-3) / 1e9 / peak,
                                  "note": "the same step on the CUDA-core streaming kernel (fpb_nvfp4_gemv_batched)"},
            "gemv_path": "tensor cores (fpb_nvfp4_gemv_batch_run)" if tensor_cores else "streaming",
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": mats * COLS * 2,
                    "d2h_bytes_per_step": g * mats * rows_per_rank * 2,
                    "path": ("firepit_b200.gemv_batch_planes" if tensor_cores else "firepit_b200.gemv_batched") +
                            "(...).submit(Graph sink): H2D x, the batched GEMVs and D2H y "
                            "in one CUDA graph" + (" + NCCL all-gathers" if g > 1 else "")},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
            "breakdown_ms": {"gemv": gemv_ms / args.steps,
                             "all_gather": (total_ms - gemv_ms) / args.steps if g > 1 else 0.0,
                             "note": ("all_gather = the step's time beyond the GEMV launches, which store the "
                                      "gathered output on every rank themselves (NVLink peer stores): the barrier"
                                      if fused else "all_gather = the step's time beyond its GEMVs (each group's "
                                      "NCCL all-gather overlaps the next group's GEMV)") if g > 1
                                     else "one GPU: no exchange"},
        }
        if g == 1 and args.cpu_seconds > 0:
            out["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    del graphs, gsink
    if overlap:
        del step_graph
    del launches_b, e2e_b
    if barrier is not None:
        barrier.close()
    for pb in peer_bufs:
        pb.close()
    dist_sync()
    return out


# ---- config 2: NVFP4 GEMM (tcgen05) ------------------------------------------------------
GEMM_N, GEMM_K, GEMM_MATS = 8192, 2048, 16


def gemm_shape(args):
    return int(args.config.rsplit("_m", 1)[1])


def gemm_bytes(m, n, k):
    """Algorithmic bytes of one GEMM launch on quantized activations: weight codes,
    factors and row globals, activation codes and factors, bf16 output."""
    return n * k // 2 + n * k // 16 + 4 * n + m * k // 2 + m * k // 16 + 2 * m * n


def gemv_batch_bytes(m, n, k):
    """Algorithmic bytes of one decode-GEMV launch of m input rows (the M <= 16
    cases of config 2): weight codes, factors and row globals, x and y bf16."""
    return n * k // 2 + n * k // 16 + 4 * n + 2 * m * k + 2 * m * n


def gemm_config(m: int, g: int) -> dict:
    if m <= 16:
        how = (f"x bf16 [{m},2048] on the tensor-core GEMV (the decode-size path of nvfp4_gemm: x as NVFP4 digit "
               f"planes, fpb_nvfp4_gemv_batch_run over the 16 matrices, {m} rows); weights NVFP4, x kept in bf16")
    else:
        how = "x bf16 quantized on the device to NVFP4 (W4A4), tcgen05 block-scaled GEMM"
    return {"workload": f"config2 NVFP4 GEMM M={m} K=2048 N=8192, {how}",
            "matrices_per_step": GEMM_MATS, "n_per_rank": GEMM_N // g,
            "l2": "inputs larger than L2 (16 distinct weights, 151 MB per step at one GPU)",
            "parallelism": f"N-split x{g} + NCCL all-gather" if g > 1 else "single GPU"}


def gemm_cpu_sample(m: int, seconds: float):
    """The host path restated on a bounded sample: the oracle's f32 kernel-order
    GEMV (M <= 16, gemv/nvfp4.rs:34-59) or dequantized NVFP4 operands times
    each other in f32 BLAS (M >= 128).  Returns (value, sample, cores); value in
    GB/s for M <= 16, TFLOP/s otherwise."""
    cores = use_all_cores()
    import numpy as np

    from oracle import oracle as O
    w = O.synth_normal(GEMM_N * GEMM_K, seed=0, stream=1, std=0.02).reshape(GEMM_N, GEMM_K)
    pw, sw, gw = O.nvfp4_quantize(w)
    x = O.bf16_to_f32(O.bf16_bits(O.synth_normal(m * GEMM_K, seed=0, stream=0))).reshape(m, GEMM_K)
    if m <= 16:
        fn = lambda: O.nvfp4_gemv_f32(pw, sw, gw, GEMM_N, GEMM_K, x)
    else:
        wd = O.nvfp4_dequantize(pw, sw, gw, GEMM_N, GEMM_K)
        pa, sa, ga = O.nvfp4_quantize(x)
        xd = O.nvfp4_dequantize(pa, sa, ga, m, GEMM_K)
        rows = min(m, 128)
        fn = lambda: xd[:rows] @ wd.T
    fn()
    n, t0 = 0, time.perf_counter()
    while n < 2 or time.perf_counter() - t0 < seconds:
        fn()
        n += 1
    dt = (time.perf_counter() - t0) / n
    if m <= 16:
        return (gemv_batch_bytes(m, GEMM_N, GEMM_K) / dt / 1e9,
                f"{n} x one W[8192,2048] NVFP4 GEMV of {m} rows (oracle f32 kernel order, OpenMP)", cores)
    rows = min(m, 128)
    return (2.0 * rows * GEMM_N * GEMM_K / dt / 1e12,
            f"{n} x ({rows} of {m} activation rows x W[8192,2048]^T), dequantized NVFP4, f32 BLAS", cores)


def gemm_reference_arm(args):
    """The host path restated (gemm_cpu_sample) on the box's cores, rank 0 only."""
    rank, _, _ = dist_env()
    if rank != 0:
        return
    m = gemm_shape(args)
    budget = min(60.0, max(5.0, 0.5 * (args.steps + args.warmup)))
    v, sample, cores = gemm_cpu_sample(m, budget)
    gbs = m <= 16
    ms = (gemv_batch_bytes(m, GEMM_N, GEMM_K) / (v * 1e9) if gbs else 2.0 * m * GEMM_N * GEMM_K / (v * 1e12)) * 1e3
    emit({"impl": "reference", "metric": "NVFP4 GEMM HBM GB/s" if gbs else "NVFP4 GEMM TFLOPS", "value": v,
          "unit": "GB/s" if gbs else "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
          "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
          "data": "synthetic (seeded Philox)", "config": gemm_config(m, args.gpus),
          "cpu_baseline": {"value": v, "unit": "GB/s" if gbs else "TFLOP/s", "cores": cores, "kind": "port",
                           "sample": sample},
          "e2e": {"value": v, "unit": "GB/s" if gbs else "TFLOP/s", "h2d_bytes_per_step": 0,
                  "d2h_bytes_per_step": 0}})


def gemm_small_arm(args):
    """Config 2 at M = 1 and 16: x bf16 [M, 2048] N(0,1) times 16 distinct NVFP4
    weights [8192, 2048] (N-split over the ranks) on the tensor-core GEMV (x
    as NVFP4 digit planes, the decode-size path of nvfp4_gemm), one prepared
    batch launch per step; HBM-bound."""
    import torch
    import torch.distributed as dist

    import firepit_b200 as F
    N_ = F._native
    BF = N_.FPB_BF16
    rank, world, local, dev = dist_init()
    g = world
    m = gemm_shape(args)
    n_rank = GEMM_N // g
    r0 = rank * n_rank
    mats = []
    for c in range(GEMM_MATS):
        w = F.synth_normal((GEMM_N, GEMM_K), seed=0, stream_id=1 + c, std=0.02, device=dev)
        packed, scales, globals_ = F.quantize_nvfp4(w)
        del w
        mats.append(F.Nvfp4Matrix.from_device(packed[r0:r0 + n_rank].contiguous(),
                                              scales[r0:r0 + n_rank].contiguous(),
                                              globals_[r0:r0 + n_rank].contiguous(), n_rank, GEMM_K))
    x = F.synth_normal((m, GEMM_K), seed=0, stream_id=0, dtype=torch.bfloat16, device=dev)
    ys = torch.empty(GEMM_MATS, m, n_rank, dtype=torch.bfloat16, device=dev)
    y_all = torch.empty(g, GEMM_MATS, m, n_rank, dtype=torch.bfloat16, device=dev)
    # the 16 matrices as one prepared tensor-core batch (x as NVFP4 digit
    # planes, tcgen05): the decode-size path of nvfp4_gemm
    bat = F.gemv_batch_planes([(mats[c], x, ys[c]) for c in range(GEMM_MATS)])

    def launch(sh):
        N_.call("fpb_nvfp4_gemv_batch_run", bat._batch, sh)

    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        launch(s.cuda_stream)
    torch.cuda.synchronize()
    before = F.launch_count()
    gr = graph_of(torch, launch, s)
    launches_per_step = F.launch_count() - before

    def step(ev=None):
        if ev:
            ev[0].record()
        gr.replay()
        if ev:
            ev[1].record()
        if g > 1:
            comm().all_gather_into(y_all, ys)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    dist_sync()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for i in range(args.steps):
            step(evs[i])
        end.record()
        torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(end), sum(e[0].elapsed_time(e[1]) for e in evs)], device=dev,
                     dtype=torch.float64)
    if g > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, gemv_ms = t.tolist()
    ms_per_step = total_ms / args.steps
    bytes_step = GEMM_MATS * gemv_batch_bytes(m, GEMM_N, GEMM_K)  # all ranks
    value = bytes_step / (ms_per_step * 1e-3) / 1e9

    xh = x.cpu().pin_memory()
    yh = torch.empty(GEMM_MATS, m, n_rank, dtype=torch.bfloat16, pin_memory=True)
    xd = torch.empty_like(x)
    e2e_b = F.gemv_batch_planes([(mats[c], xd, ys[c]) for c in range(GEMM_MATS)])
    e2e_b.submit(F.Async())
    torch.cuda.synchronize()
    gsink = F.Graph()
    with gsink:
        xd.copy_(xh, non_blocking=True)
        e2e_b.submit(gsink)
        yh.copy_(ys, non_blocking=True)
    e2e_steps = max(1, min(args.steps, 20))
    for _ in range(2):
        gsink.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        gsink.replay()
    e1.record()
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if g > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = bytes_step / (te.item() / e2e_steps * 1e-3) / 1e9

    per_launch_ms = gemv_ms / args.steps
    hbm, kind = measured_peak()
    achieved = GEMM_MATS * gemv_batch_bytes(m, n_rank, GEMM_K) / (per_launch_ms * 1e-3) / 1e9
    out = None
    if rank == 0:
        out = {"metric": "NVFP4 GEMM HBM GB/s", "value": value, "unit": "GB/s", "n_gpus": g, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
               "vs_baseline": None, "dtype": "e2m1xe4m3 weights, bf16 x/y, f32 accumulate",
               "data": "synthetic (seeded Philox: W N(0,0.02), x N(0,1) seed 0)", "config": gemm_config(m, g),
               "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                            "frac": achieved / hbm, "traffic": None, "per_launch_us": per_launch_ms * 1e3,
                            "peak_kind": f"{kind} hbm_gbs"},
               "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": m * GEMM_K * 2,
                       "d2h_bytes_per_step": GEMM_MATS * m * n_rank * 2,
                       "path": "firepit_b200.gemv_batch_planes(...).submit(Graph sink): H2D x, GEMVs, D2H y in one "
                               "CUDA graph"},
               "gpu_launches": launches_per_step * args.steps, "clocks": clocks.summary()}
        if g == 1 and args.cpu_seconds > 0:
            v, sample, cores = gemm_cpu_sample(m, args.cpu_seconds)
            out["cpu_baseline"] = {"value": v, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample}
    del gr, gsink
    dist_sync()
    return out


def gemm_arm(args):
    """Config 2 GEMM: x bf16 [M, 2048] quantized on the device to NVFP4, times
    16 distinct NVFP4 weights [8192, 2048] (N-split over the ranks) per step;
    inputs of a step (151 MB of weights per GPU at g = 1) exceed L2.  M <= 128
    (64 weight tiles per matrix, fewer than the SMs): the 16 GEMMs as one W4A4
    batch launch (firepit_b200.nvfp4_gemm_batch: x quantized once, every
    matrix's tiles in one tcgen05 launch); M = 2048: one launch per GEMM."""
    import torch
    import torch.distributed as dist

    import firepit_b200 as F
    N_ = F._native

    rank, world, local, dev = dist_init()
    g = world
    m = gemm_shape(args)
    n_rank = GEMM_N // g
    r0 = rank * n_rank
    mats = []
    for c in range(GEMM_MATS):
        w = F.synth_normal((GEMM_N, GEMM_K), seed=0, stream_id=1 + c, std=0.02, device=dev)
        packed, scales, globals_ = F.quantize_nvfp4(w)
        del w
        mat = F.Nvfp4Matrix.from_device(packed[r0:r0 + n_rank].contiguous(), scales[r0:r0 + n_rank].contiguous(),
                                        globals_[r0:r0 + n_rank].contiguous(), n_rank, GEMM_K)
        mats.append(mat)
    x = F.synth_normal((m, GEMM_K), seed=0, stream_id=0, dtype=torch.bfloat16, device=dev)
    ws_bytes = int(N_.lib.fpb_nvfp4_gemm_workspace_bytes(m, GEMM_K))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    sf_bytes = int(N_.lib.fpb_nvfp4_act_sf_bytes(m, GEMM_K))
    qa = torch.empty(m * GEMM_K // 2, dtype=torch.uint8, device=dev)
    qsf = torch.empty(sf_bytes, dtype=torch.uint8, device=dev)
    scal = torch.zeros(2, dtype=torch.float32, device=dev)
    ys = torch.empty(GEMM_MATS, m, n_rank, dtype=torch.bfloat16, device=dev)
    y_all = torch.empty(g, GEMM_MATS, m, n_rank, dtype=torch.bfloat16, device=dev)

    def quant(sh):
        N_.call("fpb_nvfp4_quantize_act", x.data_ptr(), N_.FPB_BF16, m, GEMM_K, qa.data_ptr(), qsf.data_ptr(),
                scal.data_ptr(), scal[1:].data_ptr(), sh)

    batched = m <= 128
    bat = F.nvfp4_gemm_batch([(mats[c], x, ys[c]) for c in range(GEMM_MATS)]) if batched else None

    def gemms(sh):
        if batched:  # quantize (inside the batch run) + all 16 GEMMs
            N_.call("fpb_nvfp4_gemv_batch_run", bat._batch, sh)
            return
        for c in range(GEMM_MATS):
            N_.call("fpb_nvfp4_gemm_q", mats[c].handle, 0, 0, qa.data_ptr(), qsf.data_ptr(), scal.data_ptr(), m,
                    ys[c].data_ptr(), N_.FPB_BF16, sh)

    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        quant(s.cuda_stream)
        gemms(s.cuda_stream)
    torch.cuda.synchronize()
    before = F.launch_count()
    gq, gg = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    if not batched:
        with torch.cuda.graph(gq, stream=s):
            quant(torch.cuda.current_stream().cuda_stream)
    with torch.cuda.graph(gg, stream=s):
        gemms(torch.cuda.current_stream().cuda_stream)
    launches_per_step = F.launch_count() - before

    def step(ev=None):
        if ev:
            ev[0].record()
        if not batched:
            gq.replay()
        if ev:
            ev[1].record()
        gg.replay()
        if ev:
            ev[2].record()
        if g > 1:
            comm().all_gather_into(y_all, ys)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    if g > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for i in range(args.steps):
            step(evs[i])
        end.record()
        torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(end), sum(e[0].elapsed_time(e[1]) for e in evs),
                      sum(e[1].elapsed_time(e[2]) for e in evs)], device=dev, dtype=torch.float64)
    if g > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, quant_ms, gemm_ms = t.tolist()
    ms_per_step = total_ms / args.steps
    flops_step = 2.0 * m * GEMM_N * GEMM_K * GEMM_MATS
    value = flops_step / (ms_per_step * 1e-3) / 1e12

    # end to end through the public API: x from pinned host memory, y back
    xh = x.cpu().pin_memory()
    yh = torch.empty(GEMM_MATS, m, n_rank, dtype=torch.bfloat16, pin_memory=True)
    xd = torch.empty_like(x)
    # the reference's Graph sink: H2D x, the GEMMs and D2H y in one CUDA graph
    e2e_bat = F.nvfp4_gemm_batch([(mats[c], xd, ys[c]) for c in range(GEMM_MATS)]) if batched else None
    for c in range(GEMM_MATS):
        F.nvfp4_gemm(mats[c], x, ys[c], F.GemmTile(8, 128, 32), workspace=ws).submit(F.Async())
    torch.cuda.synchronize()
    gsink = F.Graph()
    with gsink:
        xd.copy_(xh, non_blocking=True)
        if batched:
            e2e_bat.submit(gsink)
        else:
            for c in range(GEMM_MATS):
                F.nvfp4_gemm(mats[c], xd, ys[c], F.GemmTile(8, 128, 32), workspace=ws).submit(gsink)
        yh.copy_(ys, non_blocking=True)

    def e2e_step():
        gsink.replay()

    e2e_steps = max(1, min(args.steps, 20))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if g > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = flops_step / (te.item() / e2e_steps * 1e-3) / 1e12

    per_launch_ms = gemm_ms / (args.steps * GEMM_MATS)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    if m >= 1024:
        bf16 = float(peaks.get("bf16_tflops", 1590.0))
        achieved = 2.0 * m * n_rank * GEMM_K / (per_launch_ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": 4 * bf16, "unit": "TFLOP/s",
                "frac": achieved / (4 * bf16),
                "traffic": load_traffic("nvfp4_gemm_config2_m2048_traffic.txt") if (m, g) == (2048, 1) else None,
                "peak_kind": "4 x measured bf16 burst (nominal dense FP4:BF16 ratio; no FP4 measurement)"}
    else:
        hbm = float(peaks.get("hbm_gbs", 6650.0))
        achieved = gemm_bytes(m, n_rank, GEMM_K) / (per_launch_ms * 1e-3) / 1e9
        traffic = None
        if batched and (m, g) == (128, 1):  # DRAM bytes of one batch launch, scaled to one GEMM like `achieved`
            t_launch = load_traffic("nvfp4_gemm_batch_config2_m128_traffic.txt")
            traffic = t_launch / GEMM_MATS if t_launch else None
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": traffic, "algorithmic_bytes": gemm_bytes(m, n_rank, GEMM_K), "peak_kind": "measured hbm_gbs"}
    roof["per_launch_us"] = per_launch_ms * 1e3
    if batched:
        roof["per_launch_us"] = gemm_ms / args.steps * 1e3
        roof["note"] = (f"one W4A4 batch launch per step (x quantize + {GEMM_MATS} GEMMs); achieved = the "
                        f"{GEMM_MATS} GEMMs' algorithmic bytes / that launch")
    out = None
    if rank == 0:
        out = ({"metric": "NVFP4 GEMM TFLOPS", "value": value, "unit": "TFLOP/s", "n_gpus": g, "steps": args.steps,
              "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
              "vs_baseline": None, "dtype": "nvfp4 x nvfp4 (e2m1, ue4m3/16), f32 accumulate, bf16 out",
              "data": "synthetic (seeded Philox: W N(0,0.02), x N(0,1) seed 0)",
              "config": gemm_config(m, g),
              "roofline": roof,
              "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": m * GEMM_K * 2,
                      "d2h_bytes_per_step": GEMM_MATS * m * n_rank * 2,
                      "path": ("firepit_b200.nvfp4_gemm_batch" if batched else "firepit_b200.nvfp4_gemm") +
                              "(...).submit(Graph sink): H2D x, quantize + GEMMs, D2H y in one CUDA graph"},
              "gpu_launches": launches_per_step * args.steps, "clocks": clocks.summary(),
              "breakdown_ms": {"quantize_act": quant_ms / args.steps, "gemms": gemm_ms / args.steps}})
        if g == 1 and args.cpu_seconds > 0:
            v, sample, cores = gemm_cpu_sample(m, args.cpu_seconds)
            out["cpu_baseline"] = {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample}
    del gq, gg, bat, e2e_bat
    dist_sync()
    return out


# ---- config 1: FP8 E4M3 GEMM (tcgen05 kind::f8f6f4) -------------------------------------
FP8_M, FP8_K, FP8_N, FP8_MATS = 512, 4096, 14336, 4


def fp8_cpu_sample(seconds: float):
    """The host path restated on a bounded sample: dequantize both FP8 operands
    and multiply in f32 (numpy/BLAS on all host cores).  Returns (TFLOP/s,
    sample description)."""
    import numpy as np

    from oracle import oracle as O
    n = 2048  # weight rows of the sample (of 14336)
    w = O.synth_normal(n * FP8_K, seed=0, stream=1, std=0.02).reshape(n, FP8_K)
    wb, ws = O.fp8_quantize(w, 128, 128)
    wd = O.fp8_dequantize(wb, ws, 128, 128)
    x = O.bf16_to_f32(O.bf16_bits(O.synth_normal(FP8_M * FP8_K, seed=0, stream=0))).reshape(FP8_M, FP8_K)
    ab, as_ = O.fp8_quantize(x)
    xd = O.fp8_dequantize(ab, as_)
    t0 = time.perf_counter()
    _ = xd @ wd.T
    one = max(time.perf_counter() - t0, 1e-4)
    reps = max(1, int(seconds / one))
    t0 = time.perf_counter()
    for _ in range(reps):
        _ = xd @ wd.T
    dt = (time.perf_counter() - t0) / reps
    return 2.0 * FP8_M * n * FP8_K / dt / 1e12, (
        f"{reps} x (A[{FP8_M},{FP8_K}] x W[{n} of {FP8_N},{FP8_K}]^T), dequantized FP8 (128x128 blocks, per-token A), "
        f"f32 BLAS")


def fp8_config(g: int) -> dict:
    return {"workload": "config1 FP8 GEMM M=512 K=4096 N=14336, A bf16 quantized per token on device (W8A8)",
            "matrices_per_step": FP8_MATS, "n_per_rank": FP8_N // g,
            "l2": "inputs larger than L2 (4 distinct weights, 235 MB per step at one GPU)",
            "parallelism": f"N-split x{g} + NCCL all-gather" if g > 1 else "single GPU"}


def fp8_reference_arm(args):
    rank, _, _ = dist_env()
    if rank != 0:
        return
    cores = use_all_cores()
    budget = max(5.0, min(60.0, 3.0 * (args.steps + args.warmup)))
    tflops, sample = fp8_cpu_sample(budget)
    emit({"impl": "reference", "metric": "FP8 GEMM TFLOPS", "value": tflops, "unit": "TFLOP/s",
          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
          "ms_per_step": 2.0 * FP8_M * FP8_N * FP8_K / (tflops * 1e12) * 1e3, "higher_is_better": True,
          "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Philox)",
          "config": fp8_config(args.gpus),
          "cpu_baseline": {"value": tflops, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                           "sample": sample},
          "e2e": {"value": tflops, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})


def fp8_arm(args):
    """Config 1: A bf16 [512, 4096] N(0,1) quantized per token to e4m3 on the
    device, times 4 distinct W [14336, 4096] N(0,0.02) e4m3 with 128x128 block
    scales (N-split over the ranks) per step, y bf16; 235 MB of weights per
    step at g = 1 (> L2)."""
    import torch
    import torch.distributed as dist

    import firepit_b200 as F
    N_ = F._native

    rank, world, local, dev = dist_init()
    g = world
    n_rank = FP8_N // g
    r0 = rank * n_rank
    mats = []
    for c in range(FP8_MATS):
        w = F.synth_normal((FP8_N, FP8_K), seed=0, stream_id=1 + c, std=0.02, device=dev)
        bits, scales = F.quantize_fp8(w, F.Fp8Scaling(128, 128))
        del w
        sc = scales.view(FP8_N // 128, FP8_K // 128)[r0 // 128:(r0 + n_rank) // 128].contiguous()
        mats.append(F.Fp8Matrix.from_device(bits[r0:r0 + n_rank].contiguous(), sc, n_rank, FP8_K,
                                            F.Fp8Scaling(128, 128)))
        del bits, scales
    x = F.synth_normal((FP8_M, FP8_K), seed=0, stream_id=0, dtype=torch.bfloat16, device=dev)
    qa = torch.empty(FP8_M, FP8_K, dtype=torch.uint8, device=dev)
    qs = torch.empty(FP8_M, dtype=torch.float32, device=dev)
    ys = torch.empty(FP8_MATS, FP8_M, n_rank, dtype=torch.bfloat16, device=dev)
    y_all = torch.empty(g, FP8_MATS, FP8_M, n_rank, dtype=torch.bfloat16, device=dev)
    ws_bytes = int(N_.lib.fpb_fp8_gemm_workspace_bytes(FP8_M, FP8_K)) + int(
        N_.lib.fpb_fp8_gemm_split_bytes(FP8_M, FP8_K, n_rank))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    split = torch.empty(int(N_.lib.fpb_fp8_gemm_split_bytes(FP8_M, FP8_K, n_rank)), dtype=torch.uint8, device=dev)

    def quant(sh):
        N_.call("fpb_fp8_quantize", x.data_ptr(), N_.FPB_BF16, FP8_M, FP8_K, 0, 0, qa.data_ptr(), qs.data_ptr(), sh)

    def gemms(sh):
        # stream-K schedule (one CTA per SM over all tiles' K blocks)
        for c in range(FP8_MATS):
            N_.call("fpb_fp8_gemm_q_split", mats[c].handle, 0, 0, qa.data_ptr(), qs.data_ptr(), FP8_M,
                    ys[c].data_ptr(), N_.FPB_BF16, split.data_ptr(), split.numel(), sh)

    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        quant(s.cuda_stream)
        gemms(s.cuda_stream)
    torch.cuda.synchronize()
    before = F.launch_count()
    gq, gg = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(gq, stream=s):
        quant(torch.cuda.current_stream().cuda_stream)
    with torch.cuda.graph(gg, stream=s):
        gemms(torch.cuda.current_stream().cuda_stream)
    launches_per_step = F.launch_count() - before

    def step(ev=None):
        if ev:
            ev[0].record()
        gq.replay()
        if ev:
            ev[1].record()
        gg.replay()
        if ev:
            ev[2].record()
        if g > 1:
            comm().all_gather_into(y_all, ys)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    if g > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for i in range(args.steps):
            step(evs[i])
        end.record()
        torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(end), sum(e[0].elapsed_time(e[1]) for e in evs),
                      sum(e[1].elapsed_time(e[2]) for e in evs)], device=dev, dtype=torch.float64)
    if g > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, quant_ms, gemm_ms = t.tolist()
    ms_per_step = total_ms / args.steps
    flops_step = 2.0 * FP8_M * FP8_N * FP8_K * FP8_MATS
    value = flops_step / (ms_per_step * 1e-3) / 1e12

    xh = x.cpu().pin_memory()
    yh = torch.empty(FP8_MATS, FP8_M, n_rank, dtype=torch.bfloat16, pin_memory=True)
    xd = torch.empty_like(x)
    # the reference's Graph sink: H2D x, the GEMMs and D2H y in one CUDA graph
    for c in range(FP8_MATS):
        F.fp8_gemm(mats[c], x, ys[c], workspace=ws).submit(F.Async())
    torch.cuda.synchronize()
    gsink = F.Graph()
    with gsink:
        xd.copy_(xh, non_blocking=True)
        for c in range(FP8_MATS):
            F.fp8_gemm(mats[c], xd, ys[c], workspace=ws).submit(gsink)
        yh.copy_(ys, non_blocking=True)

    def e2e_step():
        gsink.replay()

    e2e_steps = max(1, min(args.steps, 20))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if g > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = flops_step / (te.item() / e2e_steps * 1e-3) / 1e12

    per_launch_ms = gemm_ms / (args.steps * FP8_MATS)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    bf16 = float(peaks.get("bf16_tflops", 1590.0))
    achieved = 2.0 * FP8_M * n_rank * FP8_K / (per_launch_ms * 1e-3) / 1e12
    roof = {"bound": "tensor", "achieved": achieved, "peak": 2 * bf16, "unit": "TFLOP/s",
            "frac": achieved / (2 * bf16), "traffic": load_traffic("fp8_gemm_config1_traffic.txt") if g == 1 else None,
            "per_launch_us": per_launch_ms * 1e3,
            "peak_kind": "2 x measured bf16 burst (nominal dense FP8:BF16 ratio; no FP8 measurement)"}
    if rank == 0:
        line = {"metric": "FP8 GEMM TFLOPS", "value": value, "unit": "TFLOP/s", "n_gpus": g, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "e4m3 x e4m3 (128x128 block / per-token f32 scales), f32 accumulate, "
                                              "bf16 out",
                "data": "synthetic (seeded Philox: W N(0,0.02), A N(0,1) seed 0)",
                "config": fp8_config(g),
                "roofline": roof,
                "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": FP8_M * FP8_K * 2,
                        "d2h_bytes_per_step": FP8_MATS * FP8_M * n_rank * 2,
                        "path": "firepit_b200.fp8_gemm(...).submit(Graph sink): H2D x, quantize + GEMMs, D2H y in "
                                "one CUDA graph"},
                "gpu_launches": launches_per_step * args.steps, "clocks": clocks.summary(),
                "breakdown_ms": {"quantize_act": quant_ms / args.steps, "gemms": gemm_ms / args.steps}}
        if g == 1 and args.cpu_seconds > 0:
            v, sample = fp8_cpu_sample(args.cpu_seconds)
            line["cpu_baseline"] = {"value": v, "unit": "TFLOP/s", "cores": use_all_cores(), "kind": "port",
                                    "sample": sample}
    del gq, gg
    dist_sync()
    return line if rank == 0 else None


# ---- config 3: grouped MoE NVFP4 layer ---------------------------------------------------
MOE_E, MOE_K, MOE_H, MOE_I = 512, 10, 2048, 512
MOE_GU_BYTES = 2 * MOE_I * MOE_H // 2 + 2 * MOE_I * MOE_H // 16 + 4   # 1,179,652 per expert (one global)
MOE_DN_BYTES = MOE_H * MOE_I // 2 + MOE_H * MOE_I // 16 + 4           # 589,828 per expert


def moe_tokens(args):
    return 4096 if args.config == "moe_t4096" else 64


def moe_flops(tokens):
    """Useful FLOPs: router x.Wr^T plus, per route, gate/up and down."""
    return 2.0 * tokens * MOE_E * MOE_H + tokens * MOE_K * 2.0 * (2 * MOE_I * MOE_H + MOE_H * MOE_I)


def moe_bytes(tokens, touched):
    """Algorithmic HBM bytes: touched experts' weights, bf16 router, x and y (bf16)."""
    return touched * (MOE_GU_BYTES + MOE_DN_BYTES) + MOE_E * MOE_H * 2 + 2 * tokens * MOE_H * 2


def moe_cpu_sample(seconds: float, tokens_sample: int = 256):
    """The host path restated on a sample of tokens: f32 router, top-k, then per
    routed expert the dequantized NVFP4 gate/up -> SwiGLU -> down over the
    tokens routed to it (numpy/BLAS on all host cores).  Expert weights are
    dequantized once, outside the timed region.  Returns (TFLOP/s of useful
    work, sample description)."""
    import numpy as np

    from oracle import oracle as O
    x = O.bf16_to_f32(O.bf16_bits(O.synth_normal(tokens_sample * MOE_H, seed=0, stream=0))).reshape(
        tokens_sample, MOE_H)
    wr = O.bf16_to_f32(O.bf16_bits(O.synth_normal(MOE_E * MOE_H, seed=0, stream=99, std=0.02))).reshape(MOE_E, MOE_H)
    ids, w = O.moe_topk(x @ wr.T, MOE_K, 16)
    cache = {}
    for e in np.unique(ids[:, :MOE_K]):
        g = O.synth_normal(2 * MOE_I * MOE_H, seed=0, stream=1000 + int(e), std=0.02).reshape(2 * MOE_I, MOE_H)
        d = O.synth_normal(MOE_H * MOE_I, seed=0, stream=5000 + int(e), std=0.02).reshape(MOE_H, MOE_I)
        pg, sg, gg = O.nvfp4_quantize(g)
        pd, sd, gd = O.nvfp4_quantize(d)
        cache[int(e)] = (O.nvfp4_dequantize(pg, sg, gg, 2 * MOE_I, MOE_H), O.nvfp4_dequantize(pd, sd, gd, MOE_H, MOE_I))

    def layer():
        idx, wts = O.moe_topk(x @ wr.T, MOE_K, 16)
        out = np.zeros_like(x)
        for e, (w1, w2) in cache.items():
            tok, slot = np.nonzero(idx[:, :MOE_K] == e)
            if tok.size == 0:
                continue
            gu = x[tok] @ w1.T
            act = gu[:, :MOE_I] / (1.0 + np.exp(-gu[:, :MOE_I])) * gu[:, MOE_I:]
            np.add.at(out, tok, wts[tok, slot][:, None] * (act @ w2.T))
        return out

    layer()
    reps, t0 = 0, time.perf_counter()
    while True:
        layer()
        reps += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / reps
    return moe_flops(tokens_sample) / dt / 1e12, (
        f"{reps} x {tokens_sample} tokens through f32 router + top-{MOE_K} of {MOE_E} + dequantized NVFP4 expert "
        f"MLPs grouped by expert (f32 BLAS; weights dequantized beforehand)")


def moe_config(tokens: int, g: int, ep: bool = False) -> dict:
    if ep:
        return {"workload": f"config3 MoE E=512 top-10 H=2048 I=512, T=4096 per rank, EP x{g}",
                "experts_per_gpu": MOE_E // g,
                "parallelism": f"EP x{g} + NCCL all-to-all" if g > 1 else "single GPU (no exchange)",
                "l2": "inputs larger than L2 (all local experts' weights per step)"}
    return {"workload": f"config3 MoE E=512 top-10 H=2048 I=512 T={tokens}, no shared expert",
            "l2": "inputs larger than L2 (the touched experts' weights per step)",
            "parallelism": "single GPU", "tile_rows": 128}


def moe_reference_arm(args):
    rank, _, _ = dist_env()
    if rank != 0:
        return
    cores = use_all_cores()
    v, sample = moe_cpu_sample(min(60.0, max(5.0, 2.0 * (args.steps + args.warmup))))
    T = 4096 if args.config == "moe_ep" else moe_tokens(args)
    emit({"impl": "reference", "metric": "NVFP4 MoE layer TFLOPS", "value": v, "unit": "TFLOP/s",
          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
          "ms_per_step": moe_flops(T) / (v * 1e12) * 1e3, "higher_is_better": True,
          "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Philox)",
          "config": moe_config(T, args.gpus, args.config == "moe_ep"),
          "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample},
          "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})


def moe_arm(args):
    """Config 3 at T = 4096 (prefill) or 64 (decode batch), one GPU: bf16 x
    [T, 2048], bf16 router [512, 2048] (cuBLAS, f32 logits), device top-10,
    device layout (128-row tiles), NVFP4 quantize of each token once + copy
    of its codes to the rows that route it, grouped gate/up
    GEMM [512 x 1024, 2048] with SwiGLU in its epilogue (h in bf16 and its
    amax), NVFP4 quantize of h, grouped down GEMM [512 x 2048, 512], weighted
    combine; one CUDA graph per step.  The layout's padding rows (each
    expert's rows rounded up to the 128-row tile) are skipped by the encoders
    and not stored by the GEMMs."""
    import torch

    import firepit_b200 as F
    N_ = F._native
    rank, world, local, dev = dist_init()
    T = moe_tokens(args)
    # weights: each expert its own global; streams 1000+e / 5000+e as in the CPU sample
    gu_parts, dn_parts = [], []
    chunk = 64
    gp = torch.empty(MOE_E * 2 * MOE_I, MOE_H // 2, dtype=torch.uint8, device=dev)
    gs = torch.empty(MOE_E * 2 * MOE_I, MOE_H // 16, dtype=torch.uint8, device=dev)
    gg = torch.empty(MOE_E * 2 * MOE_I, dtype=torch.float32, device=dev)
    dp = torch.empty(MOE_E * MOE_H, MOE_I // 2, dtype=torch.uint8, device=dev)
    ds = torch.empty(MOE_E * MOE_H, MOE_I // 16, dtype=torch.uint8, device=dev)
    dg = torch.empty(MOE_E * MOE_H, dtype=torch.float32, device=dev)
    for e0 in range(0, MOE_E, chunk):
        g = torch.empty(chunk, 2 * MOE_I, MOE_H, device=dev)
        d = torch.empty(chunk, MOE_H, MOE_I, device=dev)
        for j in range(chunk):
            F.synth_normal(g[j].shape, seed=0, stream_id=1000 + e0 + j, std=0.02, out=g[j])
            F.synth_normal(d[j].shape, seed=0, stream_id=5000 + e0 + j, std=0.02, out=d[j])
        a, b, c = F.quantize_nvfp4(g.view(-1, MOE_H), 2 * MOE_I)
        r0, r1 = e0 * 2 * MOE_I, (e0 + chunk) * 2 * MOE_I
        gp[r0:r1], gs[r0:r1], gg[r0:r1] = a, b, c
        a, b, c = F.quantize_nvfp4(d.view(-1, MOE_I), MOE_H)
        r0, r1 = e0 * MOE_H, (e0 + chunk) * MOE_H
        dp[r0:r1], ds[r0:r1], dg[r0:r1] = a, b, c
        del g, d
    W1 = F.Nvfp4Matrix.from_device(gp, gs, gg, MOE_E * 2 * MOE_I, MOE_H)
    W2 = F.Nvfp4Matrix.from_device(dp, ds, dg, MOE_E * MOE_H, MOE_I)
    del gp, gs, gg, dp, ds, dg
    s0 = torch.cuda.current_stream().cuda_stream
    W1.prepare_glu(MOE_I, s0)  # load time: the layer's calls allocate nothing
    wr = F.synth_normal((MOE_E, MOE_H), seed=0, stream_id=99, std=0.02, dtype=torch.bfloat16, device=dev)
    x = F.synth_normal((T, MOE_H), seed=0, stream_id=0, dtype=torch.bfloat16, device=dev)
    router = F.MoeDims.new(MOE_H, MOE_I, MOE_I, MOE_E, MOE_K)
    width = router.width()
    cap = F.PrefillPlan.capacity(T, router, 128)
    i32 = dict(dtype=torch.int32, device=dev)
    buf = dict(logits=torch.empty(T, MOE_E, device=dev), ids=torch.empty(T, width, **i32),
               w=torch.empty(T, width, device=dev), tr=torch.empty(cap, **i32), te=torch.empty(cap // 128, **i32),
               inv=torch.empty(T, width, **i32), rg=torch.empty(MOE_E, 2, dtype=torch.int64, device=dev),
               pad=torch.empty(1, **i32),
               a1=torch.empty(cap, MOE_H // 2, dtype=torch.uint8, device=dev),
               sf1=torch.empty(int(N_.lib.fpb_nvfp4_act_sf_bytes(cap, MOE_H)), dtype=torch.uint8, device=dev),
               h=torch.empty(cap, MOE_I, dtype=torch.bfloat16, device=dev),
               a2=torch.empty(cap, MOE_I // 2, dtype=torch.uint8, device=dev),
               sf2=torch.empty(int(N_.lib.fpb_nvfp4_act_sf_bytes(cap, MOE_I)), dtype=torch.uint8, device=dev),
               y2=torch.empty(cap, MOE_H, dtype=torch.bfloat16, device=dev),
               out=torch.empty(T, MOE_H, dtype=torch.bfloat16, device=dev),
               scal=torch.zeros(4, dtype=torch.float32, device=dev),
               lscr=torch.empty(int(N_.lib.fpb_moe_layout_scratch_bytes(T, MOE_K, MOE_E)), dtype=torch.uint8,
                                device=dev),
               gws=torch.empty(int(N_.lib.fpb_moe_gather_quantize_workspace_bytes(T, MOE_H)), dtype=torch.uint8,
                               device=dev))
    b = buf
    BF = N_.FPB_BF16

    def moe(sh, xin, ev=None):
        def mark(i):
            if ev is not None:
                ev[i].record()
        mark(0)
        torch.mm(xin, wr.t(), out_dtype=torch.float32, out=b["logits"])
        mark(1)
        N_.call("fpb_moe_topk", b["logits"].data_ptr(), MOE_E, None, T, MOE_E, MOE_K, width, b["ids"].data_ptr(),
                b["w"].data_ptr(), sh)
        N_.call("fpb_moe_layout", b["ids"].data_ptr(), T, width, MOE_K, MOE_E, 128, cap, b["tr"].data_ptr(),
                b["te"].data_ptr(), b["inv"].data_ptr(), b["rg"].data_ptr(), b["pad"].data_ptr(), b["lscr"].data_ptr(),
                b["lscr"].numel(), sh)
        # padding rows of the layout (token -1) are skipped by every stage below
        skip = N_.FPB_QUANT_SKIP_PADDING
        N_.call("fpb_moe_gather_quantize", xin.data_ptr(), BF, T, MOE_H, b["tr"].data_ptr(), cap, b["pad"].data_ptr(),
                b["a1"].data_ptr(), b["sf1"].data_ptr(), b["scal"].data_ptr(), b["scal"][1:].data_ptr(), skip,
                b["gws"].data_ptr(), b["gws"].numel(), sh)
        mark(2)
        N_.call("fpb_nvfp4_grouped_gemm_swiglu_q", W1.handle, b["a1"].data_ptr(), b["sf1"].data_ptr(),
                b["scal"].data_ptr(), cap, b["te"].data_ptr(), b["tr"].data_ptr(), MOE_I, b["h"].data_ptr(), BF,
                b["scal"][3:].data_ptr(), sh)
        mark(3)
        N_.call("fpb_rows_quantize", b["h"].data_ptr(), BF, cap, b["pad"].data_ptr(), b["tr"].data_ptr(), MOE_I,
                b["a2"].data_ptr(), b["sf2"].data_ptr(), b["scal"][2:].data_ptr(), b["scal"][3:].data_ptr(),
                N_.FPB_QUANT_AMAX_GIVEN | skip, sh)
        mark(4)
        N_.call("fpb_nvfp4_grouped_gemm_q", W2.handle, b["a2"].data_ptr(), b["sf2"].data_ptr(),
                b["scal"][2:].data_ptr(), cap, b["te"].data_ptr(), b["tr"].data_ptr(), MOE_H, b["y2"].data_ptr(), BF,
                sh)
        mark(5)
        N_.call("fpb_moe_combine", b["y2"].data_ptr(), BF, cap, MOE_H, b["inv"].data_ptr(), b["w"].data_ptr(), T,
                width, MOE_K, b["out"].data_ptr(), BF, sh)
        mark(6)

    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        moe(s.cuda_stream, x)
    torch.cuda.synchronize()
    assert F.device_error() == 0
    touched = int((b["rg"][:, 1] > 0).sum().item())
    before = F.launch_count()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        moe(torch.cuda.current_stream().cuda_stream, x)
    launches_per_step = F.launch_count() - before
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for _ in range(args.steps):
            graph.replay()
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    # per-stage breakdown (eager launches with events)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(7)]
    with torch.cuda.stream(s):
        moe(s.cuda_stream, x, evs)
    torch.cuda.synchronize()
    names = ["router_gemm", "topk_layout_gather_quant", "gate_up_swiglu_gemm", "h_quant", "down_gemm", "combine"]
    breakdown = {n: evs[i].elapsed_time(evs[i + 1]) for i, n in enumerate(names)}
    flops = moe_flops(T)
    value = flops / (ms * 1e-3) / 1e12
    nbytes = moe_bytes(T, touched)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    achieved = nbytes / (ms * 1e-3) / 1e9
    # end to end: x from pinned host, out back to pinned host, the same C-ABI
    # calls; copies and layer in one CUDA graph (the engine's graph sink)
    xh = x.cpu().pin_memory()
    oh = torch.empty(T, MOE_H, dtype=torch.bfloat16, pin_memory=True)
    xd = torch.empty_like(x)
    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e2e_graph, stream=s):
        xd.copy_(xh, non_blocking=True)
        moe(torch.cuda.current_stream().cuda_stream, xd)
        oh.copy_(b["out"], non_blocking=True)
    e2e_steps = max(1, min(args.steps, 20))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for i in range(e2e_steps + 2):
        if i == 2:
            e0.record()
        e2e_graph.replay()
    e1.record()
    torch.cuda.synchronize()
    e2e = flops / (e0.elapsed_time(e1) / e2e_steps * 1e-3) / 1e12
    del e2e_graph
    line = {"metric": "NVFP4 MoE layer TFLOPS", "value": value, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": "nvfp4 x nvfp4 experts (f32 accumulate), bf16 router (f32 logits), bf16 activations",
            "data": "synthetic (seeded Philox: W N(0,0.02) per expert, x N(0,1) seed 0)",
            "config": moe_config(T, 1),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "traffic": None, "algorithmic_bytes": nbytes, "peak_kind": "measured hbm_gbs",
                         "note": "whole MoE layer time; the grouped GEMMs are the dominant kernels"},
            "e2e": {"value": e2e, "unit": "TFLOP/s", "h2d_bytes_per_step": T * MOE_H * 2,
                    "path": "C-ABI calls of the layer with H2D x and D2H out in one CUDA graph",
                    "d2h_bytes_per_step": T * MOE_H * 2},
            "gpu_launches": launches_per_step * args.steps, "clocks": clocks.summary(), "breakdown_ms": breakdown,
            "touched_experts": touched}
    if args.cpu_seconds > 0 and rank == 0:
        v, sample = moe_cpu_sample(args.cpu_seconds)
        line["cpu_baseline"] = {"value": v, "unit": "TFLOP/s", "cores": use_all_cores(), "kind": "port",
                                "sample": sample}
    del graph
    return line if rank == 0 else None


def moe_ep_arm(args):
    """Config 3 expert-parallel: E=512 experts split over the ranks (64 per GPU
    at 8), T=4096 tokens per rank (weak scaling), firepit_b200.ep.EpMoeLayer:
    one NVFP4 record per (token, destination rank) in fixed-size chunks, NCCL
    all-to-all out and back (the library's fpb_comm_*), activation globals
    all-reduced so every rank encodes like the single-GPU layer, partial sums
    per record returned in f32; router GEMM + layer in one CUDA graph per
    rank."""
    import torch
    import torch.distributed as dist

    import firepit_b200 as F
    from firepit_b200.ep import DeviceEpOps, EpMoeLayer
    rank, world, local, dev = dist_init()
    T = 4096
    per = MOE_E // world
    e0 = rank * per
    gp = torch.empty(per * 2 * MOE_I, MOE_H // 2, dtype=torch.uint8, device=dev)
    gs = torch.empty(per * 2 * MOE_I, MOE_H // 16, dtype=torch.uint8, device=dev)
    gg = torch.empty(per * 2 * MOE_I, dtype=torch.float32, device=dev)
    dp = torch.empty(per * MOE_H, MOE_I // 2, dtype=torch.uint8, device=dev)
    ds = torch.empty(per * MOE_H, MOE_I // 16, dtype=torch.uint8, device=dev)
    dg = torch.empty(per * MOE_H, dtype=torch.float32, device=dev)
    chunk = min(64, per)
    for c0 in range(0, per, chunk):
        g = torch.empty(chunk, 2 * MOE_I, MOE_H, device=dev)
        d = torch.empty(chunk, MOE_H, MOE_I, device=dev)
        for j in range(chunk):
            F.synth_normal(g[j].shape, seed=0, stream_id=1000 + e0 + c0 + j, std=0.02, out=g[j])
            F.synth_normal(d[j].shape, seed=0, stream_id=5000 + e0 + c0 + j, std=0.02, out=d[j])
        a, b_, c = F.quantize_nvfp4(g.view(-1, MOE_H), 2 * MOE_I)
        gp[c0 * 2 * MOE_I:(c0 + chunk) * 2 * MOE_I], gs[c0 * 2 * MOE_I:(c0 + chunk) * 2 * MOE_I] = a, b_
        gg[c0 * 2 * MOE_I:(c0 + chunk) * 2 * MOE_I] = c
        a, b_, c = F.quantize_nvfp4(d.view(-1, MOE_I), MOE_H)
        dp[c0 * MOE_H:(c0 + chunk) * MOE_H], ds[c0 * MOE_H:(c0 + chunk) * MOE_H], dg[c0 * MOE_H:(c0 + chunk) * MOE_H] = (
            a, b_, c)
        del g, d
    W1 = F.Nvfp4Matrix.from_device(gp, gs, gg, per * 2 * MOE_I, MOE_H)
    W2 = F.Nvfp4Matrix.from_device(dp, ds, dg, per * MOE_H, MOE_I)
    W1.prepare_glu(MOE_I)
    del gp, gs, gg, dp, ds, dg
    wr = F.synth_normal((MOE_E, MOE_H), seed=0, stream_id=99, std=0.02, dtype=torch.bfloat16, device=dev)
    x = F.synth_normal((T, MOE_H), seed=rank, stream_id=0, dtype=torch.bfloat16, device=dev)
    # peer mode on more than one GPU: dispatch and the partial combine store
    # straight into the other GPUs' receive buffers (CUDA IPC over NVLink)
    ops = DeviceEpOps(dev, T, MOE_H, MOE_I, MOE_E, MOE_K, world, W1, W2, ipc=world > 1)
    layer = EpMoeLayer(ops, comm=comm())
    layer.connect_peers()
    logits = torch.empty(T, MOE_E, device=dev)

    def step(xin, ev=None):
        if ev is not None:
            ev[0].record()
        torch.mm(xin, wr.t(), out_dtype=torch.float32, out=logits)
        if ev is not None:
            ev[1].record()
        return layer.forward(xin, logits, None if ev is None else (lambda i: ev[i + 2].record()))

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step(x)
    torch.cuda.synchronize()
    assert F.device_error() == 0
    before = F.launch_count()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        step(x)
    launches_per_step = F.launch_count() - before
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    dist_sync()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for _ in range(args.steps):
            graph.replay()
        end.record()
        torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(end)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item() / args.steps
    flops = world * moe_flops(T)
    value = flops / (ms * 1e-3) / 1e12
    # per-stage breakdown (eager launches with events on every rank, max over ranks)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(2 + len(EpMoeLayer.STAGES))]
    dist_sync()
    with torch.cuda.stream(s):
        step(x, evs)
    torch.cuda.synchronize()
    names = ("router_gemm",) + EpMoeLayer.STAGES
    bd = torch.tensor([evs[i].elapsed_time(evs[i + 1]) for i in range(len(names))], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(bd, op=dist.ReduceOp.MAX)
    breakdown = dict(zip(names, bd.tolist()))
    # end to end through the public entry (EpMoeLayer.forward): the rank's
    # tokens copied in from pinned host memory and the output back, in the
    # same CUDA graph as the layer
    xh = x.cpu().pin_memory()
    yh = torch.empty(T, MOE_H, dtype=torch.bfloat16, pin_memory=True)
    xd = torch.empty_like(x)
    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e2e_graph, stream=s):
        xd.copy_(xh, non_blocking=True)
        yh.copy_(step(xd), non_blocking=True)
    for _ in range(2):
        e2e_graph.replay()
    torch.cuda.synchronize()
    dist_sync()
    torch.cuda.synchronize()
    e2e_steps = max(1, min(args.steps, 20))
    start.record()
    for _ in range(e2e_steps):
        e2e_graph.replay()
    end.record()
    torch.cuda.synchronize()
    te = torch.tensor([start.elapsed_time(end)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = flops / (te.item() / e2e_steps * 1e-3) / 1e12
    del graph, e2e_graph
    assert F.device_error() == 0
    torch.cuda.synchronize()
    dist_sync()
    layer.close_peers()
    dist_sync()  # no rank frees a buffer another still maps
    ops.free()
    nbytes = world * moe_bytes(T, per)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    achieved = nbytes / world / (ms * 1e-3) / 1e9
    out = None
    if rank == 0:
        out = {"metric": "NVFP4 MoE layer TFLOPS", "value": value, "unit": "TFLOP/s", "n_gpus": world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None,
               "dtype": "nvfp4 x nvfp4 experts (f32 accumulate), bf16 router, nvfp4 dispatch, f32 partials back",
               "exchange": "peer stores over NVLink (CUDA IPC) from the dispatch and partial-combine kernels, "
                           "one-word all-reduce barriers" if world > 1 else "none",
               "data": "synthetic (seeded Philox: W N(0,0.02) per expert, x N(0,1) per rank)",
               "config": moe_config(T, world, ep=True),
               "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                            "frac": achieved / hbm, "traffic": None, "peak_kind": "measured hbm_gbs",
                            "note": "per GPU: local experts' weights + router + x + y over the layer time"},
               "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": world * T * MOE_H * 2,
                       "d2h_bytes_per_step": world * T * MOE_H * 2,
                       "path": "firepit_b200.ep.EpMoeLayer.forward on x copied from pinned host memory, output "
                               "copied back, in one CUDA graph per rank"},
               "gpu_launches": launches_per_step * args.steps, "clocks": clocks.summary(), "breakdown_ms": breakdown,
               "exchange_bytes_per_rank": {"dispatch": world * T * ops.rec, "return": world * T * MOE_H * 4}}
    dist_sync()
    return out


# ---- config 4: decode of the random-init hybrid MoE decoder ------------------------------
DEC_SESSIONS, DEC_PROMPT, DEC_STEPS = 8, 2048, 256


def decode_config(g: int, prompt: int = DEC_PROMPT, steps: int = DEC_STEPS) -> dict:
    return {"workload": "config4 48-layer hybrid MoE decoder (36 GDN + 12 full-attention layers, H=2048, vocab 151936,"
                        f" 512 experts top-10 + shared, all linear weights NVFP4), 8 sessions x {prompt}-token random "
                        f"prompt, {steps} greedy tokens",
            "sessions_per_gpu": DEC_SESSIONS, "prompt": prompt, "decode_steps": steps,
            "parallelism": f"replicas x{g}: each GPU decodes its own 8 sessions, no exchange" if g > 1
            else "single GPU",
            "prompt_path": "the decode step, one prompt token per step (untimed)",
            "timing": "the 256 decode steps, one CUDA graph per step, CUDA events, max over ranks"}


def decode_cpu_sample(seconds: float, layers_sample: int = 4):
    """The host path restated (numpy): one decode step of one session at
    position 0 through the first `layers_sample` layers of a model of the
    same shapes (weights generated by the oracle, dequantized outside the
    timed region), scaled to 48 layers; tokens/s = 1 / that step time."""
    import numpy as np

    from oracle import model_ops as R
    from oracle import oracle as O
    cores = use_all_cores()
    H, I, E, K = 2048, 512, 512, 10
    rng = np.random.default_rng(0)

    def mat(rows, cols, sid):
        w = O.synth_normal(rows * cols, seed=7, stream=sid, std=0.02).reshape(rows, cols)
        p, sc, gl = O.nvfp4_quantize(w)
        return O.nvfp4_dequantize(p, sc, gl, rows, cols)

    Ls = []
    for i in range(layers_sample):
        L = {"g": np.ones(H, np.float32)}
        if (i + 1) % 4 == 0:
            L["qg"], L["k"], L["v"], L["o"] = mat(8192, H, 10 * i), mat(512, H, 10 * i + 1), mat(512, H, 10 * i + 2), \
                mat(H, 4096, 10 * i + 3)
        else:
            L["qkv"], L["z"], L["ab"], L["out"] = mat(8192, H, 10 * i), mat(4096, H, 10 * i + 1), \
                mat(64, H, 10 * i + 2), mat(H, 4096, 10 * i + 3)
            L["conv"] = rng.standard_normal((8192, 4)).astype(np.float32) * 0.2
        L["router"] = mat(E + 1, H, 10 * i + 4)
        Ls.append(L)
    experts = {}

    def expert(e):
        if e not in experts:
            experts[e] = (mat(2 * I, H, 5000 + e), mat(H, I, 9000 + e))
        return experts[e]

    x0 = rng.standard_normal(H).astype(np.float32) * 0.02
    for i in range(layers_sample):  # dequantize the experts the sample routes to
        lg = (R.rms_norm(x0, Ls[i]["g"], 1e-6) @ Ls[i]["router"].T).astype(np.float32)
        ids, _ = O.moe_topk(lg[None, :E], K, K + 1, lg[None, E:E + 1])
        for e in ids[0]:
            expert(int(e))

    def step():
        x = x0.astype(np.float64)
        for i, L in enumerate(Ls):
            n = R.rms_norm(x.astype(np.float32), L["g"], 1e-6)
            if "qkv" in L:
                qkv = n @ L["qkv"].T
                z = n @ L["z"].T
                ab = n @ L["ab"].T
                co, _ = R.conv1d_silu(qkv, np.zeros((8192, 3), np.float32), L["conv"])
                o, _ = R.delta_step(co[:2048].reshape(16, 128), co[2048:4096].reshape(16, 128),
                                    co[4096:].reshape(32, 128), ab[:32], ab[32:], np.zeros(32), np.zeros(32),
                                    np.zeros((32, 128, 128)), 1e-6, 16)
                d = R.gated_norm(o.astype(np.float32), z.reshape(32, 128), np.ones(128, np.float32), 1e-6)
                x = x + d.reshape(-1) @ L["out"].T
            else:
                qg = n @ L["qg"].T
                vv = n @ L["v"].T
                att = np.repeat(vv.reshape(2, 256), 8, axis=0)  # position 0: attention returns v
                x = x + (att * R.sigmoid(qg.reshape(16, 512)[:, 256:])).reshape(-1) @ L["o"].T
            n = R.rms_norm(x.astype(np.float32), L["g"], 1e-6)
            lg = (n @ L["router"].T).astype(np.float32)
            ids, w = O.moe_topk(lg[None, :E], K, K + 1, lg[None, E:E + 1])
            moe = np.zeros(H)
            for s_, e in enumerate(ids[0]):
                w1, w2 = expert(int(e))
                gu = n @ w1.T
                moe += w[0, s_] * ((gu[:I] * R.sigmoid(gu[:I]) * gu[I:]) @ w2.T)
            x = x + moe
        return x

    step()
    reps, t0 = 0, time.perf_counter()
    while reps < 2 or time.perf_counter() - t0 < seconds:
        step()
        reps += 1
    per_layer = (time.perf_counter() - t0) / reps / layers_sample
    step_s = per_layer * 48
    return 1.0 / step_s, (f"{reps} x one decode step of one session through the first {layers_sample} layers "
                          f"(numpy f64 on dequantized NVFP4 weights), scaled to 48 layers: {step_s * 1e3:.0f} ms "
                          f"per token"), cores


def decode_reference_arm(args):
    rank, _, _ = dist_env()
    if rank != 0:
        return
    v, sample, cores = decode_cpu_sample(min(60.0, max(5.0, 0.2 * (args.steps + args.warmup))))
    emit({"impl": "reference", "metric": "decode tokens/s", "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / v, "higher_is_better": True,
          "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded)",
          "config": decode_config(args.gpus, args.dec_prompt, args.dec_steps),
          "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
          "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})


def decode_arm(args):
    """Config 4 on each GPU (replicas): build the model, run the 8 sessions'
    2048-token prompts through the decode step (untimed), then time 256
    greedy decode steps (CUDA graph replay)."""
    import torch
    import torch.distributed as dist

    import firepit_b200 as F
    from firepit_b200.model import Decoder, HybridConfig, HybridModel
    rank, world, local, dev = dist_init()
    cfg = HybridConfig()
    t_build = time.perf_counter()
    model = HybridModel(cfg, seed=0, device=dev)
    build_s = time.perf_counter() - t_build
    B, steps, plen = DEC_SESSIONS, args.dec_steps, args.dec_prompt
    dec = Decoder(model, B, plen + steps, history_len=steps)
    prompt = torch.randint(0, cfg.vocab, (B, plen), dtype=torch.int32, device=dev,
                           generator=torch.Generator(device=dev).manual_seed(1000 + rank))
    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):  # every code path once, outside capture
        dec.step(s.cuda_stream)
    torch.cuda.synchronize()
    dec.reset()
    before = F.launch_count()
    dec.capture()
    launches_per_step = F.launch_count() - before
    dec.reset()
    t_pre = time.perf_counter()
    dec.prefill(prompt)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t_pre
    dist_sync()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        dec.generate(steps)
        end.record()
        torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(end)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item() / steps
    value = world * B * steps / (t.item() * 1e-3)
    assert F.device_error() == 0
    # routes of one more step: distinct experts each layer reads
    dec.route_log = torch.zeros(cfg.layers, B, cfg.slots, dtype=torch.int32, device=dev)
    dec.step(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    distinct = [int(torch.unique(dec.route_log[i]).numel()) for i in range(cfg.layers)]
    dec.route_log = None
    wb = model.weight_bytes()
    pos = plen + steps // 2
    kv_bytes = sum(1 for i in range(cfg.layers) if cfg.is_attention(i)) * B * pos * cfg.kv_heads * cfg.head_dim * 4 * 2
    gdn_bytes = sum(1 for i in range(cfg.layers) if not cfg.is_attention(i)) * B * cfg.value_heads * \
        cfg.key_head_dim * cfg.value_head_dim * 4 * 2
    step_bytes = wb["dense"] + wb["lm_head"] + sum(distinct) * wb["expert"] + kv_bytes + gdn_bytes
    hbm, kind = measured_peak()
    achieved = step_bytes / (ms * 1e-3) / 1e9
    # e2e: a serving loop that hands every step's tokens to the host and
    # feeds them back (pinned buffers, a synchronisation per step)
    tok_h = torch.zeros(B, dtype=torch.int32, pin_memory=True)
    e2e_steps = 32
    dec.reset()
    dec.prefill(prompt[:, :min(64, plen)])
    torch.cuda.synchronize()
    e0 = time.perf_counter()
    for i in range(e2e_steps):
        if i:
            dec.tokens.copy_(tok_h, non_blocking=True)
        dec.graph.replay()
        tok_h.copy_(dec.tokens, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e2e_s = time.perf_counter() - e0
    te = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world * B * e2e_steps / te.item()
    out = None
    if rank == 0:
        out = {"metric": "decode tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
               "warmup": plen, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None,
               "dtype": "nvfp4 weights (e2m1 x e4m3, f32 accumulate), f32 activations and state, bf16 GEMV inputs",
               "data": "synthetic (seeded Philox weights N(0,0.02) -> NVFP4; random prompt ids)",
               "config": decode_config(world, plen, steps),
               "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                            "frac": achieved / hbm, "traffic": None, "peak_kind": f"{kind} hbm_gbs",
                            "algorithmic_bytes_per_step": step_bytes,
                            "note": "per GPU per step: dense + LM-head NVFP4 weights, the distinct experts routed "
                                    "in each layer (one sampled step), KV caches at the mid position, GDN states "
                                    "read and written"},
               "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": 4 * B,
                       "d2h_bytes_per_step": 4 * B,
                       "path": "Decoder graph step with each step's tokens copied to pinned host memory and back, "
                               "a host synchronisation per step (32 steps after a 64-token prompt)"},
               "gpu_launches": launches_per_step * steps, "clocks": clocks.summary(),
               "breakdown": {"build_s": build_s, "prompt_s": prefill_s, "distinct_experts_per_layer_mean":
                             sum(distinct) / len(distinct), "step_gb": step_bytes / 1e9}}
        if world == 1 and args.cpu_seconds > 0:
            v, sample, cores = decode_cpu_sample(args.cpu_seconds)
            out["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}
    del dec, model
    torch.cuda.empty_cache()
    dist_sync()
    return out


SUB_RECORDS = [
    # (name, config, runs at one GPU, runs at several GPUs)
    ("config1_fp8_gemm", "fp8_gemm", True, True),
    ("config2_m1", "nvfp4_gemm_m1", True, True),
    ("config2_m16", "nvfp4_gemm_m16", True, True),
    ("config2_m128", "nvfp4_gemm_m128", True, True),
    ("config2_m2048", "nvfp4_gemm_m2048", True, True),
    ("config3_moe_t64", "moe_t64", True, False),
    ("config3_moe_t4096", "moe_t4096", True, False),
    ("config3_moe_ep", "moe_ep", False, True),
    ("config4_decode", "decode", True, True),
]


def product_arm(config: str):
    if config == "decode":
        return decode_arm
    if config == "moe_ep":
        return moe_ep_arm
    if config.startswith("moe_"):
        return moe_arm
    if config == "fp8_gemm":
        return fp8_arm
    if config in ("nvfp4_gemm_m1", "nvfp4_gemm_m16"):
        return gemm_small_arm
    if config.startswith("nvfp4_gemm"):
        return gemm_arm
    return ours_arm


def reference_for(config: str):
    if config == "decode":
        return decode_reference_arm
    if config.startswith("moe_"):
        return moe_reference_arm
    if config == "fp8_gemm":
        return fp8_reference_arm
    if config.startswith("nvfp4_gemm"):
        return gemm_reference_arm
    return reference_arm


def main():
    args = parse_args()
    if args.impl == "reference":
        # The CPU legs use every host core (numpy's BLAS reads this at import).
        os.environ["OMP_NUM_THREADS"] = str(os.cpu_count() or 1)
        reference_for(args.config)(args)
        return
    import copy

    import torch
    line = product_arm(args.config)(args)
    if args.config == "gemv" and not args.no_sub:
        _, world, _ = dist_env()
        subs = {}
        for name, config, one, many in SUB_RECORDS:
            if not (one if world == 1 else many):
                continue
            sub = copy.copy(args)
            sub.config, sub.steps, sub.warmup, sub.cpu_seconds = config, args.sub_steps, 3, args.sub_cpu_seconds
            rec = product_arm(config)(sub)
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
            if line is not None:
                subs[name] = rec
        if line is not None:
            line["sub_records"] = subs
    if line is not None:
        emit(line)
    dist_finish()


if __name__ == "__main__":
    main()
