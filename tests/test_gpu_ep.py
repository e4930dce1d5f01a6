"""Expert-parallel MoE on 2 GPUs over NCCL (skipped with fewer GPUs).

Two ranks, 16 experts (8 per rank), top-4, each rank routing its own 300
tokens.  The quantizers' globals are all-reduced over the ranks, so each
rank's output must equal, bit for bit, the single-GPU layer run over both
ranks' tokens with all experts (NVLS is kept off; collectives use a short
timeout)."""
import os
import socket
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
E, K, H, I, T = 16, 4, 256, 128, 300


def _rank(rank, world, port, q):
    sys.path[:0] = [ROOT, HERE]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import firepit_b200 as F
    from firepit_b200.ep import DeviceOps, ep_moe_forward
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        w1 = F.synth_normal((E * 2 * I, H), seed=1, stream_id=1, std=0.02, device=dev)
        w2 = F.synth_normal((E * H, I), seed=2, stream_id=1, std=0.02, device=dev)
        p1, s1, g1 = F.quantize_nvfp4(w1, 2 * I)
        p2, s2, g2 = F.quantize_nvfp4(w2, H)
        per = E // world
        r1 = slice(rank * per * 2 * I, (rank + 1) * per * 2 * I)
        r2 = slice(rank * per * H, (rank + 1) * per * H)
        L1 = F.Nvfp4Matrix.from_device(p1[r1].contiguous(), s1[r1].contiguous(), g1[r1].contiguous(), per * 2 * I, H)
        L2 = F.Nvfp4Matrix.from_device(p2[r2].contiguous(), s2[r2].contiguous(), g2[r2].contiguous(), per * H, I)
        A1 = F.Nvfp4Matrix.from_device(p1, s1, g1, E * 2 * I, H)
        A2 = F.Nvfp4Matrix.from_device(p2, s2, g2, E * H, I)
        x_all = F.synth_normal((world * T, H), seed=0, stream_id=0, dtype=torch.bfloat16, device=dev)
        lg_all = F.synth_normal((world * T, E), seed=0, stream_id=7, device=dev)
        rows = slice(rank * T, (rank + 1) * T)
        ops = DeviceOps(dev)
        y_ep = ep_moe_forward(ops, x_all[rows].contiguous(), lg_all[rows].contiguous(), K, E, L1, L2)
        y_one = ep_moe_forward(ops, x_all, lg_all, K, E, A1, A2, world=1)[rows]
        torch.cuda.synchronize()
        q.put((rank, F.device_error(), y_ep.float().cpu().numpy().tobytes(), y_one.float().cpu().numpy().tobytes()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_expert_parallel_two_gpus_matches_single_gpu():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, err, ep, one in results:
        a = np.frombuffer(ep, np.float32)
        b = np.frombuffer(one, np.float32)
        assert err == 0
        assert np.all(np.isfinite(a)) and np.abs(b).max() > 0
        assert np.array_equal(a, b), f"rank {rank}: max diff {np.abs(a - b).max()}"


def _rank_fixed(rank, world, port, q):
    """EpMoeLayer over the library's NCCL communicator, eager and as one
    CUDA graph per rank (replayed twice)."""
    sys.path[:0] = [ROOT, HERE]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import firepit_b200 as F
    from firepit_b200.comm import Comm
    from firepit_b200.ep import DeviceEpOps, DeviceOps, EpMoeLayer, ep_moe_forward
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    comm = None
    graph = graph_p = layer_p = None
    try:
        comm = Comm.from_torch()
        w1 = F.synth_normal((E * 2 * I, H), seed=1, stream_id=1, std=0.02, device=dev)
        w2 = F.synth_normal((E * H, I), seed=2, stream_id=1, std=0.02, device=dev)
        p1, s1, g1 = F.quantize_nvfp4(w1, 2 * I)
        p2, s2, g2 = F.quantize_nvfp4(w2, H)
        per = E // world
        r1 = slice(rank * per * 2 * I, (rank + 1) * per * 2 * I)
        r2 = slice(rank * per * H, (rank + 1) * per * H)
        L1 = F.Nvfp4Matrix.from_device(p1[r1].contiguous(), s1[r1].contiguous(), g1[r1].contiguous(), per * 2 * I, H)
        L2 = F.Nvfp4Matrix.from_device(p2[r2].contiguous(), s2[r2].contiguous(), g2[r2].contiguous(), per * H, I)
        L1.prepare_glu(I)
        A1 = F.Nvfp4Matrix.from_device(p1, s1, g1, E * 2 * I, H)
        A2 = F.Nvfp4Matrix.from_device(p2, s2, g2, E * H, I)
        x_all = F.synth_normal((world * T, H), seed=0, stream_id=0, dtype=torch.bfloat16, device=dev)
        lg_all = F.synth_normal((world * T, E), seed=0, stream_id=7, device=dev)
        rows = slice(rank * T, (rank + 1) * T)
        x, lg = x_all[rows].contiguous(), lg_all[rows].contiguous()
        layer = EpMoeLayer(DeviceEpOps(dev, T, H, I, E, K, world, L1, L2), comm=comm)
        y_eager = layer.forward(x, lg).clone()
        y_one = ep_moe_forward(DeviceOps(dev), x_all, lg_all, K, E, A1, A2, world=1)[rows]
        torch.cuda.synchronize()
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            y_g = layer.forward(x, lg)
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        # peer mode: the chunks stored straight into the other GPU's buffers (CUDA IPC), barriers instead of
        # all-to-alls; the same sums, so the same bits as the all-to-all form
        layer_p = EpMoeLayer(DeviceEpOps(dev, T, H, I, E, K, world, L1, L2, ipc=True), comm=comm)
        layer_p.connect_peers()
        y_peer = layer_p.forward(x, lg).clone()
        torch.cuda.synchronize()
        graph_p = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_p, stream=s):
            y_pg = layer_p.forward(x, lg)
        for _ in range(3):
            graph_p.replay()
        torch.cuda.synchronize()
        same = bool(torch.equal(y_peer, y_eager)) and bool(torch.equal(y_pg, y_eager))
        q.put((rank, F.device_error(), y_eager.float().cpu().numpy().tobytes(), y_g.float().cpu().numpy().tobytes(),
               y_one.float().cpu().numpy().tobytes(), same))
    finally:
        graph = graph_p = None
        if layer_p is not None:
            torch.cuda.synchronize()
            dist.barrier()
            layer_p.close_peers()
            dist.barrier()  # no rank frees a buffer another still maps
            layer_p.ops.free()
        if comm is not None:
            comm.destroy()
        dist.destroy_process_group()


def test_fixed_capacity_two_gpus_match_single_gpu():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_fixed, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, err, eager, graphed, one, peer_same in results:
        assert peer_same, f"rank {rank}: peer-store mode differs from the all-to-all form"
        a = np.frombuffer(eager, np.float32)
        g = np.frombuffer(graphed, np.float32)
        b = np.frombuffer(one, np.float32)
        assert err == 0
        assert np.array_equal(a, g), f"rank {rank}: graph replay differs from the eager call"
        assert np.all(np.isfinite(a)) and np.abs(b).max() > 0
        diff = np.abs(a - b)
        assert np.all(diff <= 2.0 ** -7 * np.abs(b) + 1e-4 * np.abs(b).max()), f"rank {rank}: {diff.max()}"
        assert np.mean(diff == 0) > 0.9
