"""N-split GEMV whose all-gather is done by the GEMV's epilogue over NVLink
(peer copies into every rank's gathered buffer, CUDA IPC), ordered by the
peer-memory barrier (fpb_peer_barrier), on 2 GPUs (skipped with fewer).  Each
rank's gathered output must equal the NCCL all-gather of the same slices bit
for bit, eagerly and over graph replays."""
import os
import socket
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
ROWS, COLS, MATS = 1024, 2048, 5


def _rank(rank, world, port, q):
    sys.path[:0] = [ROOT, HERE]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import firepit_b200 as F
    from firepit_b200.comm import Comm, PeerBarrier, PeerBuffer
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    comm = buf = graph = barrier = None
    try:
        comm = Comm.from_torch()
        per = ROWS // world
        slices = []
        for c in range(MATS):
            w = F.synth_normal((ROWS, COLS), seed=0, stream_id=1 + c, std=0.02, device=dev)
            p, s, g = F.quantize_nvfp4(w)
            r0 = rank * per
            slices.append(F.Nvfp4Matrix.from_device(p[r0:r0 + per].contiguous(), s[r0:r0 + per].contiguous(),
                                                    g[r0:r0 + per].contiguous(), per, COLS))
        x = F.synth_normal((MATS, COLS), seed=0, stream_id=0, dtype=torch.bfloat16, device=dev)
        y = torch.empty(MATS, per, dtype=torch.bfloat16, device=dev)
        # reference: the plain batch, then the library's NCCL all-gather
        F.gemv_batch_planes([(slices[c], x[c:c + 1], y[c:c + 1]) for c in range(MATS)],
                            F.GemvTile(1, 4)).submit(F.Eager())
        ref = torch.empty(world, MATS, per, dtype=torch.bfloat16, device=dev)
        comm.all_gather(y, ref)
        # fused: this rank's slice stored into every rank's gathered buffer [world, MATS, per]
        buf = PeerBuffer(world * MATS * per * 2)
        gathered = buf.local.view(torch.bfloat16).view(world, MATS, per)
        gathered.fill_(0)
        torch.cuda.synchronize()
        dist.barrier()
        peers = [[buf.ptrs[r] + ((rank * MATS + c) * per) * 2 for r in range(world)] for c in range(MATS)]
        bat = F.gemv_batch_planes([(slices[c], x[c:c + 1], y[c:c + 1]) for c in range(MATS)], F.GemvTile(1, 4),
                                  y_peers=peers)
        barrier = PeerBarrier()
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):  # eager once, then the same as a CUDA graph
            bat.submit(F.Eager())
            barrier()
        torch.cuda.synchronize()
        eager_ok = bool(torch.equal(gathered, ref))
        gathered.fill_(0)
        torch.cuda.synchronize()
        dist.barrier()
        graph = F.Graph()
        with graph:
            bat.submit(graph)
            barrier()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        graph_ok = bool(torch.equal(gathered, ref))
        # the barrier's all-reduce MAX: ranks hold 1 and 2, both end with 2
        v = torch.tensor([rank + 1], dtype=torch.int32, device=dev)
        barrier.all_reduce_max(v)
        torch.cuda.synchronize()
        q.put((rank, F.device_error(), eager_ok, graph_ok and v.item() == world))
    finally:
        graph = None
        if barrier is not None:
            barrier.close()
        if buf is not None:
            buf.close()
        if comm is not None:
            comm.destroy()
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_epilogue_all_gather_matches_nccl():
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
    for rank, err, eager_ok, graph_ok in results:
        assert err == 0
        assert eager_ok, f"rank {rank}: eager peer copies differ from the NCCL all-gather"
        assert graph_ok, f"rank {rank}: graph replay differs"
