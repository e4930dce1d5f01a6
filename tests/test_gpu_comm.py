"""Collectives through the C ABI (fpb_comm_*): the NCCL exchange steps of the
N-split and expert-parallel paths.  A one-rank communicator runs on any GPU
box; the two-rank test (two processes, one GPU each) needs two GPUs."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


def test_single_rank_collectives(torch):
    from firepit_b200.comm import Comm
    c = Comm(Comm.unique_id(), 1, 0, torch.cuda.current_device())
    x = torch.randn(3, 1000, device="cuda").to(torch.bfloat16)
    out = torch.empty(1, 3, 1000, dtype=torch.bfloat16, device="cuda")
    c.all_gather(x, out)
    a = torch.tensor([0x3f800000, 0x40000000], dtype=torch.int32, device="cuda")
    c.all_reduce_max_bits(a)
    recv = torch.empty_like(x)
    c.all_to_all(x, [3], recv, [3])
    s = torch.arange(10, dtype=torch.float32, device="cuda")
    c.all_reduce_sum(s)
    torch.cuda.synchronize()
    c.status()
    assert torch.equal(out[0], x) and torch.equal(recv, x)
    assert a.tolist() == [0x3f800000, 0x40000000]
    assert torch.equal(s, torch.arange(10, dtype=torch.float32, device="cuda"))
    c.destroy()


def _two_rank_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        from firepit_b200.comm import Comm
        c = Comm.from_torch()
        x = torch.full((4, 8), float(rank + 1), device="cuda")
        out = torch.empty(world, 4, 8, device="cuda")
        c.all_gather(x, out)
        # rank r sends r + 1 rows to every peer p, each row filled with 10 r + p
        send = torch.cat([torch.full((rank + 1, 8), 10.0 * rank + p, device="cuda") for p in range(world)])
        recv_counts = [p + 1 for p in range(world)]
        recv = torch.empty(sum(recv_counts), 8, device="cuda")
        c.all_to_all(send, [rank + 1] * world, recv, recv_counts)
        m = torch.tensor([0x3f800000 + rank], dtype=torch.int32, device="cuda")
        c.all_reduce_max_bits(m)
        torch.cuda.synchronize()
        ok = all(torch.all(out[p] == p + 1).item() for p in range(world))
        off = 0
        for p in range(world):
            ok = ok and torch.all(recv[off:off + p + 1] == 10.0 * p + rank).item()
            off += p + 1
        ok = ok and m.item() == 0x3f800000 + world - 1
        c.destroy()
        dist.destroy_process_group()
        q.put((rank, bool(ok), ""))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, False, repr(e)))


def test_two_rank_collectives(torch):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_two_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res
