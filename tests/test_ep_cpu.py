"""Expert-parallel MoE dispatch / combine on two gloo ranks (CPU).

firepit_b200.ep.ep_moe_forward runs with the oracle's CPU ops: experts split
over two ranks, each rank routing its own tokens through all-to-all.  Every
rank's output must equal the single-rank layer over all experts bit for bit
(the expert MLP depends only on a row and its expert)."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

E, K, H, I, T = 8, 3, 64, 32, 37


def _weights():
    sys.path[:0] = [ROOT, HERE]
    from oracle import oracle as O
    w1 = O.synth_normal(E * 2 * I * H, seed=1, stream=1, std=0.05).reshape(E * 2 * I, H)
    w2 = O.synth_normal(E * H * I, seed=2, stream=1, std=0.05).reshape(E * H, I)
    return w1.astype(np.float32), w2.astype(np.float32)


def _rank(rank, world, port, out_q):
    sys.path[:0] = [ROOT, HERE]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist

    from ep_host_ops import HostOps
    from firepit_b200.ep import ep_moe_forward
    from oracle import oracle as O
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        w1, w2 = _weights()
        per = E // world
        x = torch.from_numpy(O.synth_normal(T * H, seed=10 + rank, stream=3).reshape(T, H).astype(np.float32))
        logits = torch.from_numpy(O.synth_normal(T * E, seed=20 + rank, stream=4).reshape(T, E).astype(np.float32))
        local1 = w1[rank * per * 2 * I:(rank + 1) * per * 2 * I]
        local2 = w2[rank * per * H:(rank + 1) * per * H]
        ops = HostOps()
        y_ep = ep_moe_forward(ops, x, logits, K, E, local1, local2)
        y_one = ep_moe_forward(ops, x, logits, K, E, w1, w2, world=1)
        out_q.put((rank, y_ep.numpy().tobytes(), y_one.numpy().tobytes()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_expert_parallel_matches_single_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert len(results) == 2
    for _, ep, one in results:
        a = np.frombuffer(ep, np.float32)
        b = np.frombuffer(one, np.float32)
        assert np.all(np.isfinite(a)) and np.abs(b).max() > 0
        assert np.array_equal(a, b)


def _rank_fixed(rank, world, port, skew, out_q):
    sys.path[:0] = [ROOT, HERE]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist

    from ep_host_ops import HostEpOps, HostOps
    from firepit_b200.ep import EpMoeLayer, ep_moe_forward
    from oracle import oracle as O
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        w1, w2 = _weights()
        per = E // world
        x = torch.from_numpy(O.synth_normal(T * H, seed=10 + rank, stream=3).reshape(T, H).astype(np.float32))
        lg = O.synth_normal(T * E, seed=20 + rank, stream=4).reshape(T, E).astype(np.float32)
        if skew:  # every route on rank 0's experts: rank 1 receives only empty records
            lg[:, E // 2:] -= 100.0
        logits = torch.from_numpy(lg)
        ops = HostEpOps(T, H, I, E, K, world, w1[rank * per * 2 * I:(rank + 1) * per * 2 * I],
                        w2[rank * per * H:(rank + 1) * per * H])
        y_ep = EpMoeLayer(ops).forward(x, logits)
        y_one = ep_moe_forward(HostOps(), x, logits, K, E, w1, w2, world=1)
        out_q.put((rank, y_ep.numpy().tobytes(), y_one.numpy().tobytes()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("skew", [False, True])
def test_fixed_capacity_matches_single_rank(skew):
    """The fixed-capacity layer's records, empty marks, partial sums and
    rank-order final sum give the single-rank result up to the regrouping of
    the f32 sum over a token's routes."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_fixed, args=(r, 2, port, skew, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, ep, one in results:
        a = np.frombuffer(ep, np.float32)
        b = np.frombuffer(one, np.float32)
        assert np.all(np.isfinite(a)) and np.abs(b).max() > 0
        assert np.allclose(a, b, rtol=1e-5, atol=1e-6 * np.abs(b).max())
