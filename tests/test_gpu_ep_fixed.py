"""Fixed-capacity expert parallel (firepit_b200.ep.EpMoeLayer) on one GPU.

Two ranks are emulated on one GPU: each rank's DeviceEpOps holds its half of
the experts, and the test itself moves the equal-size chunks between them
(what the all-to-alls do) and takes the amax maxima (what the all-reduces
do).  No kernel waits on another rank, so the emulation runs the same
kernels as two GPUs would.  Each rank's output must match the single-GPU
layer over both ranks' tokens with all experts: the NVFP4 encodings are the
same bit for bit, and only the grouping of the f32 sum over a token's routes
(rank by rank) differs before the one bf16 rounding, so almost every element
is equal and the rest differ by at most one bf16 rounding step.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

E, K, H, I, T = 16, 4, 256, 128, 300


def _setup(skew: bool):
    import torch

    import firepit_b200 as F
    dev = torch.device("cuda", 0)
    w1 = F.synth_normal((E * 2 * I, H), seed=1, stream_id=1, std=0.02, device=dev)
    w2 = F.synth_normal((E * H, I), seed=2, stream_id=1, std=0.02, device=dev)
    p1, s1, g1 = F.quantize_nvfp4(w1, 2 * I)
    p2, s2, g2 = F.quantize_nvfp4(w2, H)
    A1 = F.Nvfp4Matrix.from_device(p1, s1, g1, E * 2 * I, H)
    A2 = F.Nvfp4Matrix.from_device(p2, s2, g2, E * H, I)
    halves = []
    per = E // 2
    for r in range(2):
        r1 = slice(r * per * 2 * I, (r + 1) * per * 2 * I)
        r2 = slice(r * per * H, (r + 1) * per * H)
        L1 = F.Nvfp4Matrix.from_device(p1[r1].contiguous(), s1[r1].contiguous(), g1[r1].contiguous(), per * 2 * I, H)
        L2 = F.Nvfp4Matrix.from_device(p2[r2].contiguous(), s2[r2].contiguous(), g2[r2].contiguous(), per * H, I)
        L1.prepare_glu(I)
        halves.append((L1, L2))
    x = F.synth_normal((2 * T, H), seed=0, stream_id=0, dtype=torch.bfloat16, device=dev)
    lg = F.synth_normal((2 * T, E), seed=0, stream_id=7, device=dev)
    if skew:  # every route on rank 0's experts: rank 1's chunks are all empty
        lg[:, E // 2:] -= 100.0
    return dev, A1, A2, halves, x, lg


def _single_gpu(dev, A1, A2, x, lg):
    from firepit_b200.ep import DeviceOps, ep_moe_forward
    return ep_moe_forward(DeviceOps(dev), x, lg, K, E, A1, A2, world=1)


def _emulated(dev, halves, x, lg):
    import torch

    from firepit_b200.ep import DeviceEpOps
    ops = [DeviceEpOps(dev, T, H, I, E, K, 2, *halves[r]) for r in range(2)]
    xs = [x[r * T:(r + 1) * T].contiguous() for r in range(2)]
    ls = [lg[r * T:(r + 1) * T].contiguous() for r in range(2)]
    routes = [o.route(l) for o, l in zip(ops, ls)]
    amax = [o.amax(xr) for o, xr in zip(ops, xs)]
    m = torch.maximum(amax[0], amax[1])
    for a in amax:
        a.copy_(m)
    sends = [o.dispatch(xr, ids, w, a) for o, xr, (ids, w), a in zip(ops, xs, routes, amax)]
    for r in range(2):
        for s in range(2):
            ops[r].recv.view(2, -1)[s].copy_(ops[s].send.view(2, -1)[r])
    ah = [o.experts_gate_up(o.recv) for o in ops]
    m = torch.maximum(ah[0], ah[1])
    for a in ah:
        a.copy_(m)
    for o in ops:
        o.experts_down()
    for r in range(2):
        for s in range(2):
            ops[r].ret_recv.view(2, -1)[s].copy_(ops[s].ret_send.view(2, -1)[r])
    outs = [o.finish(o.ret_recv, pos).clone() for o, (_, pos) in zip(ops, sends)]
    return ops, routes, [p for _, p in sends], outs


def _close(a, b):
    """Equal up to the regrouped f32 sum before one bf16 rounding."""
    a = a.float().cpu().numpy()
    b = b.float().cpu().numpy()
    assert np.all(np.isfinite(a)) and np.abs(b).max() > 0
    diff = np.abs(a - b)
    assert np.all(diff <= 2.0 ** -7 * np.abs(b) + 1e-4 * np.abs(b).max()), diff.max()
    assert np.mean(diff == 0) > 0.9


@pytest.mark.parametrize("skew", [False, True])
def test_emulated_two_ranks_match_single_gpu(skew):
    import torch

    import firepit_b200 as F
    dev, A1, A2, halves, x, lg = _setup(skew)
    y_one = _single_gpu(dev, A1, A2, x, lg)
    ops, routes, positions, outs = _emulated(dev, halves, x, lg)
    torch.cuda.synchronize()
    assert F.device_error() == 0
    per = E // 2
    for r in range(2):
        ids = routes[r][0][:, :K].cpu().numpy()
        pos = positions[r].cpu().numpy()
        table = pos[:T * 2].reshape(T, 2)
        for d in range(2):
            hit = np.any(ids // per == d, axis=1)
            assert pos[T * 2 + d] == hit.sum()
            # chunk d holds the routed tokens in token order, then nothing
            assert np.array_equal(table[hit, d], d * T + np.arange(hit.sum()))
            assert np.all(table[~hit, d] == -1)
        _close(outs[r], y_one[r * T:(r + 1) * T])
    if skew:
        for r in range(2):
            assert positions[r][T * 2 + 1].item() == 0


def test_one_rank_layer_matches_single_gpu():
    import torch

    import firepit_b200 as F
    from firepit_b200.ep import DeviceEpOps, EpMoeLayer
    dev, A1, A2, _, x, lg = _setup(False)
    A1.prepare_glu(I)
    y_one = _single_gpu(dev, A1, A2, x, lg)
    layer = EpMoeLayer(DeviceEpOps(dev, 2 * T, H, I, E, K, 1, A1, A2))
    y = layer.forward(x, lg)
    torch.cuda.synchronize()
    assert F.device_error() == 0
    # one rank: one partial per token, so the sum's grouping is the single-GPU one
    assert torch.equal(y.float(), y_one.float())


def test_dispatch_errors():
    import torch

    import firepit_b200 as F
    from firepit_b200 import _native as N
    dev = torch.device("cuda", 0)
    x = torch.zeros(4, 96, dtype=torch.bfloat16, device=dev)  # 96 % 64 != 0
    ids = torch.zeros(4, 4, dtype=torch.int32, device=dev)
    w = torch.zeros(4, 4, device=dev)
    amax = torch.zeros(1, device=dev)
    rec = torch.empty(2 * 4 * 256, dtype=torch.uint8, device=dev)
    pos = torch.empty(4 * 2 + 2, dtype=torch.int32, device=dev)
    g = torch.empty(1, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    st = N.lib.fpb_ep_dispatch(x.data_ptr(), N.FPB_BF16, 4, 96, ids.data_ptr(), w.data_ptr(), 4, 4, 16, 2,
                               amax.data_ptr(), rec.data_ptr(), pos.data_ptr(), g.data_ptr(), s)
    assert st == N.FPB_ERR_SHAPE
    st = N.lib.fpb_ep_dispatch(x.data_ptr(), N.FPB_BF16, 4, 64, ids.data_ptr(), w.data_ptr(), 4, 4, 15, 2,
                               amax.data_ptr(), rec.data_ptr(), pos.data_ptr(), g.data_ptr(), s)
    assert st == N.FPB_ERR_SHAPE  # experts not divisible by ranks
    assert F.device_error() == 0


def _emulated_peer(dev, halves, x, lg):
    """Peer mode on one GPU: each rank's chunk tables point straight into the
    other rank's receive buffers (what fpb_ipc_open gives across processes),
    so dispatch and the partial combine store there and nothing is copied."""
    import torch

    from firepit_b200.ep import DeviceEpOps
    ops = [DeviceEpOps(dev, T, H, I, E, K, 2, *halves[r]) for r in range(2)]
    for r in range(2):
        ops[r].connect([ops[d].recv.data_ptr() + r * T * ops[d].rec for d in range(2)],
                       [ops[s].ret_recv.data_ptr() + r * T * H * 4 for s in range(2)], r)
    xs = [x[r * T:(r + 1) * T].contiguous() for r in range(2)]
    ls = [lg[r * T:(r + 1) * T].contiguous() for r in range(2)]
    routes = [o.route(l) for o, l in zip(ops, ls)]
    amax = [o.amax(xr) for o, xr in zip(ops, xs)]
    m = torch.maximum(amax[0], amax[1])
    for a in amax:
        a.copy_(m)
    pos = [o.dispatch(xr, ids, w, a)[1] for o, xr, (ids, w), a in zip(ops, xs, routes, amax)]
    ah = [o.experts_gate_up(o.recv) for o in ops]
    m = torch.maximum(ah[0], ah[1])
    for a in ah:
        a.copy_(m)
    for o in ops:
        o.experts_down()
    return [o.finish(o.ret_recv, p).clone() for o, p in zip(ops, pos)]


@pytest.mark.parametrize("skew", [False, True])
def test_emulated_peer_stores_match_chunk_exchange(skew):
    import torch

    import firepit_b200 as F
    dev, A1, A2, halves, x, lg = _setup(skew)
    y_one = _single_gpu(dev, A1, A2, x, lg)
    _, _, _, outs = _emulated(dev, halves, x, lg)
    peer = _emulated_peer(dev, halves, x, lg)
    torch.cuda.synchronize()
    assert F.device_error() == 0
    for r in range(2):
        assert torch.equal(peer[r].float(), outs[r].float())  # the same sums, only the stores' addresses differ
        _close(peer[r], y_one[r * T:(r + 1) * T])


@pytest.mark.parametrize("tokens", [1, 10240, 10300])
def test_dispatch_plan_sizes(tokens):
    """The plan with every mask staged in shared memory (<= 10240 tokens) and
    computed chunk by chunk (more): positions and counts against numpy, and
    the records' routes."""
    import torch

    import firepit_b200 as F
    from firepit_b200 import _native as N
    dev = torch.device("cuda", 0)
    n, k, width, experts, cols = 4, 3, 4, 32, 64
    g = torch.Generator().manual_seed(tokens)
    ids = torch.stack([torch.randperm(experts, generator=g)[:width] for _ in range(tokens)]).to(torch.int32)
    w = torch.rand(tokens, width, generator=g)
    x = torch.randn(tokens, cols, generator=g).to(torch.bfloat16)
    rec = int(N.lib.fpb_ep_record_bytes(cols, width))
    records = torch.empty(n * tokens * rec, dtype=torch.uint8, device=dev)
    pos = torch.empty(tokens * n + n, dtype=torch.int32, device=dev)
    amax = torch.tensor([x.float().abs().max().item()], device=dev)
    glob = torch.empty(1, device=dev)
    idd, wd, xd = ids.to(dev), w.to(dev), x.to(dev)
    N.call("fpb_ep_dispatch", xd.data_ptr(), N.FPB_BF16, tokens, cols, idd.data_ptr(), wd.data_ptr(), width, k,
           experts, n, amax.data_ptr(), records.data_ptr(), pos.data_ptr(), glob.data_ptr(),
           torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert F.device_error() == 0
    p = pos.cpu().numpy()
    owner = ids[:, :k].numpy() // (experts // n)
    r = records.cpu().numpy().reshape(n * tokens, rec)
    ids_at = (cols // 2 + 15) // 16 * 16 + (cols // 16 + 15) // 16 * 16  # codes, factors, then the ids
    for d in range(n):
        hit = np.any(owner == d, axis=1)
        assert p[tokens * n + d] == hit.sum()
        col = p[:tokens * n].reshape(tokens, n)[:, d]
        assert np.array_equal(col[hit], d * tokens + np.arange(hit.sum()))
        assert np.all(col[~hit] == -1)
        got = np.ascontiguousarray(r[col[hit]][:, ids_at:ids_at + 4 * width]).view(np.int32)
        want = np.where(owner[hit] == d, ids[hit][:, :k].numpy() % (experts // n), -1)
        assert np.array_equal(got[:, :k], want) and np.all(got[:, k:] == -1)
        empty = np.ascontiguousarray(r[d * tokens + hit.sum():(d + 1) * tokens][:, ids_at:ids_at + 4 * width]).view(np.int32)
        assert np.all(empty == -1)
