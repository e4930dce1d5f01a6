"""The tensor-core NVFP4 GEMV (x as 8 NVFP4 digit planes, tcgen05
mxf4nvf4) against the oracle's f32 GEMV and f64 product.

Bar: relative Frobenius <= 1e-5 against the oracle's f32-accumulated GEMV
(the planes reproduce x to f32 round-off; the north star's matmul bar is
1e-3), and every element within the f64 inner-product bound of the
reference's own check (tests/common/check.rs:19-33) scaled by 4.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL = 1e-5


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


@pytest.fixture(scope="module")
def F(torch):
    import firepit_b200
    return firepit_b200


def _ws(torch, N, groups, k):
    n = int(N.lib.fpb_nvfp4_gemv_planes_workspace_bytes(groups, k))
    return torch.empty(n, dtype=torch.uint8, device="cuda")


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (1024, 2048), (384, 512), (128, 256), (8192, 2048)])
@pytest.mark.parametrize("tokens", [1, 3, 8, 16])
@pytest.mark.parametrize("x_f32", [False, True])
def test_planes_gemv_matches_oracle(F, torch, rows, cols, tokens, x_f32):
    N = F._native
    w = F.synth_normal((rows, cols), seed=rows + cols, stream_id=1, std=0.02)
    m = F.Nvfp4Matrix.quantize(w)
    h = m.to_host()
    x = O.synth_normal(tokens * cols, seed=tokens, stream=2).reshape(tokens, cols).astype(np.float32)
    x[0, 5] = 40.0  # an outlier: later planes resolve the rest of the row
    if not x_f32:
        x = O.bf16_to_f32(O.bf16_bits(x)).reshape(tokens, cols)
    xt = torch.from_numpy(x).cuda()
    if not x_f32:
        xt = xt.to(torch.bfloat16)
    y = torch.full((tokens, rows), float("nan"), device="cuda")
    ws = _ws(torch, N, 1, cols)
    N.call("fpb_nvfp4_gemv_planes", m.handle, 0, 0, xt.data_ptr(), N.FPB_F32 if x_f32 else N.FPB_BF16, tokens,
           y.data_ptr(), N.FPB_F32, ws.data_ptr(), ws.numel(), None)
    torch.cuda.synchronize()
    assert F.device_error() == 0
    yc = y.cpu().numpy()
    assert np.all(np.isfinite(yc))
    want = O.nvfp4_gemv_f32(h.packed, h.scales, h.row_scales, rows, cols, x)
    assert O.rel_frobenius(yc, want) <= REL
    e64, mag = O.nvfp4_gemv_f64(h.packed, h.scales, h.row_scales, rows, cols, x)
    assert O.inner_product_excess(yc, e64, mag, cols + 2) <= 4.0


def test_planes_gemv_row_range_and_bf16_out(F, torch):
    N = F._native
    rows, cols, tokens = 1024, 1024, 5
    m = F.Nvfp4Matrix.quantize(F.synth_normal((rows, cols), seed=9, stream_id=1, std=0.02))
    h = m.to_host()
    x = O.bf16_to_f32(O.bf16_bits(O.synth_normal(tokens * cols, seed=3, stream=2))).reshape(tokens, cols)
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y = torch.zeros(tokens, 384, dtype=torch.bfloat16, device="cuda")
    ws = _ws(torch, N, 1, cols)
    N.call("fpb_nvfp4_gemv_planes", m.handle, 256, 640, xt.data_ptr(), N.FPB_BF16, tokens, y.data_ptr(), N.FPB_BF16,
           ws.data_ptr(), ws.numel(), None)
    torch.cuda.synchronize()
    want = O.nvfp4_gemv_f32(h.packed, h.scales, h.row_scales, rows, cols, x)[:, 256:640]
    assert O.rel_frobenius(y.float().cpu().numpy(), want) <= 8e-3  # bf16 output


def test_planes_moe_gemv(F, torch):
    N = F._native
    experts, rpe, cols, T = 9, 1024, 2048, 8
    m = F.Nvfp4Matrix.quantize(F.synth_normal((experts * rpe, cols), seed=5, stream_id=1, std=0.02), rpe)
    h = m.to_host()
    routed = np.random.default_rng(1).integers(0, experts, size=(T, 3)).astype(np.int32)
    routed[:, 2] = 4
    distinct = np.unique(routed)
    cap = routed.size
    d = torch.full((cap,), -1, dtype=torch.int32, device="cuda")
    d[:distinct.size] = torch.from_numpy(distinct.astype(np.int32)).cuda()
    c = torch.tensor([distinct.size], dtype=torch.int32, device="cuda")
    for per_expert_x in (False, True):
        nx = cap if per_expert_x else 1
        x = O.bf16_to_f32(O.bf16_bits(O.synth_normal(nx * T * cols, seed=2, stream=7))).reshape(nx, T, cols)
        xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
        y = torch.full((cap, T, rpe), float("nan"), device="cuda")
        ws = _ws(torch, N, nx, cols)
        N.call("fpb_nvfp4_moe_gemv_planes", m.handle, rpe, d.data_ptr(), c.data_ptr(), cap, xt.data_ptr(),
               N.FPB_BF16, T * cols if per_expert_x else 0, T, y.data_ptr(), N.FPB_F32, ws.data_ptr(), ws.numel(),
               None)
        torch.cuda.synchronize()
        assert F.device_error() == 0
        yc = y.cpu().numpy()
        for u, e in enumerate(distinct):
            want = O.nvfp4_expert_gemv_f32(h.packed, h.scales, h.row_scales, cols, np.full(T, e, np.int32), rpe, 1,
                                           x[u if per_expert_x else 0])
            assert O.rel_frobenius(yc[u], want) <= REL, (per_expert_x, u)
        assert np.all(np.isnan(yc[distinct.size:]))  # groups past the count are not written


def test_planes_errors(F, torch):
    N = F._native
    m = F.Nvfp4Matrix.quantize(F.synth_normal((256, 288), seed=1, stream_id=1, std=0.02))
    x = torch.zeros(2, 288, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros(2, 256, device="cuda")
    ws = _ws(torch, N, 1, 288)
    call = N.lib.fpb_nvfp4_gemv_planes
    assert call(m.handle, 0, 0, x.data_ptr(), N.FPB_BF16, 2, y.data_ptr(), N.FPB_F32, ws.data_ptr(), ws.numel(),
                None) == N.FPB_ERR_UNSUPPORTED  # cols not a multiple of 256
    m2 = F.Nvfp4Matrix.quantize(F.synth_normal((256, 512), seed=1, stream_id=1, std=0.02))
    x2 = torch.zeros(17, 512, dtype=torch.bfloat16, device="cuda")
    y2 = torch.zeros(17, 256, device="cuda")
    ws2 = _ws(torch, N, 1, 512)
    assert call(m2.handle, 0, 0, x2.data_ptr(), N.FPB_BF16, 17, y2.data_ptr(), N.FPB_F32, ws2.data_ptr(), ws2.numel(),
                None) == N.FPB_ERR_SHAPE
    assert call(m2.handle, 0, 0, x2.data_ptr(), N.FPB_BF16, 2, y2.data_ptr(), N.FPB_F32, ws2.data_ptr(), 1024,
                None) == N.FPB_ERR_WORKSPACE
    assert call(m2.handle, 64, 0, x2.data_ptr(), N.FPB_BF16, 2, y2.data_ptr(), N.FPB_F32, ws2.data_ptr(),
                ws2.numel(), None) == N.FPB_ERR_UNSUPPORTED  # row_begin not a multiple of 128


def test_planes_moe_gemv_glu(F, torch):
    """The down projection with SwiGLU folded into the plane encoder equals
    the oracle's expert GEMV of silu(gate) * up computed in f32."""
    N = F._native
    experts, rows, inter, T = 7, 2048, 512, 8
    m = F.Nvfp4Matrix.quantize(F.synth_normal((experts * rows, inter), seed=8, stream_id=1, std=0.02), rows)
    h = m.to_host()
    distinct = np.array([0, 2, 5, 6], np.int32)
    cap = 6
    d = torch.full((cap,), -1, dtype=torch.int32, device="cuda")
    d[:4] = torch.from_numpy(distinct).cuda()
    c = torch.tensor([4], dtype=torch.int32, device="cuda")
    gu = (np.random.default_rng(4).standard_normal((cap, T, 2 * inter)) * 2).astype(np.float32)
    gut = torch.from_numpy(gu).cuda()
    y = torch.full((cap, T, rows), float("nan"), device="cuda")
    ws = _ws(torch, N, cap, inter)
    N.call("fpb_nvfp4_moe_gemv_planes_glu", m.handle, rows, d.data_ptr(), c.data_ptr(), cap, gut.data_ptr(),
           T * 2 * inter, T, y.data_ptr(), N.FPB_F32, ws.data_ptr(), ws.numel(), None)
    torch.cuda.synchronize()
    assert F.device_error() == 0
    yc = y.cpu().numpy()
    for u, e in enumerate(distinct):
        g, up = gu[u, :, :inter].astype(np.float64), gu[u, :, inter:].astype(np.float64)
        act = (g / (1.0 + np.exp(-g)) * up).astype(np.float32)
        want = O.nvfp4_expert_gemv_f32(h.packed, h.scales, h.row_scales, inter, np.full(T, e, np.int32), rows, 1, act)
        assert O.rel_frobenius(yc[u], want) <= REL
    assert np.all(np.isnan(yc[4:]))


@pytest.mark.parametrize("rows,cols,mats,batch", [(4096, 4096, 16, 1), (1024, 2048, 5, 8), (256, 512, 3, 16)])
def test_planes_batch_matches_single(F, torch, rows, cols, mats, batch):
    """A prepared batch (one launch over several matrices, each its own x)
    equals the oracle per member, including a row range that starts past 0,
    under a CUDA graph."""
    weights = [F.Nvfp4Matrix.quantize(F.synth_normal((rows, cols), seed=40 + i, stream_id=1, std=0.02))
               for i in range(mats)]
    hosts = [w.to_host() for w in weights]
    xs = [O.bf16_to_f32(O.bf16_bits(O.synth_normal(batch * cols, seed=i, stream=3))).reshape(batch, cols)
          for i in range(mats)]
    xt = [torch.from_numpy(x).cuda().to(torch.bfloat16) for x in xs]
    ys = [torch.full((batch, rows if i else rows - 128), float("nan"), device="cuda") for i in range(mats)]
    members = [(weights[i], xt[i], ys[i]) + ((range(128, rows),) if i == 0 else ()) for i in range(mats)]
    b = F.gemv_batch_planes(members, F.GemvTile(1, 4))
    g = F.Graph()
    with g:
        b.submit(g)
    g.replay()
    torch.cuda.synchronize()
    assert F.device_error() == 0
    for i in range(mats):
        want = O.nvfp4_gemv_f32(hosts[i].packed, hosts[i].scales, hosts[i].row_scales, rows, cols, xs[i])
        if i == 0:
            want = want[:, 128:]
        assert O.rel_frobenius(ys[i].cpu().numpy(), want) <= REL, i
    with pytest.raises(F.ShapeError):  # row range not starting at a multiple of 128
        F.gemv_batch_planes([(weights[0], xt[0], ys[0][:, :rows - 192], range(64, rows - 128))], F.GemvTile(1, 4))


@pytest.mark.parametrize("out_bf16", [True, False])
def test_planes_batch_peer_copies(F, torch, out_bf16):
    """fpb_nvfp4_gemv_batch_create_peers: each member's result goes to its
    copies (here three places in one local buffer, standing for this rank's
    slice in three ranks' gathered outputs), equal to the plain batch's y bit
    for bit, and the member's own y is left alone."""
    rows, cols, mats, batch = 512, 1024, 3, 2
    yd = torch.bfloat16 if out_bf16 else torch.float32
    weights = []
    for c in range(mats):
        w = F.synth_normal((rows, cols), seed=70 + c, stream_id=1, std=0.02)
        packed, scales, g = F.quantize_nvfp4(w)
        weights.append(F.Nvfp4Matrix.from_device(packed, scales, g, rows, cols))
    xs = [F.synth_normal((batch, cols), seed=80 + c, stream_id=0, dtype=torch.bfloat16) for c in range(mats)]
    ys = [torch.empty(batch, rows, dtype=yd, device="cuda") for _ in range(mats)]
    F.gemv_batch_planes([(weights[c], xs[c], ys[c]) for c in range(mats)], F.GemvTile(1, 4)).submit(F.Eager())
    ranks = 3
    gathered = torch.full((ranks, mats, batch, rows), -7.0, dtype=yd, device="cuda")
    own = [torch.full((batch, rows), -3.0, dtype=yd, device="cuda") for _ in range(mats)]
    peers = [[gathered[r, c].data_ptr() for r in range(ranks)] for c in range(mats)]
    F.gemv_batch_planes([(weights[c], xs[c], own[c]) for c in range(mats)], F.GemvTile(1, 4),
                        y_peers=peers).submit(F.Eager())
    torch.cuda.synchronize()
    for c in range(mats):
        for r in range(ranks):
            assert torch.equal(gathered[r, c], ys[c])
        assert bool((own[c] == -3.0).all())
    assert F.device_error() == 0
    with pytest.raises(Exception):
        F.gemv_batch_planes([(weights[0], xs[0], own[0])], F.GemvTile(1, 4), y_peers=[[gathered[0, 0].data_ptr()] * 9])
