"""The decode MoE over distinct experts: fpb_moe_decode_plan, fpb_nvfp4_moe_gemv
and fpb_moe_decode_combine_add_norm against numpy and the oracle.

The reference runs expert_gemv_weight_view once per (token, slot)
(gemv/mod.rs:137-206); here each distinct routed expert is read once for
every token of the batch.  Bars: the plan (distinct ids, count, map) exact;
every live (expert, token) output within relative Frobenius 1e-3 of the
oracle's f32-accumulated expert GEMV (the north star's matmul bar); the
mapped combine within 1e-5 (f32, a different summation order); and the whole
top-k -> plan -> GEMVs chain in one CUDA graph equal to the per-slot
results of fresh ids on every replay.
"""
import numpy as np
import pytest

from oracle import model_ops as R
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_FROB_TOL = 1e-3


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


@pytest.fixture(scope="module")
def F(torch):
    import firepit_b200
    return firepit_b200


def _plan(F, torch, ids_np, slots, experts):
    N = F._native
    T, width = ids_np.shape
    cap = T * slots
    ids = torch.from_numpy(ids_np.astype(np.int32)).cuda()
    distinct = torch.full((cap,), 12345, dtype=torch.int32, device="cuda")
    count = torch.full((1,), -5, dtype=torch.int32, device="cuda")
    mp = torch.full((T * slots,), 777, dtype=torch.int32, device="cuda")
    N.call("fpb_moe_decode_plan", ids.data_ptr(), T, width, slots, experts, distinct.data_ptr(), count.data_ptr(),
           cap, mp.data_ptr(), None)
    torch.cuda.synchronize()
    return distinct.cpu().numpy(), int(count.item()), mp.cpu().numpy()


@pytest.mark.parametrize("T,slots,width,experts", [(8, 11, 11, 513), (1, 11, 16, 513), (5, 3, 4, 40),
                                                   (16, 11, 11, 513), (3, 2, 2, 70000 // 2)])
def test_plan_matches_unique(F, torch, T, slots, width, experts):
    rng = np.random.default_rng(T * 100 + slots)
    ids = rng.integers(0, experts, size=(T, width)).astype(np.int32)
    ids[:, min(slots - 1, 1)] = ids[0, 0]  # a shared expert in every row
    distinct, count, mp = _plan(F, torch, ids, slots, experts)
    want = np.unique(ids[:, :slots])
    assert count == want.size
    assert np.array_equal(distinct[:count], want)
    assert np.all(distinct[count:] == -1)
    assert np.array_equal(distinct[mp].reshape(T, slots), ids[:, :slots])
    assert F.device_error() == 0


def test_plan_bad_id_is_recorded(F, torch):
    ids = np.array([[3, 9, 600], [3, 1, 2]], np.int32)  # 600 is outside 513 experts
    F.device_error()  # read and cleared
    distinct, count, mp = _plan(F, torch, ids, 3, 513)
    assert F.device_error() == 107
    assert count == 4 and np.array_equal(distinct[:4], [1, 2, 3, 9])
    assert mp[2] == -1 and np.array_equal(distinct[mp[[0, 1, 3, 4, 5]]], [3, 9, 3, 1, 2])


def test_plan_errors(F, torch):
    N = F._native
    ids = torch.zeros(2, 4, dtype=torch.int32, device="cuda")
    d = torch.zeros(8, dtype=torch.int32, device="cuda")
    c = torch.zeros(1, dtype=torch.int32, device="cuda")
    m = torch.zeros(8, dtype=torch.int32, device="cuda")
    assert N.lib.fpb_moe_decode_plan(ids.data_ptr(), 2, 4, 4, 16, d.data_ptr(), c.data_ptr(), 7, m.data_ptr(),
                                     None) == N.FPB_ERR_SHAPE  # cap below tokens x slots
    assert N.lib.fpb_moe_decode_plan(ids.data_ptr(), 2, 4, 5, 16, d.data_ptr(), c.data_ptr(), 8, m.data_ptr(),
                                     None) == N.FPB_ERR_SHAPE  # slots above width
    assert N.lib.fpb_moe_decode_plan(None, 2, 4, 4, 16, d.data_ptr(), c.data_ptr(), 8, m.data_ptr(),
                                     None) == N.FPB_ERR_INVALID_ARGUMENT


def _experts(F, experts, rpe, cols, seed):
    w = F.synth_normal((experts * rpe, cols), seed=seed, stream_id=1, std=0.02)
    m = F.Nvfp4Matrix.quantize(w, rpe)
    return m, m.to_host()


@pytest.mark.parametrize("rpe,cols,T,per_segment_x,x_f32", [
    (1024, 2048, 8, False, False),   # config-4 gate/up: streaming kernel, one x for all
    (2048, 512, 8, True, False),     # config-4 down: streaming, x per segment
    (1024, 2048, 3, True, True),     # f32 x (hi/lo)
    (1024, 2048, 12, False, False),  # more than 8 tokens: register kernel
    (96, 160, 4, True, False),       # K not a multiple of 128: register kernel
    (64, 5120, 2, False, False),     # K above 4096: register kernel over K slices (f32 y)
])
def test_moe_gemv_matches_oracle(F, torch, rpe, cols, T, per_segment_x, x_f32):
    N = F._native
    experts = 9
    m, h = _experts(F, experts, rpe, cols, seed=rpe + cols)
    routed = np.random.default_rng(rpe + T).integers(0, experts, size=(T, 3)).astype(np.int32)
    routed[:, 2] = 4  # one expert routed by every token, as the shared expert is
    distinct, count, _ = _plan(F, torch, routed, routed.shape[1], experts)
    cap = routed.size
    nx = cap if per_segment_x else 1
    x = O.synth_normal(nx * T * cols, seed=T, stream=3).reshape(nx, T, cols).astype(np.float32)
    if not x_f32:
        x = O.bf16_to_f32(O.bf16_bits(x)).reshape(nx, T, cols)
    xt = torch.from_numpy(x).cuda()
    if not x_f32:
        xt = xt.to(torch.bfloat16)
    y = torch.full((cap, T, rpe), float("nan"), device="cuda")
    d = torch.from_numpy(distinct).cuda()
    c = torch.tensor([count], dtype=torch.int32, device="cuda")
    N.call("fpb_nvfp4_moe_gemv", m.handle, rpe, d.data_ptr(), c.data_ptr(), cap, xt.data_ptr(),
           N.FPB_F32 if x_f32 else N.FPB_BF16, T * cols if per_segment_x else 0, T, y.data_ptr(), N.FPB_F32, None)
    torch.cuda.synchronize()
    assert F.device_error() == 0
    yc = y.cpu().numpy()
    for u in range(count):
        xu = x[u if per_segment_x else 0]
        want = O.nvfp4_expert_gemv_f32(h.packed, h.scales, h.row_scales, cols, np.full(T, distinct[u], np.int32),
                                       rpe, 1, xu)
        assert np.all(np.isfinite(yc[u])), u
        assert O.rel_frobenius(yc[u], want) <= REL_FROB_TOL, u


def test_moe_gemv_errors(F, torch):
    N = F._native
    m, _ = _experts(F, 2, 64, 256, seed=1)
    d = torch.zeros(4, dtype=torch.int32, device="cuda")
    c = torch.ones(1, dtype=torch.int32, device="cuda")
    x = torch.zeros(4, 256, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros(4, 4, 64, device="cuda")
    call = N.lib.fpb_nvfp4_moe_gemv
    assert call(m.handle, 64, d.data_ptr(), c.data_ptr(), 4, x.data_ptr(), N.FPB_BF16, 0, 17, y.data_ptr(),
                N.FPB_F32, None) == N.FPB_ERR_SHAPE  # tokens
    assert call(m.handle, 48, d.data_ptr(), c.data_ptr(), 4, x.data_ptr(), N.FPB_BF16, 0, 1, y.data_ptr(),
                N.FPB_F32, None) == N.FPB_ERR_SHAPE  # rows not a multiple of rows_per_expert
    assert call(m.handle, 64, d.data_ptr(), c.data_ptr(), 4, x.data_ptr(), N.FPB_BF16, 3, 1, y.data_ptr(),
                N.FPB_F32, None) == N.FPB_ERR_INVALID_ARGUMENT  # x_stride breaks 16-byte alignment
    assert call(m.handle, 64, None, c.data_ptr(), 4, x.data_ptr(), N.FPB_BF16, 0, 1, y.data_ptr(), N.FPB_F32,
                None) == N.FPB_ERR_INVALID_ARGUMENT


def test_mapped_combine(F, torch):
    N = F._native
    T, slots, h, experts = 8, 11, 512, 40
    rng = np.random.default_rng(5)
    ids = rng.integers(0, experts, size=(T, slots)).astype(np.int32)
    distinct, count, mp = _plan(F, torch, ids, slots, experts)
    cap = T * slots
    routed = torch.from_numpy(rng.standard_normal((cap, T, h)).astype(np.float32)).cuda()
    wts = torch.rand(T, slots, device="cuda")
    resid = torch.from_numpy(rng.standard_normal((T, h)).astype(np.float32)).cuda()
    gamma = torch.from_numpy((rng.standard_normal(h) * 0.1 + 1).astype(np.float32)).cuda()
    out = torch.empty(T, h, device="cuda")
    normed = torch.empty(T, h, device="cuda")
    mt = torch.from_numpy(mp).cuda()
    N.call("fpb_moe_decode_combine_add_norm", routed.data_ptr(), mt.data_ptr(), wts.data_ptr(), slots, slots,
           resid.data_ptr(), gamma.data_ptr(), T, h, 1e-6, out.data_ptr(), normed.data_ptr(), N.FPB_F32, None)
    torch.cuda.synchronize()
    r = routed.cpu().numpy()
    w = wts.cpu().numpy()
    ref = resid.cpu().numpy().astype(np.float64)
    for t in range(T):
        for s in range(slots):
            ref[t] += w[t, s] * r[mp[t * slots + s], t]
    assert np.allclose(out.cpu().numpy(), ref, rtol=1e-5, atol=1e-5)
    assert np.allclose(normed.cpu().numpy(), R.rms_norm(out.cpu().numpy(), gamma.cpu().numpy(), 1e-6), rtol=1e-5,
                       atol=1e-6)
    bad = N.lib.fpb_moe_decode_combine_add_norm(routed.data_ptr(), None, wts.data_ptr(), slots, slots,
                                                resid.data_ptr(), gamma.data_ptr(), T, h, 1e-6, out.data_ptr(),
                                                normed.data_ptr(), N.FPB_F32, None)
    assert bad == N.FPB_ERR_INVALID_ARGUMENT


def test_topk_plan_moe_gemv_in_one_graph(F, torch):
    """Router top-k, the plan and both GEMVs on one stream in one CUDA graph:
    each replay first overwrites the ids with a stale expert; the outputs must
    be those of the fresh routing (programmatic dependent launch must not let
    a kernel read its predecessor's outputs early)."""
    N = F._native
    experts, rpe, cols, T, k = 32, 256, 1024, 8, 4
    m, h = _experts(F, experts, rpe, cols, seed=77)
    x = F.synth_normal((T, cols), seed=0, stream_id=5, dtype=torch.bfloat16)
    xf = x.float().cpu().numpy()
    logits = torch.empty(T, experts, device="cuda")
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    wts = torch.empty(T, k, device="cuda")
    cap = T * k
    distinct = torch.empty(cap, dtype=torch.int32, device="cuda")
    count = torch.empty(1, dtype=torch.int32, device="cuda")
    mp = torch.empty(cap, dtype=torch.int32, device="cuda")
    y = torch.empty(cap, T, rpe, device="cuda")

    def ops(stream):
        ids.fill_(3)
        N.call("fpb_moe_topk", logits.data_ptr(), experts, None, T, experts, k, k, ids.data_ptr(), wts.data_ptr(),
               stream)
        N.call("fpb_moe_decode_plan", ids.data_ptr(), T, k, k, experts, distinct.data_ptr(), count.data_ptr(), cap,
               mp.data_ptr(), stream)
        N.call("fpb_nvfp4_moe_gemv", m.handle, rpe, distinct.data_ptr(), count.data_ptr(), cap, x.data_ptr(),
               N.FPB_BF16, 0, T, y.data_ptr(), N.FPB_F32, stream)

    rng = np.random.default_rng(9)
    logits.copy_(torch.from_numpy(rng.standard_normal((T, experts)).astype(np.float32)))
    ops(torch.cuda.current_stream().cuda_stream)  # every code path initialised outside capture
    torch.cuda.synchronize()
    g = F.Graph()
    with g:
        g.run("chain", ops)
    for r in range(4):
        lg = rng.standard_normal((T, experts)).astype(np.float32)
        logits.copy_(torch.from_numpy(lg))
        g.replay()
        torch.cuda.synchronize()
        want_ids, _ = O.moe_topk(lg, k, k)
        got_ids = ids.cpu().numpy()
        assert np.array_equal(got_ids, want_ids)
        d, c, mpc, yc = distinct.cpu().numpy(), int(count.item()), mp.cpu().numpy(), y.cpu().numpy()
        assert np.array_equal(d[:c], np.unique(want_ids))
        for t in range(T):
            for s_ in range(k):
                u = mpc[t * k + s_]
                want = O.nvfp4_expert_gemv_f32(h.packed, h.scales, h.row_scales, cols,
                                               np.array([want_ids[t, s_]], np.int32), rpe, 0, xf[t:t + 1])
                assert O.rel_frobenius(yc[u, t:t + 1], want) <= REL_FROB_TOL
    assert F.device_error() == 0


@pytest.mark.parametrize("T,experts,k,gate", [(8, 512, 10, True), (1, 512, 10, True), (32, 128, 4, False),
                                              (5, 40, 8, True), (16, 512, 10, False)])
def test_fused_route_equals_topk_then_plan(F, torch, T, experts, k, gate):
    """fpb_moe_decode_route (gate logit as a column of the router output) ==
    fpb_moe_topk (gate as its own array) followed by fpb_moe_decode_plan."""
    N = F._native
    ld = (experts + 1 + 3) // 4 * 4
    rng = np.random.default_rng(T * 7 + experts)
    lg = rng.standard_normal((T, ld)).astype(np.float32)
    lg[0, 3] = lg[0, 5]  # a tie: the lower id first
    logits = torch.from_numpy(lg).cuda()
    slots = k + (1 if gate else 0)
    width = slots
    cap = T * slots
    g = torch.from_numpy(np.ascontiguousarray(lg[:, experts])).cuda()
    ids_a = torch.full((T, width), -7, dtype=torch.int32, device="cuda")
    w_a = torch.zeros(T, width, device="cuda")
    N.call("fpb_moe_topk", logits.data_ptr(), ld, g.data_ptr() if gate else None, T, experts, k, width,
           ids_a.data_ptr(), w_a.data_ptr(), None)
    d_a = torch.zeros(cap, dtype=torch.int32, device="cuda")
    c_a = torch.zeros(1, dtype=torch.int32, device="cuda")
    m_a = torch.zeros(cap, dtype=torch.int32, device="cuda")
    N.call("fpb_moe_decode_plan", ids_a.data_ptr(), T, width, slots, experts + (1 if gate else 0), d_a.data_ptr(),
           c_a.data_ptr(), cap, m_a.data_ptr(), None)
    ids_b = torch.full((T, width), -7, dtype=torch.int32, device="cuda")
    w_b = torch.zeros(T, width, device="cuda")
    d_b = torch.full((cap,), 99, dtype=torch.int32, device="cuda")
    c_b = torch.zeros(1, dtype=torch.int32, device="cuda")
    m_b = torch.full((cap,), 99, dtype=torch.int32, device="cuda")
    N.call("fpb_moe_decode_route", logits.data_ptr(), ld, experts if gate else -1, T, experts, k, width,
           ids_b.data_ptr(), w_b.data_ptr(), d_b.data_ptr(), c_b.data_ptr(), cap, m_b.data_ptr(), None)
    torch.cuda.synchronize()
    assert torch.equal(ids_a, ids_b)
    assert torch.equal(w_a, w_b)
    assert int(c_a.item()) == int(c_b.item())
    assert torch.equal(d_a, d_b) and torch.equal(m_a, m_b)
    want_ids, want_w = O.moe_topk(lg[:, :experts], k, width, lg[:, experts] if gate else None)
    assert np.array_equal(ids_b.cpu().numpy(), want_ids)
    assert np.allclose(w_b.cpu().numpy(), want_w, rtol=2e-6, atol=1e-7)
    assert F.device_error() == 0
    bad = N.lib.fpb_moe_decode_route(logits.data_ptr(), ld, -1, 33, experts, k, k, ids_b.data_ptr(), w_b.data_ptr(),
                                     d_b.data_ptr(), c_b.data_ptr(), 33 * k, m_b.data_ptr(), None)
    assert bad == N.FPB_ERR_SHAPE
