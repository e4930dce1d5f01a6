"""The decode-step kernels of the hybrid decoder against
the oracle's restatement of firepit-kernels (oracle/model_ops.py).

Bars: embedding, argmax, cache layout: exact; RMSNorm, RoPE, conv, gated
norm: relative 1e-5 (f32 arithmetic in a different order, hardware exp and
sincos); attention and the delta rule: relative Frobenius 1e-5 against f64.
"""
import math

import numpy as np
import pytest

from oracle import model_ops as R
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


@pytest.fixture(scope="module")
def F(torch):
    import firepit_b200
    return firepit_b200


def _rand(torch, *shape, seed=0, scale=1.0):
    g = np.random.default_rng(seed)
    return torch.from_numpy((g.standard_normal(shape) * scale).astype(np.float32)).cuda()


def test_embedding_and_norms(F, torch):
    N = F._native
    vocab, h, rows = 1000, 512, 6
    table = _rand(torch, vocab, h, seed=1).to(torch.bfloat16)
    ids = torch.tensor([3, 999, 0, 500, 3, 42], dtype=torch.int32, device="cuda")
    out = torch.empty(rows, h, device="cuda")
    N.call("fpb_embedding", table.data_ptr(), vocab, h, ids.data_ptr(), rows, out.data_ptr(), None)
    assert torch.equal(out, table.float()[ids.long()])
    gamma = _rand(torch, h, seed=2, scale=0.1) + 1.0
    delta = _rand(torch, rows, h, seed=3)
    s = torch.empty(rows, h, device="cuda")
    nb = torch.empty(rows, h, dtype=torch.bfloat16, device="cuda")
    nf = torch.empty(rows, h, device="cuda")
    N.call("fpb_rms_norm", out.data_ptr(), N.FPB_F32, h, delta.data_ptr(), s.data_ptr(), rows, h, gamma.data_ptr(),
           1e-6, nf.data_ptr(), N.FPB_F32, h, None)
    N.call("fpb_rms_norm", out.data_ptr(), N.FPB_F32, h, None, None, rows, h, gamma.data_ptr(), 1e-6, nb.data_ptr(),
           N.FPB_BF16, h, None)
    torch.cuda.synchronize()
    xs = out.cpu().numpy() + delta.cpu().numpy()
    assert np.array_equal(s.cpu().numpy(), xs)
    assert np.allclose(nf.cpu().numpy(), R.rms_norm(xs, gamma.cpu().numpy(), 1e-6), rtol=1e-5, atol=1e-6)
    ref_b = R.rms_norm(out.cpu().numpy(), gamma.cpu().numpy(), 1e-6)
    assert np.allclose(nb.float().cpu().numpy(), ref_b, rtol=8e-3, atol=1e-6)  # bf16 output


@pytest.mark.parametrize("h", [2048, 5000, 10000])
@pytest.mark.parametrize("rows", [1, 8])
def test_norm_widths(F, torch, h, rows):
    """Rows spread over a thread-block cluster (up to 8 CTAs, 2048 and 5000
    columns) and the one-CTA-per-row kernels (10000 columns)."""
    N = F._native
    x = _rand(torch, rows, h, seed=h)
    delta = _rand(torch, rows, h, seed=h + 1)
    gamma = _rand(torch, h, seed=h + 2, scale=0.1) + 1.0
    s = torch.empty(rows, h, device="cuda")
    nf = torch.empty(rows, h, device="cuda")
    N.call("fpb_rms_norm", x.data_ptr(), N.FPB_F32, h, delta.data_ptr(), s.data_ptr(), rows, h, gamma.data_ptr(),
           1e-6, nf.data_ptr(), N.FPB_F32, h, None)
    xb = x.to(torch.bfloat16)
    nb = torch.empty(rows, h, device="cuda")
    N.call("fpb_rms_norm", xb.data_ptr(), N.FPB_BF16, h, None, None, rows, h, gamma.data_ptr(), 1e-6, nb.data_ptr(),
           N.FPB_F32, h, None)
    slots = 11
    routed = _rand(torch, rows * slots, h, seed=h + 3)
    wts = torch.rand(rows, slots, device="cuda")
    out = torch.empty(rows, h, device="cuda")
    normed = torch.empty(rows, h, device="cuda")
    N.call("fpb_decode_combine_add_norm", routed.data_ptr(), wts.data_ptr(), slots, slots, x.data_ptr(),
           gamma.data_ptr(), rows, h, 1e-6, out.data_ptr(), normed.data_ptr(), N.FPB_F32, None)
    torch.cuda.synchronize()
    g = gamma.cpu().numpy()
    xs = x.cpu().numpy() + delta.cpu().numpy()
    assert np.array_equal(s.cpu().numpy(), xs)
    assert np.allclose(nf.cpu().numpy(), R.rms_norm(xs, g, 1e-6), rtol=1e-5, atol=1e-6)
    assert np.allclose(nb.cpu().numpy(), R.rms_norm(xb.float().cpu().numpy(), g, 1e-6), rtol=1e-5, atol=1e-6)
    ref = x.cpu().numpy() + np.einsum("ts,tsh->th", wts.cpu().numpy(), routed.cpu().numpy().reshape(rows, slots, h))
    assert np.allclose(out.cpu().numpy(), ref, rtol=1e-5, atol=1e-5)
    assert np.allclose(normed.cpu().numpy(), R.rms_norm(out.cpu().numpy(), g, 1e-6), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("chunk,hq,hkv,D", [(64, 16, 2, 256), (32, 16, 2, 256), (32, 8, 1, 128), (32, 32, 1, 64)])
def test_attention_prepare_and_decode(F, torch, chunk, hq, hkv, D):
    """chunk 32: shared-memory tiles and the per-head merge; 64: one warp per
    query head streaming positions."""
    N = F._native
    B, rot, max_seq, theta = 3, 64, 300, 1e7
    positions = torch.tensor([0, 157, 299], dtype=torch.int32, device="cuda")
    kc = torch.zeros(B, max_seq, hkv, D, device="cuda")
    vc = torch.zeros(B, max_seq, hkv, D, device="cuda")
    # fill the caches' earlier positions with random keys and values
    kc[:] = _rand(torch, B, max_seq, hkv, D, seed=4)
    vc[:] = _rand(torch, B, max_seq, hkv, D, seed=5)
    qg = _rand(torch, B, 2 * hq * D, seed=6)
    k = _rand(torch, B, hkv * D, seed=7)
    v = _rand(torch, B, hkv * D, seed=8)
    qn, kn = _rand(torch, D, seed=9, scale=0.1) + 1, _rand(torch, D, seed=10, scale=0.1) + 1
    q_rot = torch.empty(B, hq, D, device="cuda")
    N.call("fpb_attn_prepare", qg.data_ptr(), qg.shape[1], k.data_ptr(), k.shape[1], v.data_ptr(), v.shape[1],
           qn.data_ptr(), kn.data_ptr(), positions.data_ptr(), B, hq, hkv, D, rot, theta, 1e-6, max_seq,
           q_rot.data_ptr(), kc.data_ptr(), vc.data_ptr(), None)
    ws = torch.empty(int(N.lib.fpb_attn_decode_workspace_bytes(B, hq, D, max_seq, chunk)), dtype=torch.uint8,
                     device="cuda")
    out = torch.empty(B, hq * D, device="cuda")
    scale = 1.0 / math.sqrt(D)
    N.call("fpb_attn_decode", q_rot.data_ptr(), kc.data_ptr(), vc.data_ptr(), positions.data_ptr(), qg.data_ptr(),
           qg.shape[1], B, hq, hkv, D, max_seq, chunk, scale, ws.data_ptr(), ws.numel(), out.data_ptr(), N.FPB_F32,
           None)
    torch.cuda.synchronize()
    assert F.device_error() == 0
    qg_c, k_c, v_c = qg.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy()
    kc_c, vc_c, qr_c = kc.cpu().numpy(), vc.cpu().numpy(), q_rot.cpu().numpy()
    for b in range(B):
        p = int(positions[b])
        for hh in range(hq):
            qh = R.rms_norm(qg_c[b, hh * 2 * D:hh * 2 * D + D], qn.cpu().numpy(), 1e-6)
            assert np.allclose(qr_c[b, hh], R.rope(qh, p, rot, theta), rtol=1e-5, atol=2e-5)
        for hh in range(hkv):
            kh = R.rms_norm(k_c[b, hh * D:(hh + 1) * D], kn.cpu().numpy(), 1e-6)
            assert np.allclose(kc_c[b, p, hh], R.rope(kh, p, rot, theta), rtol=1e-5, atol=2e-5)
            assert np.array_equal(vc_c[b, p, hh], v_c[b, hh * D:(hh + 1) * D])
        att = R.attention_decode(qr_c[b], kc_c[b], vc_c[b], p, scale)
        gate = qg_c[b].reshape(hq, 2 * D)[:, D:]
        want = (att * R.sigmoid(gate)).reshape(-1)
        assert O.rel_frobenius(out.cpu().numpy()[b], want) <= 1e-5


def test_gdn_conv_delta_gated_norm(F, torch):
    N = F._native
    B, hk, hv, dk, dv, kern = 2, 4, 8, 128, 128, 4
    conv_dim = 2 * hk * dk + hv * dv
    x = _rand(torch, B, conv_dim, seed=11)
    state = _rand(torch, B, conv_dim, kern - 1, seed=12)
    w = _rand(torch, conv_dim, kern, seed=13, scale=0.3)
    conv_out = torch.empty(B, conv_dim, device="cuda")
    st0 = state.cpu().numpy().copy()
    N.call("fpb_gdn_conv", x.data_ptr(), conv_dim, state.data_ptr(), w.data_ptr(), B, conv_dim, kern,
           conv_out.data_ptr(), None)
    torch.cuda.synchronize()
    for b in range(B):
        o, ns = R.conv1d_silu(x.cpu().numpy()[b], st0[b], w.cpu().numpy())
        assert np.allclose(conv_out.cpu().numpy()[b], o, rtol=1e-5, atol=1e-6)
        assert np.array_equal(state.cpu().numpy()[b], ns)
    a = _rand(torch, B, hv, seed=14)
    bg = _rand(torch, B, hv, seed=15)
    a[0, 0] = -20.0  # the series branch of the softplus
    a_log = torch.log(1.0 + 15.0 * torch.rand(hv, device="cuda"))
    dt = _rand(torch, hv, seed=16, scale=0.5)
    S = _rand(torch, B, hv, dk, dv, seed=17, scale=0.1)
    S0 = S.cpu().numpy().copy()
    out = torch.empty(B, hv, dv, device="cuda")
    N.call("fpb_gdn_delta", conv_out.data_ptr(), a.data_ptr(), bg.data_ptr(), hv, a_log.data_ptr(), dt.data_ptr(),
           S.data_ptr(), B, hk, hv, dk, dv, 1e-6, out.data_ptr(), None)
    torch.cuda.synchronize()
    co = conv_out.cpu().numpy()
    for b in range(B):
        q = co[b, :hk * dk].reshape(hk, dk)
        k = co[b, hk * dk:2 * hk * dk].reshape(hk, dk)
        v = co[b, 2 * hk * dk:].reshape(hv, dv)
        o, ns = R.delta_step(q, k, v, bg.cpu().numpy()[b], a.cpu().numpy()[b], a_log.cpu().numpy(),
                             dt.cpu().numpy(), S0[b], 1e-6, hk)
        assert O.rel_frobenius(out.cpu().numpy()[b], o) <= 1e-5
        assert O.rel_frobenius(S.cpu().numpy()[b], ns) <= 1e-5
    z = _rand(torch, B, hv * dv, seed=18)
    gamma = _rand(torch, dv, seed=19, scale=0.1) + 1
    g_out = torch.empty(B, hv * dv, device="cuda")
    N.call("fpb_gdn_gated_norm", out.data_ptr(), z.data_ptr(), hv * dv, gamma.data_ptr(), B, hv, dv, 1e-6,
           g_out.data_ptr(), N.FPB_F32, None)
    torch.cuda.synchronize()
    for b in range(B):
        want = R.gated_norm(out.cpu().numpy()[b], z.cpu().numpy()[b].reshape(hv, dv), gamma.cpu().numpy(), 1e-6)
        assert np.allclose(g_out.cpu().numpy()[b], want.reshape(-1), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("B,hk,kern", [(2, 4, 4), (8, 16, 4), (3, 2, 2), (1, 1, 8)])
def test_gdn_step_equals_conv_delta_gated_norm(F, torch, B, hk, kern):
    """fpb_gdn_step (one launch) against the oracle's conv, delta rule and
    gated norm chained in f64, and the three entries' state updates."""
    N = F._native
    hv, dk, dv = 2 * hk, 128, 128
    conv_dim = 2 * hk * dk + hv * dv
    x = _rand(torch, B, conv_dim, seed=31)
    cst = _rand(torch, B, conv_dim, kern - 1, seed=32)
    w = _rand(torch, conv_dim, kern, seed=33, scale=0.3)
    a = _rand(torch, B, hv, seed=34)
    bg = _rand(torch, B, hv, seed=35)
    a[0, 0] = -20.0  # the series branch of the softplus
    a_log = torch.log(1.0 + 15.0 * torch.rand(hv, device="cuda"))
    dt = _rand(torch, hv, seed=36, scale=0.5)
    S = _rand(torch, B, hv, dk, dv, seed=37, scale=0.1)
    z = _rand(torch, B, hv * dv, seed=38)
    gamma = _rand(torch, dv, seed=39, scale=0.1) + 1
    c0, S0 = cst.cpu().numpy().copy(), S.cpu().numpy().copy()
    out = torch.empty(B, hv * dv, device="cuda")
    N.call("fpb_gdn_step", x.data_ptr(), conv_dim, cst.data_ptr(), w.data_ptr(), kern, a.data_ptr(), bg.data_ptr(),
           hv, a_log.data_ptr(), dt.data_ptr(), S.data_ptr(), z.data_ptr(), hv * dv, gamma.data_ptr(), B, hk, hv, dk,
           dv, 1e-6, out.data_ptr(), N.FPB_F32, None)
    torch.cuda.synchronize()
    assert F.device_error() == 0
    for b in range(B):
        co, ns = R.conv1d_silu(x.cpu().numpy()[b], c0[b], w.cpu().numpy())
        assert np.array_equal(cst.cpu().numpy()[b], ns)
        q = co[:hk * dk].reshape(hk, dk)
        k = co[hk * dk:2 * hk * dk].reshape(hk, dk)
        v = co[2 * hk * dk:].reshape(hv, dv)
        o, nS = R.delta_step(q, k, v, bg.cpu().numpy()[b], a.cpu().numpy()[b], a_log.cpu().numpy(), dt.cpu().numpy(),
                             S0[b], 1e-6, hk)
        assert O.rel_frobenius(S.cpu().numpy()[b], nS) <= 1e-5
        want = R.gated_norm(o.astype(np.float32), z.cpu().numpy()[b].reshape(hv, dv), gamma.cpu().numpy(), 1e-6)
        assert O.rel_frobenius(out.cpu().numpy()[b], want.reshape(-1)) <= 1e-5
    bad = N.lib.fpb_gdn_step(x.data_ptr(), conv_dim, cst.data_ptr(), w.data_ptr(), kern, a.data_ptr(), bg.data_ptr(),
                             hv, a_log.data_ptr(), dt.data_ptr(), S.data_ptr(), z.data_ptr(), hv * dv, gamma.data_ptr(),
                             B, hk, hk, dk, dv, 1e-6, out.data_ptr(), N.FPB_F32, None)
    assert bad == N.FPB_ERR_UNSUPPORTED  # one value head per key head


def test_combine_argmax_and_expert_tokens(F, torch):
    N = F._native
    T, slots, h, vocab = 4, 11, 256, 5000
    routed = _rand(torch, T * slots, h, seed=20)
    wts = torch.rand(T, slots, device="cuda")
    resid = _rand(torch, T, h, seed=21)
    gamma = _rand(torch, h, seed=22, scale=0.1) + 1
    out = torch.empty(T, h, device="cuda")
    normed = torch.empty(T, h, device="cuda")
    N.call("fpb_decode_combine_add_norm", routed.data_ptr(), wts.data_ptr(), slots, slots, resid.data_ptr(),
           gamma.data_ptr(), T, h, 1e-6, out.data_ptr(), normed.data_ptr(), N.FPB_F32, None)
    torch.cuda.synchronize()
    ref = resid.cpu().numpy() + np.einsum("ts,tsh->th", wts.cpu().numpy(), routed.cpu().numpy().reshape(T, slots, h))
    assert np.allclose(out.cpu().numpy(), ref, rtol=1e-5, atol=1e-5)
    assert np.allclose(normed.cpu().numpy(), R.rms_norm(out.cpu().numpy(), gamma.cpu().numpy(), 1e-6), rtol=1e-5,
                       atol=1e-6)
    logits = _rand(torch, T, vocab, seed=23)
    logits[1, 17] = float("nan")
    logits[1, 4000] = 50.0
    logits[1, 100] = 50.0  # ties: the lowest index
    logits[2, :] = -float("inf")
    logits[2, 9] = float("inf")  # no finite logit but one: inf is not finite either
    tokens = torch.zeros(T, dtype=torch.int32, device="cuda")
    pos = torch.arange(T, dtype=torch.int32, device="cuda")
    hist = torch.full((T, 3), -1, dtype=torch.int32, device="cuda")
    step = torch.zeros(2, dtype=torch.int32, device="cuda")
    for _ in range(2):
        N.call("fpb_argmax_advance", logits.data_ptr(), T, vocab, tokens.data_ptr(), pos.data_ptr(), hist.data_ptr(),
               3, step.data_ptr(), None)
    torch.cuda.synchronize()
    want = [R.greedy(r) for r in logits.cpu().numpy()]
    want[2] = 0  # no finite logit: token 0
    assert tokens.tolist() == want
    assert pos.tolist() == [2, 3, 4, 5]
    assert hist[:, 0].tolist() == want and hist[:, 1].tolist() == want and hist[:, 2].tolist() == [-1] * T
    assert step.tolist() == [2, 0]
    # expert GEMV over tokens: slot t*slots + j reads x row t
    E, rpe, cols = 6, 128, 512
    w = F.synth_normal((E * rpe, cols), seed=3, stream_id=1, std=0.02)
    W = F.Nvfp4Matrix.quantize(w, rpe)
    hm = W.to_host()
    ids = torch.randint(0, E, (T, 3), dtype=torch.int32, device="cuda")
    x = _rand(torch, T, cols, seed=24).to(torch.bfloat16)
    y = torch.empty(T * 3, rpe, device="cuda")
    N.call("fpb_nvfp4_expert_gemv_tokens", W.handle, x.data_ptr(), N.FPB_BF16, ids.data_ptr(), T, 3, rpe,
           y.data_ptr(), N.FPB_F32, None)
    torch.cuda.synchronize()
    xr = np.repeat(x.float().cpu().numpy(), 3, axis=0)
    ref = O.nvfp4_expert_gemv_f32(hm.packed, hm.scales, hm.row_scales, cols, ids.cpu().numpy().reshape(-1), rpe, 1,
                                  xr)
    assert O.rel_frobenius(y.cpu().numpy(), ref) <= 1e-3
