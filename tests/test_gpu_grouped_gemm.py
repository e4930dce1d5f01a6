"""GPU parity of the grouped (MoE) tcgen05 NVFP4 GEMM against the CPU oracle.

The prefill layout (moe.rs:452-516) is built on the host with 128-row tiles,
the activations are gathered into its padded rows (padding rows zero), and
row tile t is compared with the f64 product of the dequantized activations
and the dequantized rows of expert tile_experts[t] (the reference's grouped
kernel, gemm/nvfp4.rs:56-107, on the same quantized operands): relative
Frobenius error <= 1e-3 and a per-element bound of 1e-5 * sum |a||w|.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu
REL_FROB_TOL = 1e-3


@pytest.fixture(scope="module")
def torch():
    import torch as t
    return t


@pytest.fixture(scope="module")
def F(torch):
    import firepit_b200
    return firepit_b200


def routed_indices(tokens, experts, top_k, seed, skip_expert=None):
    rng = np.random.default_rng(seed)
    pool = [e for e in range(experts) if e != skip_expert]
    return np.stack([rng.choice(pool, size=top_k, replace=False) for _ in range(tokens)]).astype(np.int32)


@pytest.mark.parametrize("tokens,experts,top_k,rpe,k,out", [
    (100, 8, 2, 256, 512, "f32"),
    (300, 4, 2, 128, 2048, "bf16"),
    (37, 16, 4, 384, 256, "f32"),
])
def test_grouped_gemm_vs_oracle(F, torch, tokens, experts, top_k, rpe, k, out):
    dims = F.MoeDims.new(256, 128, 128, experts, top_k)  # the layout reads experts and top_k only
    idx = routed_indices(tokens, experts, top_k, seed=tokens, skip_expert=1)
    layout = F.PrefillLayout.from_indices(idx, dims, 128)
    assert layout.ranges[1][1] == 0  # one expert receives no rows: no tile is launched for it
    w = F.synth_normal((experts * rpe, k), seed=k, stream_id=1, std=0.02)
    W = F.Nvfp4Matrix.quantize(w)
    h = W.to_host()
    x_tok = F.synth_normal((tokens, k), seed=tokens + 1, stream_id=2)
    rows = torch.from_numpy(layout.token_rows.astype(np.int64)).cuda()
    x = torch.where((rows >= 0)[:, None], x_tok[rows.clamp(min=0)], torch.zeros((), device="cuda"))
    ydt = torch.bfloat16 if out == "bf16" else torch.float32
    y = torch.full((layout.padded_rows(), rpe), float("nan"), dtype=ydt, device="cuda")
    F.nvfp4_grouped_gemm_view(W, x, y, layout, experts, rpe).submit(F.Eager())
    assert F.device_error() == 0
    got = y.float().cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(got))

    xc = x.cpu().numpy()
    pa, sa, ga = O.nvfp4_quantize(xc)
    a = O.nvfp4_dequantize(pa, sa, ga, *xc.shape).astype(np.float64)
    wd = O.nvfp4_dequantize(h.packed, h.scales, h.row_scales, h.rows, h.cols).astype(np.float64)
    exp = np.empty_like(got)
    mag = np.empty_like(got)
    for t, e in enumerate(layout.tile_experts):
        we = wd[e * rpe:(e + 1) * rpe]
        at = a[t * 128:(t + 1) * 128]
        exp[t * 128:(t + 1) * 128] = at @ we.T
        mag[t * 128:(t + 1) * 128] = np.abs(at) @ np.abs(we).T
    pad = layout.token_rows < 0
    assert np.all(got[pad] == 0.0)
    if out == "bf16":
        exp_b = O.bf16_to_f32(O.bf16_bits(exp.astype(np.float32))).astype(np.float64)
        assert O.rel_frobenius(got, exp_b) <= REL_FROB_TOL
        assert np.all(np.abs(got - exp) <= 2.0 ** -8 * np.abs(exp) + 1e-5 * mag + 1e-30)
    else:
        assert O.rel_frobenius(got, exp) <= REL_FROB_TOL
        assert np.all(np.abs(got - exp) <= 1e-5 * mag + 1e-30)


def test_grouped_gemm_rejects_bad_shapes(F, torch):
    w = F.synth_normal((512, 256), seed=3, stream_id=1, std=0.02)
    W = F.Nvfp4Matrix.quantize(w)
    a = torch.zeros(128, 128, dtype=torch.uint8, device="cuda")
    te = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = torch.empty(128, 192, device="cuda")
    with pytest.raises(F.FpbError) as e:  # 192 rows per expert: not a multiple of 128
        from firepit_b200 import _native as N
        N.call("fpb_nvfp4_grouped_gemm_q", W.handle, a.data_ptr(), a.data_ptr(), y.data_ptr(), 128, te.data_ptr(),
               None, 192, y.data_ptr(), N.FPB_F32, None)
    assert e.value.status == 2


def _silu_mul(g, u):
    return g / (1.0 + np.exp(-g)) * u


@pytest.mark.parametrize("tokens,experts,top_k,inter,k,out", [
    (100, 8, 2, 64, 512, "f32"),
    (300, 4, 2, 512, 2048, "bf16"),
    (37, 16, 4, 192, 256, "f32"),
    (200, 6, 3, 128, 768, "bf16"),
])
def test_grouped_gemm_swiglu_vs_oracle(F, torch, tokens, experts, top_k, inter, k, out):
    """The gate/up GEMM fused with SwiGLU: h = silu(gate) * up from the f32
    products (swiglu.rs:16 on the grouped GEMM's output), its amax, and the
    row quantizer fed with that amax (bit-exact against the oracle's quantizer
    of the h the device stored)."""
    dims = F.MoeDims.new(256, 128, 128, experts, top_k)
    idx = routed_indices(tokens, experts, top_k, seed=tokens + inter, skip_expert=1)
    layout = F.PrefillLayout.from_indices(idx, dims, 128)
    rpe = 2 * inter
    w = F.synth_normal((experts * rpe, k), seed=k + 5, stream_id=1, std=0.02)
    W = F.Nvfp4Matrix.quantize(w)
    hw = W.to_host()
    x_tok = F.synth_normal((tokens, k), seed=tokens + 2, stream_id=2)
    rows = torch.from_numpy(layout.token_rows.astype(np.int64)).cuda()
    x = torch.where((rows >= 0)[:, None], x_tok[rows.clamp(min=0)], torch.zeros((), device="cuda"))
    packed, sf, ga = F.quantize_act(x)
    te = torch.from_numpy(layout.tile_experts).cuda()
    hdt = torch.bfloat16 if out == "bf16" else torch.float32
    pad = layout.padded_rows()
    h = torch.full((pad, inter), float("nan"), dtype=hdt, device="cuda")
    amax = F.nvfp4_grouped_gemm_swiglu_q(W, packed, sf, ga, te, inter, h)
    assert F.device_error() == 0
    got = h.float().cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(got))

    xc = x.cpu().numpy()
    pa, sa, gq = O.nvfp4_quantize(xc)
    a = O.nvfp4_dequantize(pa, sa, gq, *xc.shape).astype(np.float64)
    wd = O.nvfp4_dequantize(hw.packed, hw.scales, hw.row_scales, hw.rows, hw.cols).astype(np.float64)
    exp = np.empty_like(got)
    tol = np.empty_like(got)
    for t, e in enumerate(layout.tile_experts):
        at = a[t * 128:(t + 1) * 128]
        wg, wu = wd[e * rpe:e * rpe + inter], wd[e * rpe + inter:(e + 1) * rpe]
        g, u = at @ wg.T, at @ wu.T
        eg, eu = 1e-5 * (np.abs(at) @ np.abs(wg).T), 1e-5 * (np.abs(at) @ np.abs(wu).T)
        exp[t * 128:(t + 1) * 128] = _silu_mul(g, u)
        # |d silu/dg| <= 1.1
        tol[t * 128:(t + 1) * 128] = 1.1 * eg * (np.abs(u) + eu) + (np.abs(g) + eg) * eu
    # the epilogue's exp2 / reciprocal approximations and roundings: 4e-6 relative
    tol += 4e-6 * np.abs(exp) + 1e-30
    if out == "bf16":
        tol += 2.0 ** -8 * np.abs(exp)
    assert np.all(np.abs(got - exp) <= tol)
    assert np.all(got[layout.token_rows < 0] == 0.0)
    # amax = max |h| as stored, exactly
    assert amax.view(torch.float32).item() == float(np.abs(got).max())

    q_packed, q_sf, q_g = F.rows_quantize(h, amax=amax)
    hp = h.float().cpu().numpy()
    op, os_, og = O.nvfp4_quantize(hp)
    assert q_g.item() == og[0]
    assert np.array_equal(q_packed.cpu().numpy().reshape(-1), op)
    from test_gpu_gemm import tiled_to_rowmajor
    assert np.array_equal(tiled_to_rowmajor(q_sf.cpu().numpy(), pad, inter).reshape(-1), os_)


def test_grouped_gemm_swiglu_rejects_bad_inter(F, torch):
    w = F.synth_normal((4 * 96, 256), seed=3, stream_id=1, std=0.02)
    W = F.Nvfp4Matrix.quantize(w)
    a = torch.zeros(128, 128, dtype=torch.uint8, device="cuda")
    te = torch.zeros(1, dtype=torch.int32, device="cuda")
    h = torch.empty(128, 96, device="cuda")
    with pytest.raises(F.FpbError) as e:  # inter 96: not a multiple of 64
        F.nvfp4_grouped_gemm_swiglu_q(W, a, a, h[0, :1], te, 96, h)
    assert e.value.status == 2


@pytest.mark.parametrize("per_token", [False, True])
def test_moe_chain_skips_padding_rows(F, torch, per_token):
    """FPB_QUANT_SKIP_PADDING + token_rows: the gather encoder leaves padding
    rows untouched (here: garbage, including NaN factors), the fused GEMM keeps
    them out of h's amax and does not need them, the row quantizer skips them,
    and the down GEMM's live rows still equal the zero-padded computation."""
    from firepit_b200 import _native as N
    tokens, experts, top_k, inter, hid = 150, 8, 2, 128, 256
    dims = F.MoeDims.new(hid, inter, inter, experts, top_k)
    idx = routed_indices(tokens, experts, top_k, seed=11)
    layout = F.PrefillLayout.from_indices(idx, dims, 128)
    pad = layout.padded_rows()
    W1 = F.Nvfp4Matrix.quantize(F.synth_normal((experts * 2 * inter, hid), seed=21, stream_id=1, std=0.02))
    W2 = F.Nvfp4Matrix.quantize(F.synth_normal((experts * hid, inter), seed=22, stream_id=1, std=0.02))
    x = F.synth_normal((tokens, hid), seed=23, stream_id=2, dtype=torch.bfloat16)
    tr = torch.from_numpy(layout.token_rows).cuda()
    te = torch.from_numpy(layout.tile_experts).cuda()
    live = layout.token_rows >= 0
    g = torch.Generator(device="cuda").manual_seed(5)

    def garbage(n):
        return torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda", generator=g)

    def run(skip):
        a1 = garbage(pad * hid // 2).view(pad, hid // 2)
        sf1 = garbage(int(N.lib.fpb_nvfp4_act_sf_bytes(pad, hid)))
        scal = torch.zeros(4, dtype=torch.float32, device="cuda")
        flags = N.FPB_QUANT_SKIP_PADDING if skip else 0
        ws_bytes = int(N.lib.fpb_moe_gather_quantize_workspace_bytes(tokens, hid)) if per_token else 0
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
        N.call("fpb_moe_gather_quantize", x.data_ptr(), N.FPB_BF16, tokens, hid, tr.data_ptr(), pad, None,
               a1.data_ptr(), sf1.data_ptr(), scal.data_ptr(), scal[1:].data_ptr(), flags,
               ws.data_ptr() if per_token else None, ws_bytes, None)
        h = torch.full((pad, inter), float("nan"), dtype=torch.bfloat16, device="cuda")
        amax = F.nvfp4_grouped_gemm_swiglu_q(W1, a1, sf1, scal[:1], te, inter, h, token_rows=tr if skip else None)
        a2 = garbage(pad * inter // 2).view(pad, inter // 2)
        sf2 = garbage(int(N.lib.fpb_nvfp4_act_sf_bytes(pad, inter)))
        _, _, g2 = F.rows_quantize(h, amax=amax, token_rows=tr if skip else None, out=(a2, sf2))
        y = torch.full((pad, hid), float("nan"), dtype=torch.bfloat16, device="cuda")
        F.nvfp4_grouped_gemm_q(W2, a2, sf2, g2, te, hid, y, token_rows=tr if skip else None)
        torch.cuda.synchronize()
        assert F.device_error() == 0
        return h.float().cpu().numpy(), amax.view(torch.float32).item(), y.float().cpu().numpy()

    h0, amax0, y0 = run(False)  # zero padding rows, everything written
    h1, amax1, y1 = run(True)
    assert np.array_equal(h1[live], h0[live])
    assert amax1 == float(np.abs(h0[live]).max()) == amax0  # padding rows of h0 are zeros
    assert np.array_equal(y1[live], y0[live])
    # a 32-row group with no live row is not written at all
    groups = live.reshape(-1, 32).any(axis=1)
    dead = np.repeat(~groups, 32)
    assert dead.any() and np.isnan(y1[dead]).all() and np.isnan(h1[dead]).all()
