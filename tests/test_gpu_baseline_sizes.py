"""Parity at BASELINE's own sizes.

* Config 3: the whole MoE layer at E = 512 experts, top-10, H = 2048,
  I = 512, for T = 64 (decode batch) and T = 4096 (prefill), every stage
  checked against the oracle on the previous stage's device output
  (moe.rs:15-147 top-k / layout / combine, gemm/nvfp4.rs:57-105 grouped GEMM,
  swiglu.rs:16):
    - top-k ids, the expert-sorted layout and every quantized byte: exact;
    - routing weights: relative 2e-6 (device and host exp differ in the last
      place);
    - gate/up + SwiGLU and down GEMMs: relative Frobenius error <= 1e-3
      against the f64 product of the same dequantized operands, on every live
      row at T = 64 and on a sample of 24 row tiles (3072 rows) at T = 4096;
    - combine: relative 1e-6.
* Config 2 at M = 1 and M = 16 (K = 2048, N = 8192): through the decode GEMV
  entry (bf16 x kept, W4A16) against the oracle's f32 kernel-order GEMV, and
  through the public nvfp4_gemm entry (x quantized to NVFP4, W4A4) against
  the f64 product of the dequantized operands; relative Frobenius <= 1e-3.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu
REL_FROB_TOL = 1e-3
E, K, H, I = 512, 10, 2048, 512
WIDTH = 16


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


@pytest.fixture(scope="module")
def F(torch):
    import firepit_b200
    return firepit_b200


def tiled_to_rowmajor(sf_tiled: np.ndarray, rows: int, cols: int) -> np.ndarray:
    groups = cols // 16
    kb64 = (cols + 255) // 256 * 4
    r = np.arange(rows)[:, None]
    g = np.arange(groups)[None, :]
    off = ((r // 128) * kb64 + g // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + g % 4
    return sf_tiled[off]


@pytest.fixture(scope="module")
def experts(F, torch):
    """512 experts' gate/up [2I, H] and down [H, I] from N(0, 0.02), NVFP4
    with one global per expert, stacked (streams 1000+e / 5000+e)."""
    dev = torch.device("cuda")
    gp, gs, gg, dp, ds, dg = [], [], [], [], [], []
    chunk = 64
    for e0 in range(0, E, chunk):
        g = torch.empty(chunk, 2 * I, H, device=dev)
        d = torch.empty(chunk, H, I, device=dev)
        for j in range(chunk):
            F.synth_normal(g[j].shape, seed=0, stream_id=1000 + e0 + j, std=0.02, out=g[j])
            F.synth_normal(d[j].shape, seed=0, stream_id=5000 + e0 + j, std=0.02, out=d[j])
        a, b, c = F.quantize_nvfp4(g.view(-1, H), 2 * I)
        gp.append(a), gs.append(b), gg.append(c)
        a, b, c = F.quantize_nvfp4(d.view(-1, I), H)
        dp.append(a), ds.append(b), dg.append(c)
        del g, d
    W1 = F.Nvfp4Matrix.from_device(torch.cat(gp), torch.cat(gs), torch.cat(gg), E * 2 * I, H)
    W2 = F.Nvfp4Matrix.from_device(torch.cat(dp), torch.cat(ds), torch.cat(dg), E * H, I)
    W1.prepare_glu(I)
    return W1, W2, W1.to_host(), W2.to_host()


def _dequant_rows(h, r0, r1, cols):
    """Rows [r0, r1) of a host NVFP4 matrix, dequantized (f64)."""
    p = h.packed.reshape(h.rows, cols // 2)[r0:r1].reshape(-1)
    s = h.scales.reshape(h.rows, cols // 16)[r0:r1].reshape(-1)
    return O.nvfp4_dequantize(p, s, h.row_scales[r0:r1], r1 - r0, cols).astype(np.float64)


def _dequant_act(packed, sf, g, rows, cols, sel):
    pk = packed.reshape(rows, cols // 2)[sel]
    fac = tiled_to_rowmajor(sf, rows, cols)[sel]
    return O.nvfp4_dequantize(pk.reshape(-1), fac.reshape(-1), np.full(len(sel), g, np.float32), len(sel),
                              cols).astype(np.float64)


@pytest.mark.parametrize("T", [64, 4096])
def test_config3_moe_layer_stage_by_stage(F, torch, experts, T):
    N_ = F._native
    F32 = N_.FPB_F32
    W1, W2, h1, h2 = experts
    dev = torch.device("cuda")
    s = torch.cuda.current_stream().cuda_stream
    wr = F.synth_normal((E, H), seed=0, stream_id=99, std=0.02, dtype=torch.bfloat16)
    x = F.synth_normal((T, H), seed=0, stream_id=0, dtype=torch.bfloat16)
    logits = torch.mm(x, wr.t(), out_dtype=torch.float32)
    router = F.MoeDims.new(H, I, I, E, K)
    cap = F.PrefillPlan.capacity(T, router, 128)
    i32 = dict(dtype=torch.int32, device=dev)
    ids, w = torch.empty(T, WIDTH, **i32), torch.empty(T, WIDTH, device=dev)
    tr, te = torch.empty(cap, **i32), torch.empty(cap // 128, **i32)
    inv, rg, pad = torch.empty(T, WIDTH, **i32), torch.empty(E, 2, dtype=torch.int64, device=dev), torch.empty(1, **i32)
    lscr = torch.empty(int(N_.lib.fpb_moe_layout_scratch_bytes(T, K, E)), dtype=torch.uint8, device=dev)
    gws = torch.empty(int(N_.lib.fpb_moe_gather_quantize_workspace_bytes(T, H)), dtype=torch.uint8, device=dev)
    a1 = torch.empty(cap, H // 2, dtype=torch.uint8, device=dev)
    sf1 = torch.zeros(int(N_.lib.fpb_nvfp4_act_sf_bytes(cap, H)), dtype=torch.uint8, device=dev)
    hh = torch.zeros(cap, I, device=dev)
    a2 = torch.empty(cap, I // 2, dtype=torch.uint8, device=dev)
    sf2 = torch.zeros(int(N_.lib.fpb_nvfp4_act_sf_bytes(cap, I)), dtype=torch.uint8, device=dev)
    y2 = torch.zeros(cap, H, device=dev)
    out = torch.empty(T, H, device=dev)
    scal = torch.zeros(4, device=dev)
    skip = N_.FPB_QUANT_SKIP_PADDING
    N_.call("fpb_moe_topk", logits.data_ptr(), E, None, T, E, K, WIDTH, ids.data_ptr(), w.data_ptr(), s)
    N_.call("fpb_moe_layout", ids.data_ptr(), T, WIDTH, K, E, 128, cap, tr.data_ptr(), te.data_ptr(), inv.data_ptr(),
            rg.data_ptr(), pad.data_ptr(), lscr.data_ptr(), lscr.numel(), s)
    N_.call("fpb_moe_gather_quantize", x.data_ptr(), N_.FPB_BF16, T, H, tr.data_ptr(), cap, pad.data_ptr(),
            a1.data_ptr(), sf1.data_ptr(), scal.data_ptr(), scal[1:].data_ptr(), skip, gws.data_ptr(), gws.numel(), s)
    N_.call("fpb_nvfp4_grouped_gemm_swiglu_q", W1.handle, a1.data_ptr(), sf1.data_ptr(), scal.data_ptr(), cap,
            te.data_ptr(), tr.data_ptr(), I, hh.data_ptr(), F32, scal[3:].data_ptr(), s)
    N_.call("fpb_rows_quantize", hh.data_ptr(), F32, cap, pad.data_ptr(), tr.data_ptr(), I, a2.data_ptr(),
            sf2.data_ptr(), scal[2:].data_ptr(), scal[3:].data_ptr(), N_.FPB_QUANT_AMAX_GIVEN | skip, s)
    N_.call("fpb_nvfp4_grouped_gemm_q", W2.handle, a2.data_ptr(), sf2.data_ptr(), scal[2:].data_ptr(), cap,
            te.data_ptr(), tr.data_ptr(), H, y2.data_ptr(), F32, s)
    N_.call("fpb_moe_combine", y2.data_ptr(), F32, cap, H, inv.data_ptr(), w.data_ptr(), T, WIDTH, K,
            out.data_ptr(), F32, s)
    torch.cuda.synchronize()
    assert F.device_error() == 0

    # top-k (moe.rs:15-68) on the same f32 logits
    ids_ref, w_ref = O.moe_topk(logits.cpu().numpy(), K, WIDTH)
    ids_c, w_c = ids.cpu().numpy(), w.cpu().numpy()
    assert np.array_equal(ids_c[:, :K], ids_ref[:, :K])
    assert np.allclose(w_c[:, :K], w_ref[:, :K], rtol=2e-6, atol=0)
    # layout (moe.rs:452-516, 128-row tiles)
    tr_ref, te_ref, inv_ref, rg_ref, pad_ref = O.moe_layout(ids_c, K, E, 128, cap)
    padded = int(pad.item())
    assert padded == pad_ref
    assert np.array_equal(tr.cpu().numpy()[:padded], tr_ref[:padded])
    assert np.array_equal(te.cpu().numpy()[:padded // 128], te_ref[:padded // 128])
    assert np.array_equal(inv.cpu().numpy()[:, :K], inv_ref[:, :K])
    assert np.array_equal(rg.cpu().numpy(), rg_ref)
    tr_c = tr.cpu().numpy()[:padded]
    live = np.nonzero(tr_c >= 0)[0]
    assert live.size == T * K
    # gather + quantize: every live row equals the oracle's encoding of its token
    xp, xs, xg = O.nvfp4_quantize(x.float().cpu().numpy())
    a1_c = a1.cpu().numpy()
    sf1_c = sf1.cpu().numpy()
    assert scal[0].item() == xg[0]
    assert np.array_equal(a1_c[live], xp.reshape(T, H // 2)[tr_c[live]])
    assert np.array_equal(tiled_to_rowmajor(sf1_c, cap, H)[live], xs.reshape(T, H // 16)[tr_c[live]])
    # the rows checked against f64 products: all at T = 64, 24 tiles at T = 4096
    te_c = te.cpu().numpy()[:padded // 128]
    tiles = np.arange(te_c.size)
    if T > 64:
        rng = np.random.default_rng(3)
        tiles = np.unique(np.concatenate([[0, te_c.size - 1], rng.choice(te_c.size, 22, replace=False)]))
    hh_c = hh.cpu().numpy()
    g1 = float(scal[0].item())
    for t in tiles:
        e = int(te_c[t])
        rows = np.arange(t * 128, (t + 1) * 128)
        rows = rows[tr_c[rows] >= 0]
        a = _dequant_act(a1_c, sf1_c, g1, cap, H, rows)
        gu = a @ _dequant_rows(h1, e * 2 * I, (e + 1) * 2 * I, H).T
        want = gu[:, :I] / (1.0 + np.exp(-gu[:, :I])) * gu[:, I:]
        assert O.rel_frobenius(hh_c[rows].astype(np.float64), want) <= REL_FROB_TOL, f"gate/up tile {t}"
    # h quantize: the oracle's quantizer on the device's own h (live rows, one global)
    hp, hs, hg = O.nvfp4_quantize(hh_c[live])
    a2_c, sf2_c = a2.cpu().numpy(), sf2.cpu().numpy()
    assert np.array_equal(a2_c[live], hp.reshape(live.size, I // 2))
    assert np.array_equal(tiled_to_rowmajor(sf2_c, cap, I)[live], hs.reshape(live.size, I // 16))
    assert scal[2].item() == hg[0]
    y2_c = y2.cpu().numpy()
    for t in tiles:
        e = int(te_c[t])
        rows = np.arange(t * 128, (t + 1) * 128)
        rows = rows[tr_c[rows] >= 0]
        a = _dequant_act(a2_c, sf2_c, float(hg[0]), cap, I, rows)
        want = a @ _dequant_rows(h2, e * H, (e + 1) * H, I).T
        assert O.rel_frobenius(y2_c[rows].astype(np.float64), want) <= REL_FROB_TOL, f"down tile {t}"
    ref = O.moe_combine(y2_c, inv.cpu().numpy(), w_c, K)
    assert np.allclose(out.cpu().numpy(), ref, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("m", [1, 16])
def test_config2_small_m_through_public_entries(F, torch, m):
    n, k = 8192, 2048
    w = F.synth_normal((n, k), seed=0, stream_id=1, std=0.02)
    W = F.Nvfp4Matrix.quantize(w)
    h = W.to_host()
    x = F.synth_normal((m, k), seed=0, stream_id=0, dtype=torch.bfloat16)
    xf = x.float().cpu().numpy()
    # decode GEMV entry: bf16 x as is (W4A16), the reference's kernel order
    y = torch.full((m, n), float("nan"), device="cuda")
    F.gemv(W, x, y).submit(F.Eager())
    ref = O.nvfp4_gemv_f32(h.packed, h.scales, h.row_scales, n, k, xf)
    assert O.rel_frobenius(y.cpu().numpy(), ref) <= REL_FROB_TOL
    # GEMM entry: config 2 keeps decode-size activations in bf16 (its NVFP4
    # activation rule is for M >= 128), so nvfp4_gemm runs the tensor-core
    # GEMV (x as NVFP4 digit planes): the f64 product of bf16 x and the
    # dequantized weights
    yg = torch.full((m, n), float("nan"), device="cuda")
    F.nvfp4_gemm(W, x, yg, F.GemmTile(m, 128, 32)).submit(F.Eager())
    assert F.device_error() == 0
    wd = O.nvfp4_dequantize(h.packed, h.scales, h.row_scales, n, k).astype(np.float64)
    assert O.rel_frobenius(yg.cpu().numpy().astype(np.float64), xf.astype(np.float64) @ wd.T) <= 1e-5
