"""GPU parity of the device MoE pieces against the CPU oracle.

* top-k (moe.rs:15-68): ids identical, weights within 2 ulp-scale relative
  error (the device and host exp differ in the last place).
* layout (moe.rs:452-516): identical to the oracle's stable counting sort and
  to the library's host sort.
* gather + NVFP4 quantize and SwiGLU + NVFP4 quantize: bit-exact against the
  oracle's quantizer applied to the same rows.
* combine / combine_add_norm (moe.rs:91-147): relative error <= 1e-6 / 1e-5.
* A small full prefill MoE (router top-k -> layout -> gather-quantize ->
  grouped gate/up GEMM -> SwiGLU-quantize -> grouped down GEMM -> combine),
  every stage checked against the oracle on the previous stage's device output.
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


def tiled_padding(sf_tiled: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Bytes of the tiled factor layout past the last 16-column group (K padded to 256)."""
    kb64 = (cols + 255) // 256 * 4
    chunk = np.arange(sf_tiled.size) // 512
    byte = np.arange(sf_tiled.size) % 512
    group = (chunk % kb64) * 4 + byte % 4
    return sf_tiled[group >= cols // 16]


def tiled_to_rowmajor(sf_tiled: np.ndarray, rows: int, cols: int) -> np.ndarray:
    groups = cols // 16
    kb64 = (cols + 255) // 256 * 4
    r = np.arange(rows)[:, None]
    g = np.arange(groups)[None, :]
    off = ((r // 128) * kb64 + g // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + g % 4
    return sf_tiled[off]


@pytest.mark.parametrize("tokens,experts,k,shared,ties", [(64, 512, 10, False, False), (300, 512, 10, True, False),
                                                         (100, 100, 4, True, False), (50, 8, 2, False, False),
                                                         (200, 64, 6, True, True), (7, 2048, 8, True, False)])
def test_topk_vs_oracle(F, torch, tokens, experts, k, shared, ties):
    rng = np.random.default_rng(tokens + experts)
    logits = (rng.integers(-4, 4, (tokens, experts)) if ties else rng.standard_normal((tokens, experts)) * 2)
    logits = logits.astype(np.float32)
    gate = rng.standard_normal(tokens).astype(np.float32) if shared else None
    width = 1 << (k + (1 if shared else 0) - 1).bit_length()
    ids_d, w_d = F.topk_device(torch.from_numpy(logits).cuda(), k, width,
                               None if gate is None else torch.from_numpy(gate).cuda().view(tokens, 1))
    ids_o, w_o = O.moe_topk(logits, k, width, gate)
    assert np.array_equal(ids_d.cpu().numpy(), ids_o)
    assert np.allclose(w_d.cpu().numpy(), w_o, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("tokens,experts,k,tile", [(4096, 512, 10, 128), (64, 512, 10, 128), (300, 513, 11, 32),
                                                   (1000, 17, 3, 128), (5, 4, 4, 128), (5000, 4, 4, 128),
                                                   (20000, 160, 8, 128)])
def test_layout_vs_oracle(F, torch, tokens, experts, k, tile):
    rng = np.random.default_rng(tokens)
    width = 1 << (k - 1).bit_length()
    ids = np.zeros((tokens, width), np.int32)
    for t in range(tokens):
        ids[t, :k] = rng.choice(experts, k, replace=False)
    dims = F.MoeDims(256, 128, 128, experts, k)
    cap = F.PrefillPlan.capacity(tokens, dims, tile)
    out = {n: torch.empty(sz, dtype=dt, device="cuda") for n, sz, dt in
           [("tr", (cap,), torch.int32), ("te", (cap // tile,), torch.int32), ("inv", (tokens, width), torch.int32),
            ("rg", (experts, 2), torch.int64), ("pad", (1,), torch.int32)]}
    scratch = F.moe.layout_scratch(tokens, k, experts, "cuda")
    F._native.call("fpb_moe_layout", torch.from_numpy(ids).cuda().data_ptr(), tokens, width, k, experts, tile, cap,
                   out["tr"].data_ptr(), out["te"].data_ptr(), out["inv"].data_ptr(), out["rg"].data_ptr(),
                   out["pad"].data_ptr(), scratch.data_ptr(), scratch.numel(), torch.cuda.current_stream().cuda_stream)
    assert F.device_error() == 0
    tr, te, inv, rg, pad = O.moe_layout(ids, k, experts, tile, cap)
    assert int(out["pad"].item()) == pad
    assert np.array_equal(out["tr"].cpu().numpy(), tr)
    assert np.array_equal(out["te"].cpu().numpy(), te)
    assert np.array_equal(out["inv"].cpu().numpy(), inv)
    assert np.array_equal(out["rg"].cpu().numpy(), rg)
    host = F.PrefillLayout.from_indices(ids[:, :k], dims, tile)  # the library's host sort
    assert np.array_equal(host.token_rows, tr[:pad]) and np.array_equal(host.inverse, inv[:, :k].reshape(-1))


def test_plan_top_k_matches_host_parse(F, torch):
    tokens, experts, k = 257, 64, 6
    router = F.MoeDims.new(256, 128, 128, experts, k)
    rng = np.random.default_rng(3)
    logits = torch.from_numpy(rng.standard_normal((tokens, experts)).astype(np.float32)).cuda()
    gate = torch.from_numpy(rng.standard_normal((tokens, 1)).astype(np.float32)).cuda()
    plan = F.PrefillPlan.top_k(logits, gate, router, 128)
    ids = plan.indices.cpu().numpy()[:, :k + 1]
    ref = F.PrefillLayout.from_indices(ids, router.with_shared_expert(), 128)
    got = plan.layout()
    assert np.array_equal(got.token_rows, ref.token_rows)
    assert np.array_equal(got.tile_experts, ref.tile_experts)
    assert np.array_equal(got.inverse, ref.inverse)
    assert got.ranges == ref.ranges
    assert np.all(ids[:, k] == experts)


@pytest.mark.parametrize("per_token", [True, False])
@pytest.mark.parametrize("dtype,h", [("f32", 512), ("bf16", 512), ("bf16", 384), ("bf16", 2048), ("f32", 1024)])
def test_gather_and_gather_quantize(F, torch, dtype, h, per_token):
    tokens, experts, k = 300, 16, 4
    router = F.MoeDims(h, 128, 128, experts, k)  # routing reads experts and top_k only (h = 384 is not a MoeDims)
    rng = np.random.default_rng(11)
    logits = torch.from_numpy(rng.standard_normal((tokens, experts)).astype(np.float32)).cuda()
    plan = F.PrefillPlan.top_k(logits, None, router, 128)
    x = F.synth_normal((tokens, h), seed=1, stream_id=3)
    if dtype == "bf16":
        x = x.to(torch.bfloat16)
    sorted_ = torch.empty(plan.cap, h, device="cuda")
    F.gather_prefill_view(sorted_, x, plan)
    tr = plan.token_rows.cpu().numpy()
    xc = x.float().cpu().numpy()
    want = np.where((tr >= 0)[:, None], xc[np.maximum(tr, 0)], 0).astype(np.float32)
    assert np.array_equal(sorted_.cpu().numpy(), want)
    packed, sf, g = F.gather_quantize(x, plan, per_token=per_token)
    pad = plan.padded_rows()  # rows past the layout's end are left unwritten
    pa, sa, ga = O.nvfp4_quantize(want[:pad])
    assert g.cpu().numpy()[0] == ga[0]
    assert np.array_equal(packed.cpu().numpy()[:pad].reshape(-1), pa)
    assert np.array_equal(tiled_to_rowmajor(sf.cpu().numpy(), plan.cap, h)[:pad].reshape(-1), sa)
    assert np.all(tiled_padding(sf.cpu().numpy(), plan.cap, h) == 0)


@pytest.mark.parametrize("dtype,inter", [("f32", 256), ("bf16", 256), ("f32", 128), ("bf16", 96), ("bf16", 512),
                                         ("f32", 1024), ("bf16", 2048)])
def test_swiglu_and_swiglu_quantize(F, torch, dtype, inter):
    rows = 384
    gu = F.synth_normal((rows, 2 * inter), seed=2, stream_id=5, std=3.0)
    if dtype == "bf16":
        gu = gu.to(torch.bfloat16)
    out = torch.empty(rows, inter, device="cuda")
    F.swiglu(out, gu)
    ref = O.swiglu(gu.float().cpu().numpy())
    got = out.cpu().numpy()
    assert np.allclose(got, ref, rtol=2e-6, atol=1e-7)
    packed, sf, g = F.swiglu_quantize(gu)
    pa, sa, ga = O.nvfp4_quantize(got)  # same device silu values, oracle quantizer
    assert g.cpu().numpy()[0] == ga[0]
    assert np.array_equal(packed.cpu().numpy().reshape(-1), pa)
    assert np.array_equal(tiled_to_rowmajor(sf.cpu().numpy(), rows, inter).reshape(-1), sa)
    assert np.all(tiled_padding(sf.cpu().numpy(), rows, inter) == 0)  # K padding read by the tensor cores


@pytest.mark.parametrize("out_dtype", ["f32", "bf16"])
def test_combine_and_add_norm(F, torch, out_dtype):
    tokens, h, experts, k = 200, 512, 16, 4
    router = F.MoeDims.new(h, 128, 128, experts, k)
    rng = np.random.default_rng(5)
    logits = torch.from_numpy(rng.standard_normal((tokens, experts)).astype(np.float32)).cuda()
    gate = torch.from_numpy(rng.standard_normal((tokens, 1)).astype(np.float32)).cuda()
    plan = F.PrefillPlan.top_k(logits, gate, router, 128)
    routed = F.synth_normal((plan.cap, h), seed=7, stream_id=1)
    odt = torch.bfloat16 if out_dtype == "bf16" else torch.float32
    out = torch.empty(tokens, h, dtype=odt, device="cuda")
    F.combine_prefill(out, routed, plan)
    inv, w = plan.inverse.cpu().numpy(), plan.weights.cpu().numpy()
    ref = O.moe_combine(routed.cpu().numpy(), inv, w, k + 1)
    tol = 2.0 ** -8 if out_dtype == "bf16" else 1e-6
    assert np.allclose(out.float().cpu().numpy(), ref, rtol=tol, atol=1e-6)
    res = F.synth_normal((tokens, h), seed=8, stream_id=1)
    gamma = F.synth_normal((h,), seed=9, stream_id=1, mean=1.0, std=0.1)
    o2 = torch.empty(tokens, h, device="cuda")
    nrm = torch.empty(tokens, h, device="cuda")
    F.combine_add_norm_prefill(o2, nrm, routed, plan, res, gamma, 1e-6)
    r_out, r_norm = O.moe_combine(routed.cpu().numpy(), inv, w, k + 1, res.cpu().numpy(), gamma.cpu().numpy(), 1e-6)
    assert np.allclose(o2.cpu().numpy(), r_out, rtol=1e-6, atol=1e-6)
    assert np.allclose(nrm.cpu().numpy(), r_norm, rtol=1e-5, atol=1e-5)
    # decode combine over one token's selection (routed rows in slot order)
    sel = F.ExpertSelection.parse([3, 1, 7, 0], [0.1, 0.2, 0.3, 0.4], router)
    rt = F.synth_normal((4, h), seed=10, stream_id=1)
    o3 = torch.empty(1, h, device="cuda")
    F.combine(o3, rt, sel)
    want = (np.array([0.1, 0.2, 0.3, 0.4], np.float32)[:, None] * rt.cpu().numpy()).sum(0)
    assert np.allclose(o3.cpu().numpy()[0], want, rtol=1e-6, atol=1e-6)


def _dequant_act(packed, sf, g, rows, cols):
    return O.nvfp4_dequantize(packed.cpu().numpy().reshape(-1), tiled_to_rowmajor(sf.cpu().numpy(), rows, cols)
                              .reshape(-1), np.full(rows, g.cpu().numpy()[0], np.float32), rows, cols)


def test_moe_prefill_pipeline(F, torch):
    tokens, h, inter, experts, k = 200, 256, 128, 16, 4
    router = F.MoeDims.new(h, inter, inter, experts, k)
    dims = router.with_shared_expert()
    e_all = dims.experts
    rng = np.random.default_rng(21)
    logits = torch.from_numpy(rng.standard_normal((tokens, experts)).astype(np.float32)).cuda()
    gate = torch.from_numpy(rng.standard_normal((tokens, 1)).astype(np.float32)).cuda()
    x = F.synth_normal((tokens, h), seed=0, stream_id=0, dtype=torch.bfloat16)
    w1 = F.synth_normal((e_all * 2 * inter, h), seed=1, stream_id=1, std=0.02)
    w2 = F.synth_normal((e_all * h, inter), seed=2, stream_id=1, std=0.02)
    W1 = F.Nvfp4Matrix.quantize(w1, 2 * inter)  # one global per expert
    W2 = F.Nvfp4Matrix.quantize(w2, h)
    plan = F.PrefillPlan.top_k(logits, gate, router, 128)
    te = plan.tile_experts
    a1, sf1, g1 = F.gather_quantize(x, plan)
    y1 = torch.zeros(plan.cap, 2 * inter, device="cuda")
    F.nvfp4_grouped_gemm_q(W1, a1, sf1, g1, te, 2 * inter, y1)
    a2, sf2, g2 = F.swiglu_quantize(y1, valid_rows=plan.padded_rows_dev)
    y2 = torch.zeros(plan.cap, h, device="cuda")
    F.nvfp4_grouped_gemm_q(W2, a2, sf2, g2, te, h, y2)
    out = torch.empty(tokens, h, device="cuda")
    F.combine_prefill(out, y2, plan)
    assert F.device_error() == 0
    pad = plan.padded_rows()
    tiles = plan.tile_experts.cpu().numpy()[:pad // 128]
    h1, h2 = W1.to_host(), W2.to_host()
    wd1 = O.nvfp4_dequantize(h1.packed, h1.scales, h1.row_scales, h1.rows, h1.cols).astype(np.float64)
    wd2 = O.nvfp4_dequantize(h2.packed, h2.scales, h2.row_scales, h2.rows, h2.cols).astype(np.float64)
    ad1 = _dequant_act(a1, sf1, g1, plan.cap, h).astype(np.float64)
    ad2 = _dequant_act(a2, sf2, g2, plan.cap, inter).astype(np.float64)
    y1c, y2c = y1.cpu().numpy(), y2.cpu().numpy()
    for t, e in enumerate(tiles):
        rs = slice(t * 128, (t + 1) * 128)
        e1 = ad1[rs] @ wd1[e * 2 * inter:(e + 1) * 2 * inter].T
        e2 = ad2[rs] @ wd2[e * h:(e + 1) * h].T
        assert O.rel_frobenius(y1c[rs].astype(np.float64), e1) <= REL_FROB_TOL
        assert O.rel_frobenius(y2c[rs].astype(np.float64), e2) <= REL_FROB_TOL
    ref = O.moe_combine(y2c, plan.inverse.cpu().numpy(), plan.weights.cpu().numpy(), k + 1)
    assert np.allclose(out.cpu().numpy(), ref, rtol=1e-6, atol=1e-6)
    # Smoke check, not a parity claim (parity is the stage-by-stage checks
    # above and tests/test_gpu_baseline_sizes.py): against f64 from the
    # unquantized operands, where NVFP4 weights and activations cost a few
    # percent, the bar only catches gross errors such as a wrong expert.
    xs = x.float().cpu().numpy().astype(np.float64)
    ids, wts = plan.indices.cpu().numpy(), plan.weights.cpu().numpy()
    e2e = np.zeros((tokens, h))
    w1f, w2f = w1.cpu().numpy().astype(np.float64), w2.cpu().numpy().astype(np.float64)
    for t in range(tokens):
        for s in range(k + 1):
            e = ids[t, s]
            gu = xs[t] @ w1f[e * 2 * inter:(e + 1) * 2 * inter].T
            act = gu[:inter] / (1 + np.exp(-gu[:inter])) * gu[inter:]
            e2e[t] += wts[t, s] * (act @ w2f[e * h:(e + 1) * h].T)
    assert O.rel_frobenius(out.cpu().numpy().astype(np.float64), e2e) <= 0.25
