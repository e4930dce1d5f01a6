"""GPU parity of the NVFP4 path against the CPU oracle, through the C ABI.

Bars: bit-exact for the generator, quantize, pack and dequantize; the
reference's per-element Higham-Mary bound (kernels tests/common/check.rs,
n = K + 2 for the GEMV, nvfp4_oracle.rs:219) and relative Frobenius error
<= 1e-3 against the oracle's f32 kernel-order result for the GEMVs.
"""
import numpy as np
import pytest

import refcases as R
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_FROB_TOL = 1e-3  # north star: matmul outputs vs fp32-accumulated oracle


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


@pytest.fixture(scope="module")
def F(torch):
    import firepit_b200
    return firepit_b200


def host_matrix(F, packed, scales, row_globals, rows, cols):
    return F.HostNvfp4Matrix(np.ascontiguousarray(packed, np.uint8), np.ascontiguousarray(scales, np.uint8),
                             np.ascontiguousarray(row_globals, np.float32), rows, cols)


# ---- synthetic data ---------------------------------------------------------------------
@pytest.mark.parametrize("seed,stream,offset", [(0, 0, 0), (7, 3, 12345), (2 ** 40 + 5, 11, 2 ** 33 + 1)])
def test_synth_normal_bit_exact(F, torch, seed, stream, offset):
    n = 1 << 20
    dev = F.synth_normal((n,), seed=seed, stream_id=stream, mean=0.25, std=0.5, offset=offset).cpu().numpy()
    cpu = O.synth_normal(n, seed, stream, mean=0.25, std=0.5, offset=offset)
    assert np.array_equal(dev.view(np.uint32), cpu.view(np.uint32))
    assert abs(cpu.mean() - 0.25) < 0.01 and abs(cpu.std() - 0.5) < 0.01
    bf = F.synth_normal((4096,), seed=seed, stream_id=stream, mean=0.25, std=0.5, dtype=torch.bfloat16,
                        offset=offset)
    assert np.array_equal(bf.view(torch.int16).cpu().numpy().view(np.uint16), O.bf16_bits(cpu[:4096]))


# ---- quantize / dequantize ---------------------------------------------------------------
@pytest.mark.parametrize("rows,cols,rpg,std", [(256, 512, 256, 0.02), (96, 4096, 32, 1.0), (64, 160, 1, 3.0),
                                               (8, 32, 8, 1e-30)])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_quantize_bit_exact(F, torch, rows, cols, rpg, std, dtype):
    w = F.synth_normal((rows, cols), seed=rows + cols, stream_id=1, std=std)
    if dtype == "bf16":
        w = w.to(torch.bfloat16)
    packed, scales, g = F.quantize_nvfp4(w, rpg)
    w_cpu = w.float().cpu().numpy()
    p_ref, s_ref, g_ref = O.nvfp4_quantize(w_cpu, rpg)
    assert np.array_equal(g.cpu().numpy().view(np.uint32), g_ref.view(np.uint32))
    assert np.array_equal(scales.cpu().numpy().reshape(-1), s_ref)
    assert np.array_equal(packed.cpu().numpy().reshape(-1), p_ref)


def test_quantize_edge_values(F, torch):
    rows, cols = 4, 64
    w = np.zeros((rows, cols), np.float32)
    w[0, :16] = [0.0, -0.0, 1e-38, -1e-38, 6.0, -6.0, 3.0, 5.0, 2.5, 1.75, 0.25, 0.75, 1e-7, -1e-7, 7.0, -7.0]
    w[1, :] = np.linspace(-1, 1, cols)
    w[2, 5] = 1e30
    w[3, :] = -0.0
    t = torch.from_numpy(w).cuda()
    packed, scales, g = F.quantize_nvfp4(t, 1)
    p_ref, s_ref, g_ref = O.nvfp4_quantize(w, 1)
    assert np.array_equal(g.cpu().numpy().view(np.uint32), g_ref.view(np.uint32))
    assert np.array_equal(scales.cpu().numpy().reshape(-1), s_ref)
    assert np.array_equal(packed.cpu().numpy().reshape(-1), p_ref)


def _boundary_blocks(rows: int, cols: int, seed: int) -> np.ndarray:
    """Blocks whose quotients v / d land exactly on every e2m1 rounding
    boundary (ties), and one representable value either side of it.  With
    global = 2^-6 (amax 42 = 2688 * 2^-6) and a block maximum of 6 * d for an
    e4m3 value S = d / global, the block's factor is S and d = S * 2^-6 is
    exact, so m * d is exact for every boundary m."""
    rng = np.random.default_rng(seed)
    s_vals = np.array([0.5, 0.75, 1.0, 1.125, 1.75, 3.0, 6.5, 13.0, 0.015625, 0.0234375, 240.0], np.float32)
    marks = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 0.5, 1.0, 3.0], np.float32)
    w = np.zeros((rows, cols), np.float32)
    for r in range(rows):
        for b in range(cols // 16):
            d = np.float32(rng.choice(s_vals)) * np.float32(2.0 ** -6)
            blk = np.empty(16, np.float32)
            blk[0] = np.float32(6.0) * d
            for i in range(1, 16):
                v = np.float32(rng.choice(marks)) * d
                step = rng.integers(-1, 2)  # below, on, above the boundary
                if step:
                    v = np.nextafter(v, np.float32(np.inf) if step > 0 else np.float32(0))
                blk[i] = -v if rng.random() < 0.3 else v
            w[r, b * 16:(b + 1) * 16] = blk
    w[0, 0] = np.float32(42.0)  # amax: global = 2^-6 exactly (its block: S = 448)
    return w


def test_quantize_rounding_boundaries(F, torch):
    """Weights and activations whose quotients sit on or next to the e2m1
    rounding boundaries: the device's shortcut (one reciprocal per group,
    correctly rounded division only near a boundary) must give the oracle's
    codes bit for bit."""
    w = _boundary_blocks(64, 256, seed=3)
    packed, scales, g = F.quantize_nvfp4(torch.from_numpy(w).cuda())
    p_ref, s_ref, g_ref = O.nvfp4_quantize(w)
    assert g_ref[0] == np.float32(2.0 ** -6)
    assert np.array_equal(g.cpu().numpy().view(np.uint32), g_ref.view(np.uint32))
    assert np.array_equal(scales.cpu().numpy().reshape(-1), s_ref)
    assert np.array_equal(packed.cpu().numpy().reshape(-1), p_ref)
    a_packed, a_sf, a_g = F.quantize_act(torch.from_numpy(w).cuda())
    assert a_g.item() == g_ref[0]
    assert np.array_equal(a_packed.cpu().numpy().reshape(-1), p_ref)


def test_dequantize_bit_exact_and_roundtrip(F, torch):
    packed, scales, g, rows, cols = R.kernels_case(1, 29)[:5]
    m = host_matrix(F, packed, scales, g, rows, cols).upload()
    dq = m.dequantize().cpu().numpy()
    ref = O.nvfp4_dequantize(packed, scales, g, rows, cols)
    assert np.array_equal(dq.view(np.uint32), ref.view(np.uint32))
    back = m.to_host()
    assert np.array_equal(back.packed, packed) and np.array_equal(back.scales, scales)


def test_create_rejects_bad_formats(F, torch):
    rows, cols = 2, 64
    bad = np.zeros(rows * cols // 16, np.uint8)
    bad[3] = 0x7F
    with pytest.raises(F.FpbError) as e:
        host_matrix(F, np.zeros(rows * cols // 2), bad, [1.0, 1.0], rows, cols).upload()
    assert e.value.status == 3
    dev = torch.zeros(rows * cols // 2, dtype=torch.uint8, device="cuda")
    sc = torch.from_numpy(bad).cuda()
    with pytest.raises(F.FpbError):
        F.Nvfp4Matrix.from_device(dev, sc, torch.ones(rows, device="cuda"), rows, cols)
    with pytest.raises(F.FpbError):
        F.Nvfp4Matrix.from_device(dev, torch.zeros_like(sc), torch.tensor([1.0, float("inf")], device="cuda"),
                                  rows, cols)


# ---- GEMV: the reference's own cases ----------------------------------------------------------
def _gemv(F, torch, m, x, batch, x_dtype=None, y_dtype=None, rows=None):
    x_dtype = x_dtype or torch.float32
    y_dtype = y_dtype or torch.float32
    n = m.rows if rows is None else len(rows)
    xt = torch.from_numpy(np.ascontiguousarray(x, np.float32).reshape(batch, m.cols)).cuda().to(x_dtype)
    y = torch.full((batch, n), float("nan"), dtype=y_dtype, device="cuda")
    F.gemv(m, xt, y, F.GemvTile(1, 1), rows=rows).submit(F.Eager())
    return y.float().cpu().numpy()


@pytest.mark.parametrize("k_blocks", [0, 1])
@pytest.mark.parametrize("seed", R.SEEDS)
def test_reference_cases_dense_and_expert(F, torch, k_blocks, seed):
    """nvfp4_kernels_match_dequantized_f64_oracle (nvfp4_oracle.rs:241-267)."""
    packed, scales, g, rows, cols, x, selected = R.kernels_case(k_blocks, seed)
    m = host_matrix(F, packed, scales, g, rows, cols).upload()
    expected, magnitude = O.nvfp4_gemv_f64(packed, scales, g, rows, cols, x)
    assert np.all(np.isfinite(expected))
    y = _gemv(F, torch, m, x, 1)
    assert O.inner_product_excess(y, expected, magnitude, cols + 2) <= 1.0
    # expert GEMV: experts of 128 rows, the selected one, input_stride 0
    dims = F.MoeDims.new(cols, R.PART_ROWS, R.PART_ROWS, 2, 1)
    sel = F.ExpertSelection.parse([selected], [1.0], dims)
    xt = torch.from_numpy(x.reshape(1, cols)).cuda()
    ye = torch.full((1, R.PART_ROWS), float("nan"), device="cuda")
    F.expert_gemv_weight_view(m, xt, sel, ye, R.PART_ROWS, 0).submit(F.Eager())
    part = slice(selected * R.PART_ROWS, (selected + 1) * R.PART_ROWS)
    assert O.inner_product_excess(ye.cpu().numpy(), expected[0, part], magnitude[0, part], cols + 2) <= 1.0


@pytest.mark.parametrize("case", [0, 1, 2])
@pytest.mark.parametrize("seed", R.SEEDS[:6])
def test_reference_extreme_cases(F, torch, case, seed):
    """nvfp4_extreme_finite_values_match_f64_oracle (nvfp4_oracle.rs:269-321)."""
    packed, scales, g, rows, cols, x, selected = R.extreme_case(case, seed)
    m = host_matrix(F, packed, scales, g, rows, cols).upload()
    expected, magnitude = O.nvfp4_gemv_f64(packed, scales, g, rows, cols, x)
    assert np.all(np.isfinite(expected))
    y = _gemv(F, torch, m, x, 1)
    assert np.all(np.isfinite(y))
    assert O.inner_product_excess(y, expected, magnitude, cols + 2) <= 1.0


# ---- GEMV: shapes, dtypes, batches ---------------------------------------------------------
def _synthetic(F, torch, rows, cols, seed=0, rpg=None):
    w = F.synth_normal((rows, cols), seed=seed, stream_id=1, std=0.02)
    m = F.Nvfp4Matrix.quantize(w, rpg)
    h = m.to_host()
    return m, h


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (8192, 2048), (1000, 512), (24, 96), (130, 2080),
                                       (7, 32), (2048, 4000), (8192, 4096), (20000, 512), (1002, 1024)])
@pytest.mark.parametrize("batch", [1, 3, 8, 16])
def test_gemv_shapes_batches(F, torch, rows, cols, batch):
    m, h = _synthetic(F, torch, rows, cols, seed=rows * 7 + cols)
    x = O.synth_normal(batch * cols, seed=batch, stream=2).reshape(batch, cols)
    xb = O.bf16_to_f32(O.bf16_bits(x)).reshape(batch, cols)  # the values the bf16 kernel sees
    y_ref = O.nvfp4_gemv_f32(h.packed, h.scales, h.row_scales, rows, cols, xb)
    e64, mag = O.nvfp4_gemv_f64(h.packed, h.scales, h.row_scales, rows, cols, xb)
    y = _gemv(F, torch, m, xb, batch, x_dtype=torch.bfloat16)
    assert O.rel_frobenius(y, y_ref) <= REL_FROB_TOL
    assert O.inner_product_excess(y, e64, mag, cols + 2) <= 1.0
    y32 = _gemv(F, torch, m, x, batch, x_dtype=torch.float32)
    e64, mag = O.nvfp4_gemv_f64(h.packed, h.scales, h.row_scales, rows, cols, x)
    assert O.inner_product_excess(y32, e64, mag, cols + 2) <= 1.0


def test_gemv_bf16_output_and_row_range(F, torch):
    rows, cols = 4096, 4096
    m, h = _synthetic(F, torch, rows, cols, seed=5)
    x = O.bf16_to_f32(O.bf16_bits(O.synth_normal(cols, seed=0, stream=0)))
    y_ref = O.nvfp4_gemv_f32(h.packed, h.scales, h.row_scales, rows, cols, x)[0]
    yb = _gemv(F, torch, m, x, 1, x_dtype=torch.bfloat16, y_dtype=torch.bfloat16)[0]
    assert np.array_equal(O.bf16_bits(yb), yb.astype(np.float32).view(np.uint32).__rshift__(16).astype(np.uint16))
    assert O.rel_frobenius(yb, y_ref) <= 4e-3  # bf16 output rounding (2^-9) dominates
    sub = _gemv(F, torch, m, x, 1, x_dtype=torch.bfloat16, rows=range(1000, 3000))[0]
    assert O.rel_frobenius(sub, y_ref[1000:3000]) <= REL_FROB_TOL


def test_config0_full_size(F, torch):
    """x bf16 [1,4096] N(0,1) seed 0, W [4096,4096] N(0,0.02) -> NVFP4, y bf16."""
    rows = cols = 4096
    w = F.synth_normal((rows, cols), seed=0, stream_id=1, std=0.02)
    m = F.Nvfp4Matrix.quantize(w)
    h = m.to_host()
    p_ref, s_ref, g_ref = O.nvfp4_quantize(w.cpu().numpy())
    assert np.array_equal(h.packed, p_ref) and np.array_equal(h.scales, s_ref)
    x = F.synth_normal((1, cols), seed=0, stream_id=0, dtype=torch.bfloat16)
    xf = x.float().cpu().numpy()
    y = torch.empty(1, rows, dtype=torch.bfloat16, device="cuda")
    F.gemv(m, x, y).submit(F.Eager())
    y_ref = O.nvfp4_gemv_f32(p_ref, s_ref, g_ref, rows, cols, xf)
    assert O.rel_frobenius(y.float().cpu().numpy(), y_ref) <= 4e-3
    y32 = torch.empty(1, rows, dtype=torch.float32, device="cuda")
    F.gemv(m, x, y32).submit(F.Eager())
    assert O.rel_frobenius(y32.cpu().numpy(), y_ref) <= REL_FROB_TOL
    e64, mag = O.nvfp4_gemv_f64(p_ref, s_ref, g_ref, rows, cols, xf)
    assert O.inner_product_excess(y32.cpu().numpy(), e64, mag, cols + 2) <= 1.0


def test_expert_gemv_slots_and_strides(F, torch):
    experts, rpe, cols = 9, 1024, 2048
    m, h = _synthetic(F, torch, experts * rpe, cols, seed=11, rpg=rpe)
    ids = np.array([3, 0, 8, 5, 1], np.int32)
    x = O.bf16_to_f32(O.bf16_bits(O.synth_normal(len(ids) * cols, seed=4, stream=2))).reshape(len(ids), cols)
    for stride in (0, 1):
        y_ref = O.nvfp4_expert_gemv_f32(h.packed, h.scales, h.row_scales, cols, ids, rpe, stride, x)
        xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
        y = torch.full((len(ids), rpe), float("nan"), device="cuda")
        dims = F.MoeDims.new(cols, 512, 512, experts, len(ids))
        sel = F.ExpertSelection.parse(ids, np.full(len(ids), 0.2, np.float32), dims)
        F.expert_gemv_weight_view(m, xt, sel, y, rpe, stride).submit(F.Eager())
        assert O.rel_frobenius(y.cpu().numpy(), y_ref) <= REL_FROB_TOL


def test_gemv_errors_are_statuses(F, torch):
    m, _ = _synthetic(F, torch, 64, 128)
    x = torch.zeros(1, 128, device="cuda")
    y = torch.zeros(1, 64, device="cuda")
    from firepit_b200 import _native as N
    st = N.lib.fpb_nvfp4_gemv(m.handle, 10, 5, x.data_ptr(), 0, y.data_ptr(), 0, 1, None)
    assert st == N.FPB_ERR_SHAPE
    st = N.lib.fpb_nvfp4_gemv(m.handle, 0, 0, x.data_ptr(), 0, y.data_ptr(), 0, 17, None)
    assert st == N.FPB_ERR_SHAPE
    st = N.lib.fpb_nvfp4_gemv(m.handle, 0, 65, x.data_ptr(), 0, y.data_ptr(), 0, 1, None)
    assert st == N.FPB_ERR_SHAPE
    with pytest.raises(F.ShapeError):
        F.gemv(m, torch.zeros(1, 96, device="cuda"), y)
    big, _ = _synthetic(F, torch, 32, 8192)
    xb = torch.zeros(1, 8192, device="cuda")
    # K > 4096 adds the K slices' sums in y, so it needs an f32 y
    st = N.lib.fpb_nvfp4_gemv(big.handle, 0, 0, xb.data_ptr(), 0, y.data_ptr(), N.FPB_BF16, 1, None)
    assert st == N.FPB_ERR_UNSUPPORTED
    torch.cuda.synchronize()


@pytest.mark.parametrize("rows,cols", [(512, 8192), (256, 4128), (128, 12288)])
@pytest.mark.parametrize("batch", [1, 5])
@pytest.mark.parametrize("xdt", ["bf16", "f32"])
def test_gemv_long_rows(F, torch, rows, cols, batch, xdt):
    """K > 4096 (the reference loops any K that is a multiple of 32,
    gemv/nvfp4.rs:34): consecutive 4096-column slices add into f32 y."""
    m, h = _synthetic(F, torch, rows, cols, seed=cols)
    x = O.synth_normal(batch * cols, seed=batch, stream=2).reshape(batch, cols)
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16 if xdt == "bf16" else torch.float32)
    xf = xt.float().cpu().numpy()
    y = torch.full((batch, rows), float("nan"), device="cuda")
    F.gemv(m, xt, y, F.GemvTile(16, 1)).submit(F.Eager())  # 4128 = 129 blocks of 32
    ref = O.nvfp4_gemv_f32(h.packed, h.scales, h.row_scales, rows, cols, xf)
    assert O.rel_frobenius(y.cpu().numpy(), ref) <= REL_FROB_TOL
    e64, mag = O.nvfp4_gemv_f64(h.packed, h.scales, h.row_scales, rows, cols, xf)
    assert O.inner_product_excess(y.cpu().numpy(), e64, mag, cols + 2) <= 1.0


def test_expert_gemv_long_rows(F, torch):
    experts, rpe, cols = 4, 256, 6144
    m, h = _synthetic(F, torch, experts * rpe, cols, seed=17, rpg=rpe)
    ids = np.array([2, 0, 3], np.int32)
    x = O.bf16_to_f32(O.bf16_bits(O.synth_normal(len(ids) * cols, seed=6, stream=2))).reshape(len(ids), cols)
    y_ref = O.nvfp4_expert_gemv_f32(h.packed, h.scales, h.row_scales, cols, ids, rpe, 1, x)
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y = torch.full((len(ids), rpe), float("nan"), device="cuda")
    dims = F.MoeDims.new(2048, 512, 512, experts, len(ids))
    sel = F.ExpertSelection.parse(ids, np.full(len(ids), 0.2, np.float32), dims)
    F.expert_gemv_weight_view(m, xt, sel, y, rpe, 1).submit(F.Eager())
    assert O.rel_frobenius(y.cpu().numpy(), y_ref) <= REL_FROB_TOL
