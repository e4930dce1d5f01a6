"""GPU parity of the FP8 E4M3 path against the CPU oracle.

* Quantizers (weights per 128x128 block or per row, activations per token)
  are bit-exact against the oracle.
* The tcgen05 FP8 GEMM quantizes its activations per token (the config-1
  W8A8 setting) and is compared with the f64 product of the same quantized
  operands: relative Frobenius error <= 1e-3 and, per element,
  |y - e| <= (gamma~(K+1) + 2^-16) * sum|a||w| (the reference's GEMM bound,
  fp8_oracle.rs:28-31, with the bf16 split term of its hi/lo method replaced by
  2^-16), on the reference's own deterministic and extreme cases
  (fp8_oracle.rs:119-300) and on seeded normal data up to config-1 size.
"""
import numpy as np
import pytest

import refcases as R
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


def _check(got, a_bits, a_s, w_bits, w_s, bn, bk, k, out_bf16=False, frobenius=True):
    e, mag = O.fp8_gemm_f64(a_bits, a_s, w_bits, w_s, bn, bk)
    got = got.astype(np.float64)
    assert np.all(np.isfinite(got))
    if not frobenius:  # cancelling extreme cases: the per-element bound only, as the reference checks them
        assert np.all(np.abs(got - e) <= (O.gamma_tilde(k + 1) + 2.0 ** -16) * mag + 1e-300)
        return
    if out_bf16:
        eb = O.bf16_to_f32(O.bf16_bits(e.astype(np.float32))).astype(np.float64)
        assert O.rel_frobenius(got, eb) <= REL_FROB_TOL
        bound = 2.0 ** -8 * np.abs(e) + (O.gamma_tilde(k + 1) + 2.0 ** -16) * mag
    else:
        assert O.rel_frobenius(got, e) <= REL_FROB_TOL
        bound = (O.gamma_tilde(k + 1) + 2.0 ** -16) * mag
    assert np.all(np.abs(got - e) <= bound + 1e-300)


@pytest.mark.parametrize("rows,cols,block", [(256, 384, (128, 128)), (384, 256, (0, 0)), (100, 4096, (0, 0)),
                                             (512, 1024, (256, 128))])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_fp8_quantize_bit_exact(F, torch, rows, cols, block, dtype):
    w = F.synth_normal((rows, cols), seed=rows + cols, stream_id=4, std=0.02 if block != (0, 0) else 1.0)
    if dtype == "bf16":
        w = w.to(torch.bfloat16)
    bits, scales = F.quantize_fp8(w, F.Fp8Scaling(*block))
    rb, rs = O.fp8_quantize(w.float().cpu().numpy(), *block)
    assert np.array_equal(bits.cpu().numpy(), rb)
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), rs.view(np.uint32))


def _gemm_ref_case(F, torch, bits, scales, x_row, rows, cols, bn, bk, frobenius=True):
    m = 64
    W = (F.HostFp8Matrix.from_parts(bits, scales, rows, cols, bn, bk) if bn else
         F.HostFp8Matrix.with_row_scales(bits, scales, rows, cols)).upload()
    x = np.tile(x_row, (m, 1)).astype(np.float32)
    y = torch.full((m, rows), float("nan"), device="cuda")
    F.fp8_gemm(W, torch.from_numpy(x).cuda(), y, F.GemmTile(64, 128, 32)).submit(F.Eager())
    assert F.device_error() == 0
    a_bits, a_s = O.fp8_quantize(x)
    _check(y.cpu().numpy(), a_bits, a_s, bits, scales, bn, bk, cols, frobenius=frobenius)


@pytest.mark.parametrize("n_blocks,k_blocks", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("seed", R.SEEDS[:8])
def test_fp8_gemm_reference_cases(F, torch, n_blocks, k_blocks, seed):
    bits, scales, x, rows, cols = R.fp8_kernels_case(n_blocks, k_blocks, seed)
    _gemm_ref_case(F, torch, bits, scales, x, rows, cols, 128, 128)


@pytest.mark.parametrize("case", [0, 1, 2])
@pytest.mark.parametrize("seed", R.SEEDS[:6])
def test_fp8_gemm_extreme_cases(F, torch, case, seed):
    bits, scales, x, rows, cols = R.fp8_extreme_case(case, seed)
    _gemm_ref_case(F, torch, bits, scales, x, rows, cols, 128, 128, frobenius=False)


@pytest.mark.parametrize("m,n,k,block", [(128, 128, 128, (128, 128)), (200, 384, 1024, (128, 128)),
                                         (64, 256, 4096, (0, 0)), (300, 512, 2080, (0, 0)),
                                         (256, 512, 1024, (256, 128)), (512, 1024, 4096, (128, 128))])
@pytest.mark.parametrize("out", ["f32", "bf16"])
def test_fp8_gemm_synthetic(F, torch, m, n, k, block, out):
    w = F.synth_normal((n, k), seed=n + k, stream_id=1, std=0.02)
    W = F.Fp8Matrix.quantize(w, F.Fp8Scaling(*block))
    h = W.to_host()
    x = F.synth_normal((m, k), seed=m, stream_id=2, dtype=torch.bfloat16)
    ydt = torch.bfloat16 if out == "bf16" else torch.float32
    y = torch.full((m, n), float("nan"), dtype=ydt, device="cuda")
    tile = F.GemmTile(m if m % 64 else 64, 128, 32)
    F.fp8_gemm(W, x, y, tile).submit(F.Eager())
    assert F.device_error() == 0
    a_bits, a_s = O.fp8_quantize(x.float().cpu().numpy())
    _check(y.float().cpu().numpy(), a_bits, a_s, h.bits.reshape(n, k), h.scales, *block, k, out_bf16=out == "bf16")


def test_fp8_gemm_config1_full_size(F, torch):
    """Config 1: A [512, 4096] N(0,1) per-token e4m3, W [14336, 4096] N(0,0.02)
    128x128 blocks, y bf16.  The oracle checks 64 of the 512 rows."""
    m, n, k = 512, 14336, 4096
    w = F.synth_normal((n, k), seed=0, stream_id=1, std=0.02)
    W = F.Fp8Matrix.quantize(w, F.Fp8Scaling(128, 128))
    h = W.to_host()
    x = F.synth_normal((m, k), seed=0, stream_id=0, dtype=torch.bfloat16)
    y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    F.fp8_gemm(W, x, y).submit(F.Eager())
    assert F.device_error() == 0
    rows = np.arange(0, m, 8)
    a_bits, a_s = O.fp8_quantize(x.float().cpu().numpy())
    _check(y.float().cpu().numpy()[rows], a_bits[rows], a_s[rows], h.bits.reshape(n, k), h.scales, 128, 128, k,
           out_bf16=True)


@pytest.mark.parametrize("out", ["f32", "bf16"])
def test_fp8_gemm_persistent_ragged(F, torch, out):
    """168 tiles of 128 x 256 on 148 persistent CTAs (20 run a second tile),
    a ragged last row tile, TMA-stored output.  Checked against the oracle on
    a row sample, and bit for bit between two runs."""
    m, n, k = 300, 14336, 4096
    w = F.synth_normal((n, k), seed=5, stream_id=1, std=0.02)
    W = F.Fp8Matrix.quantize(w, F.Fp8Scaling(128, 128))
    h = W.to_host()
    x = F.synth_normal((m, k), seed=6, stream_id=2, dtype=torch.bfloat16)
    ydt = torch.bfloat16 if out == "bf16" else torch.float32
    ys = []
    for _ in range(2):
        y = torch.full((m, n), float("nan"), dtype=ydt, device="cuda")
        F.fp8_gemm(W, x, y, F.GemmTile(m, 128, 32)).submit(F.Eager())
        assert F.device_error() == 0
        ys.append(y)
    assert torch.equal(ys[0].view(torch.int16 if out == "bf16" else torch.int32),
                       ys[1].view(torch.int16 if out == "bf16" else torch.int32))
    rows = np.concatenate([np.arange(0, m, 9), np.arange(m - 4, m)])
    a_bits, a_s = O.fp8_quantize(x.float().cpu().numpy())
    _check(ys[0].float().cpu().numpy()[rows], a_bits[rows], a_s[rows], h.bits.reshape(n, k), h.scales, 128, 128, k,
           out_bf16=out == "bf16")


def test_fp8_gemm_view_and_errors(F, torch):
    n, k = 1024, 512
    w = F.synth_normal((n, k), seed=3, stream_id=1, std=0.02)
    W = F.Fp8Matrix.quantize(w, F.Fp8Scaling(128, 128))
    h = W.to_host()
    x = F.synth_normal((128, k), seed=4, stream_id=2)
    y = torch.full((128, 384), float("nan"), device="cuda")
    F.fp8_gemm_view(W, range(256, 640), x, y).submit(F.Eager())
    a_bits, a_s = O.fp8_quantize(x.cpu().numpy())
    wb = h.bits.reshape(n, k)[256:640]
    ws = h.scales.reshape(n // 128, k // 128)[2:5].reshape(-1)
    _check(y.cpu().numpy(), a_bits, a_s, wb, ws, 128, 128, k)
    with pytest.raises(F.ShapeError):  # rows not aligned to block_n (gemm/mod.rs:596-599)
        F.fp8_gemm_view(W, range(64, 192), x, torch.empty(128, 128, device="cuda"))
    W64 = F.Fp8Matrix.quantize(w, F.Fp8Scaling(64, 64))
    with pytest.raises(F.FpbError) as e:  # valid for the reference's tiles, not for the 128-wide tensor-core tile
        F.fp8_gemm(W64, x, torch.empty(128, n, device="cuda"), F.GemmTile(64, 64, 32)).submit(F.Eager())
    assert e.value.status == F._native.FPB_ERR_UNSUPPORTED


@pytest.mark.parametrize("block", [(128, 128), (0, 0)])
def test_fp8_grouped_gemm(F, torch, block):
    experts, rpe, k, tokens, top_k = 4, 256, 512, 150, 2
    dims = F.MoeDims.new(256, 128, 128, experts, top_k)
    rng = np.random.default_rng(9)
    idx = np.stack([rng.choice(experts, top_k, replace=False) for _ in range(tokens)]).astype(np.int32)
    layout = F.PrefillLayout.from_indices(idx, dims, 128)
    w = F.synth_normal((experts * rpe, k), seed=5, stream_id=1, std=0.02)
    W = F.Fp8Matrix.quantize(w, F.Fp8Scaling(*block))
    h = W.to_host()
    x_tok = F.synth_normal((tokens, k), seed=6, stream_id=2)
    rows = torch.from_numpy(layout.token_rows.astype(np.int64)).cuda()
    x = torch.where((rows >= 0)[:, None], x_tok[rows.clamp(min=0)], torch.zeros((), device="cuda"))
    y = torch.full((layout.padded_rows(), rpe), float("nan"), device="cuda")
    F.fp8_grouped_gemm_view(W, x, y, layout, experts, rpe).submit(F.Eager())
    assert F.device_error() == 0
    got = y.cpu().numpy()
    a_bits, a_s = O.fp8_quantize(x.cpu().numpy())
    wb = h.bits.reshape(experts * rpe, k)
    for t, e in enumerate(layout.tile_experts):
        sl = slice(t * 128, (t + 1) * 128)
        ws = h.scales if block == (0, 0) else h.scales.reshape(-1, k // 128)
        ws_e = ws[e * rpe:(e + 1) * rpe] if block == (0, 0) else ws[e * rpe // 128:(e + 1) * rpe // 128].reshape(-1)
        _check(got[sl], a_bits[sl], a_s[sl], wb[e * rpe:(e + 1) * rpe], ws_e, *block, k)
    assert np.all(got[layout.token_rows < 0] == 0.0)


# ---- decode GEMV on FP8 weights (gemv/fp8.rs) -----------------------------------------
def _fp8_gemv_expected(h, rows, cols, block, x):
    """f64 product of the dequantized weights (e4m3 x scale in f32, the
    reference's dequant) with x, and the magnitudes |W| |x| for the bound."""
    if block == (0, 0):
        wd = O.fp8_dequantize(h.bits.reshape(rows, cols), h.scales, 0, 0)
    else:
        wd = O.fp8_dequantize(h.bits.reshape(rows, cols), h.scales.reshape(rows // block[0], cols // block[1]),
                              *block)
    wd = np.asarray(wd, np.float64).reshape(rows, cols)
    return x.astype(np.float64) @ wd.T, np.abs(x.astype(np.float64)) @ np.abs(wd).T


@pytest.mark.parametrize("rows,cols,block", [(4096, 4096, (128, 128)), (1024, 2048, (0, 0)),
                                             (512, 1536, (256, 128)), (96, 96 * 4, (0, 0))])
@pytest.mark.parametrize("batch", [1, 3, 8, 16])
@pytest.mark.parametrize("xdt", ["bf16", "f32"])
def test_fp8_gemv_dense(F, torch, rows, cols, block, batch, xdt):
    """gemv(&Weight::Fp8, ...) (gemv/fp8.rs:186-246) against the f64 product
    of the dequantized weights: the inner-product error bound and the
    relative Frobenius tolerance."""
    w = F.synth_normal((rows, cols), seed=rows + cols, stream_id=1, std=0.02)
    W = F.Fp8Matrix.quantize(w, F.Fp8Scaling(*block))
    h = W.to_host()
    x = O.synth_normal(batch * cols, seed=batch, stream=2).reshape(batch, cols).astype(np.float32)
    if xdt == "bf16":
        x = O.bf16_to_f32(O.bf16_bits(x)).reshape(batch, cols)
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16 if xdt == "bf16" else torch.float32)
    y = torch.full((batch, rows), float("nan"), device="cuda")
    tile = F.GemvTile(16 if rows % 16 == 0 else 8, 4 if cols % 128 == 0 else 1)
    F.gemv(W, xt, y, tile).submit(F.Eager())
    e, mag = _fp8_gemv_expected(h, rows, cols, block, x)
    got = y.cpu().numpy()
    assert O.rel_frobenius(got, e) <= REL_FROB_TOL
    assert O.inner_product_excess(got, e, mag, cols + 2) <= 1.0


def test_fp8_gemv_row_range_and_bf16_out(F, torch):
    rows, cols = 2048, 4096
    w = F.synth_normal((rows, cols), seed=9, stream_id=1, std=0.02)
    W = F.Fp8Matrix.quantize(w, F.Fp8Scaling(128, 128))
    h = W.to_host()
    x = O.bf16_to_f32(O.bf16_bits(O.synth_normal(cols, seed=0, stream=0))).reshape(1, cols)
    e, mag = _fp8_gemv_expected(h, rows, cols, (128, 128), x)
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y = torch.full((1, 768), float("nan"), device="cuda")
    F.gemv(W, xt, y, rows=range(256, 1024)).submit(F.Eager())
    assert O.inner_product_excess(y.cpu().numpy(), e[:, 256:1024], mag[:, 256:1024], cols + 2) <= 1.0
    yb = torch.full((1, rows), float("nan"), dtype=torch.bfloat16, device="cuda")
    F.gemv(W, xt, yb).submit(F.Eager())
    assert O.rel_frobenius(yb.float().cpu().numpy(), e) <= 4e-3  # bf16 output rounding


@pytest.mark.parametrize("block", [(128, 128), (0, 0)])
def test_fp8_expert_gemv(F, torch, block):
    """expert_gemv_weight_view(&Weight::Fp8, ...) (gemv/fp8.rs:248-281): x row
    s * input_stride, weight rows of expert ids[s]."""
    experts, rpe, cols = 6, 512, 2048
    w = F.synth_normal((experts * rpe, cols), seed=13, stream_id=1, std=0.02)
    W = F.Fp8Matrix.quantize(w, F.Fp8Scaling(*block))
    h = W.to_host()
    ids = np.array([3, 0, 5, 2, 1], np.int32)
    x = O.bf16_to_f32(O.bf16_bits(O.synth_normal(len(ids) * cols, seed=4, stream=2))).reshape(len(ids), cols)
    e_all, mag_all = _fp8_gemv_expected(h, experts * rpe, cols, block, x)
    for stride in (0, 1):
        xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
        y = torch.full((len(ids), rpe), float("nan"), device="cuda")
        dims = F.MoeDims.new(cols, 512, 512, experts, len(ids))
        sel = F.ExpertSelection.parse(ids, np.full(len(ids), 0.2, np.float32), dims)
        F.expert_gemv_weight_view(W, xt, sel, y, rpe, stride).submit(F.Eager())
        got = y.cpu().numpy()
        for s, e in enumerate(ids):
            xr = s * stride
            rows = slice(e * rpe, (e + 1) * rpe)
            assert O.inner_product_excess(got[s:s + 1], e_all[xr:xr + 1, rows], mag_all[xr:xr + 1, rows],
                                          cols + 2) <= 1.0


def test_fp8_gemv_errors(F, torch):
    from firepit_b200 import _native as N
    W = F.Fp8Matrix.quantize(F.synth_normal((256, 256), seed=1, stream_id=1, std=0.02), F.Fp8Scaling(128, 128))
    x = torch.zeros(1, 256, device="cuda")
    y = torch.zeros(1, 256, device="cuda")
    assert N.lib.fpb_fp8_gemv(W.handle, 10, 5, x.data_ptr(), 0, y.data_ptr(), 0, 1, None) == N.FPB_ERR_SHAPE
    assert N.lib.fpb_fp8_gemv(W.handle, 0, 0, x.data_ptr(), 0, y.data_ptr(), 0, 17, None) == N.FPB_ERR_SHAPE
    assert N.lib.fpb_fp8_gemv(W.handle, 0, 257, x.data_ptr(), 0, y.data_ptr(), 0, 1, None) == N.FPB_ERR_SHAPE
    assert N.lib.fpb_fp8_expert_gemv(W.handle, x.data_ptr(), 0, None, 1, 128, 0, y.data_ptr(), 0,
                                     None) == N.FPB_ERR_INVALID_ARGUMENT
    ids = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert N.lib.fpb_fp8_expert_gemv(W.handle, x.data_ptr(), 0, ids.data_ptr(), 1, 64, 0, y.data_ptr(), 0,
                                     None) == N.FPB_ERR_SHAPE  # 64 rows per expert, block_n 128
    with pytest.raises(F.ShapeError):
        F.gemv(W, x, y, F.GemvTile(256, 4))  # a tile taller than the 128-row scale block
