"""The reference's activation semantics for the prefill GEMMs (act="hilo").

nvfp4_gemm (gemm/nvfp4.rs:33-50) and fp8_gemm (gemm/mod.rs:87-100, 155-168)
keep the activations in f32 and multiply their bf16 hi and lo halves by the
weights in bf16, accumulating in f32.  Checked against the f64 product of the
f32 activations and the dequantized weights: relative Frobenius <= 1e-3 and,
per element, |y - y64| <= (gamma_{K+2} + 2^-15) * sum |x| |w| (hi + lo holds x
to 2^-16; gamma covers the f32 accumulation).
"""
import numpy as np
import pytest

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


def _bound(k):
    u = 2.0 ** -24
    return (k + 2) * u / (1 - (k + 2) * u) + 2.0 ** -15


def _check(got, x64, wd, k):
    exp = x64 @ wd.T
    mag = np.abs(x64) @ np.abs(wd).T
    got = got.astype(np.float64)
    assert np.all(np.isfinite(got))
    assert O.rel_frobenius(got, exp) <= REL_FROB_TOL
    assert np.all(np.abs(got - exp) <= _bound(k) * mag + 1e-30)


@pytest.mark.parametrize("m,n,k,rows", [(128, 256, 512, None), (200, 384, 2048, (100, 356)), (64, 128, 96, None),
                                        (2048, 8192, 2048, None), (1, 8192, 2048, None)])
@pytest.mark.parametrize("xdt", ["f32", "bf16"])
def test_nvfp4_gemm_hilo(F, torch, m, n, k, rows, xdt):
    w = F.synth_normal((n, k), seed=n + k, stream_id=1, std=0.02)
    W = F.Nvfp4Matrix.quantize(w)
    h = W.to_host()
    x = F.synth_normal((m, k), seed=m, stream_id=2)
    if xdt == "bf16":
        x = x.to(torch.bfloat16)
    r = range(*rows) if rows else range(0, n)
    y = torch.full((m, len(r)), float("nan"), device="cuda")
    F.nvfp4_gemm_view(W, r, x, y, F.GemmTile(1, 4, 32), act="hilo").submit(F.Eager())
    assert F.device_error() == 0
    wd = O.nvfp4_dequantize(h.packed, h.scales, h.row_scales, n, k).astype(np.float64)[r.start:r.stop]
    _check(y.cpu().numpy(), x.float().cpu().numpy().astype(np.float64), wd, k)


@pytest.mark.parametrize("block", [(128, 128), (64, 32), (0, 0)])
@pytest.mark.parametrize("xdt", ["f32", "bf16"])
def test_fp8_gemm_hilo(F, torch, block, xdt):
    m, n, k = 256, 1024, 1024
    w = F.synth_normal((n, k), seed=7, stream_id=1, std=0.02)
    W = F.Fp8Matrix.quantize(w, F.Fp8Scaling(*block))
    h = W.to_host()
    x = F.synth_normal((m, k), seed=8, stream_id=2)
    if xdt == "bf16":
        x = x.to(torch.bfloat16)
    y = torch.full((m, n), float("nan"), device="cuda")
    tile = F.GemmTile(1, 32 if block[0] else 128, 32)
    F.fp8_gemm(W, x, y, tile, act="hilo").submit(F.Eager())
    assert F.device_error() == 0
    if block == (0, 0):
        wd = O.fp8_dequantize(h.bits.reshape(n, k), h.scales, 0, 0)
    else:
        wd = O.fp8_dequantize(h.bits.reshape(n, k), h.scales.reshape(n // block[0], k // block[1]), *block)
    _check(y.cpu().numpy(), x.float().cpu().numpy().astype(np.float64), np.asarray(wd, np.float64).reshape(n, k), k)


def test_config1_fp8_hilo_full_size(F, torch):
    """BASELINE config 1 shapes (M=512, K=4096, N=14336, 128x128 blocks) with
    the reference's f32 activations."""
    m, n, k = 512, 14336, 4096
    w = F.synth_normal((n, k), seed=0, stream_id=1, std=0.02)
    W = F.Fp8Matrix.quantize(w, F.Fp8Scaling(128, 128))
    h = W.to_host()
    x = F.synth_normal((m, k), seed=0, stream_id=0)
    y = torch.full((m, n), float("nan"), device="cuda")
    F.fp8_gemm(W, x, y, act="hilo").submit(F.Eager())
    assert F.device_error() == 0
    rows = np.arange(0, n, 7)  # every 7th output column against f64 (2048 of them)
    wd = np.asarray(O.fp8_dequantize(h.bits.reshape(n, k)[rows], np.repeat(
        h.scales.reshape(n // 128, k // 128), 128, axis=0)[rows].reshape(-1), 1, 128), np.float64).reshape(-1, k)
    _check(y.cpu().numpy()[:, rows], x.cpu().numpy().astype(np.float64), wd, k)
