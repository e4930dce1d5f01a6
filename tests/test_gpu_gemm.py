"""GPU parity of the tcgen05 NVFP4 GEMM against the CPU oracle.

Activations are quantized to NVFP4 on the device (bit-exact against the
oracle's quantizer); the GEMM output is compared with the f64 product of the
dequantized operands (the same quantized values): relative Frobenius error
<= 1e-3 (north star) and a per-element bound of 1e-5 * sum |a||w|.
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


def tiled_to_rowmajor(sf_tiled: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Inverse of the tensor-core factor layout (byte (r%32)*16 + (r%128)/32*4 + s of each 512-byte chunk)."""
    groups = cols // 16
    kb64 = (cols + 255) // 256 * 4
    r = np.arange(rows)[:, None]
    g = np.arange(groups)[None, :]
    off = ((r // 128) * kb64 + g // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + g % 4
    return sf_tiled[off]


def make_weight(F, rows, cols, seed):
    w = F.synth_normal((rows, cols), seed=seed, stream_id=1, std=0.02)
    m = F.Nvfp4Matrix.quantize(w)
    return m, m.to_host()


def expected_gemm(h, x_cpu: np.ndarray, rows: range):
    m, k = x_cpu.shape
    pa, sa, ga = O.nvfp4_quantize(x_cpu)  # one global for the whole activation tensor
    a = O.nvfp4_dequantize(pa, sa, ga, m, k).astype(np.float64)
    w = O.nvfp4_dequantize(h.packed, h.scales, h.row_scales, h.rows, h.cols)[rows.start:rows.stop].astype(np.float64)
    return a @ w.T, np.abs(a) @ np.abs(w).T


@pytest.mark.parametrize("m,k", [(128, 256), (200, 2048), (64, 96), (2048, 2048)])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_quantize_act_bit_exact(F, torch, m, k, dtype):
    x = F.synth_normal((m, k), seed=m + k, stream_id=3)
    if dtype == "bf16":
        x = x.to(torch.bfloat16)
    packed, sf, g = F.quantize_act(x)
    pa, sa, ga = O.nvfp4_quantize(x.float().cpu().numpy())
    assert np.array_equal(packed.cpu().numpy().reshape(-1), pa)
    assert g.cpu().numpy()[0] == ga[0]
    assert np.array_equal(tiled_to_rowmajor(sf.cpu().numpy(), m, k).reshape(-1), sa)


@pytest.mark.parametrize("m,n,k", [(128, 128, 256), (64, 256, 512), (200, 384, 2048), (256, 128, 96),
                                   (128, 8192, 2048), (2048, 8192, 2048)])
def test_gemm_vs_oracle(F, torch, m, n, k):
    W, h = make_weight(F, n, k, seed=n + k)
    x = F.synth_normal((m, k), seed=m, stream_id=2, dtype=torch.bfloat16)
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    F.nvfp4_gemm(W, x, y, F.GemmTile(8, 128, 32)).submit(F.Eager())
    assert F.device_error() == 0
    exp, mag = expected_gemm(h, x.float().cpu().numpy(), range(0, n))
    got = y.cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(got))
    assert O.rel_frobenius(got, exp) <= REL_FROB_TOL
    assert np.all(np.abs(got - exp) <= 1e-5 * mag + 1e-30)


@pytest.mark.parametrize("m,n,dtype", [(200, 200, "f32"), (130, 200, "bf16"), (130, 98, "bf16"), (77, 99, "f32"),
                                       (300, 520, "bf16")])
def test_gemm_ragged_output(F, torch, m, n, dtype):
    """Ragged M and N: tiled stores clipped at the edges (row pitch a multiple
    of 16 bytes) and direct stores (unaligned pitch, e.g. 98 bf16 columns)."""
    k = 512
    W, h = make_weight(F, n, k, seed=n + 7)
    x = F.synth_normal((m, k), seed=m + 1, stream_id=2, dtype=torch.bfloat16)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    y = torch.full((m + 1, n), float("nan"), dtype=tdt, device="cuda")  # one guard row past the output
    F.nvfp4_gemm(W, x, y[:m], F.GemmTile(1, 1, 32)).submit(F.Eager())
    assert F.device_error() == 0
    exp, mag = expected_gemm(h, x.float().cpu().numpy(), range(0, n))
    got = y[:m].float().cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(got))
    assert torch.isnan(y[m].float()).all()  # nothing written past the last row
    tol = 1e-5 if dtype == "f32" else 4e-3
    assert np.all(np.abs(got - exp) <= tol * mag + 1e-30)


def test_gemm_view_bf16_output(F, torch):
    W, h = make_weight(F, 512, 1024, seed=9)
    x = F.synth_normal((128, 1024), seed=4, stream_id=2, dtype=torch.bfloat16)
    y = torch.empty((128, 256), dtype=torch.bfloat16, device="cuda")
    F.nvfp4_gemm_view(W, range(128, 384), x, y).submit(F.Eager())
    exp, _ = expected_gemm(h, x.float().cpu().numpy(), range(128, 384))
    assert O.rel_frobenius(y.float().cpu().numpy(), exp) <= 4e-3  # bf16 output rounding
    with pytest.raises(F.FpbError):  # views must start on a 128-row boundary
        F.nvfp4_gemm_view(W, range(64, 192), x, torch.empty((128, 128), device="cuda")).submit(F.Eager())


def test_gemm_negative_block_scales(F, torch):
    rows, cols = 256, 512
    rng = np.random.default_rng(5)
    packed = rng.integers(0, 256, rows * cols // 2, dtype=np.uint8)
    scales = rng.choice(np.array([0x38, 0xB8, 0x30, 0xC0, 0x01, 0x81], np.uint8), rows * cols // 16)
    host = F.HostNvfp4Matrix(packed, scales, np.full(rows, 0.5, np.float32), rows, cols)
    W = host.upload()
    x = F.synth_normal((128, cols), seed=8, stream_id=2, dtype=torch.bfloat16)
    y = torch.empty((128, rows), device="cuda")
    F.nvfp4_gemm(W, x, y).submit(F.Eager())
    exp, _ = expected_gemm(host, x.float().cpu().numpy(), range(0, rows))
    assert O.rel_frobenius(y.cpu().numpy(), exp) <= REL_FROB_TOL


def test_first_gemm_call_on_fresh_handle_recorded_in_graph(F, torch):
    """The GEMM-side copies are built when the handle is created, so the very
    first GEMM (and GEMV) call on a fresh handle can be recorded by the
    reference's Graph sink (sink.rs:94-105): nothing allocates or
    synchronises inside the calls."""
    m, n, k = 256, 1024, 2048
    w = F.synth_normal((n, k), seed=77, stream_id=1, std=0.02)
    packed, scales, g = F.quantize_nvfp4(w)
    h = F.HostNvfp4Matrix(packed.cpu().numpy(), scales.cpu().numpy(), g.cpu().numpy(), n, k)
    W = h.upload()  # fresh handle: no GEMM has run on it
    x = F.synth_normal((m, k), seed=5, stream_id=2, dtype=torch.bfloat16)
    ws = torch.empty(int(F._native.lib.fpb_nvfp4_gemm_workspace_bytes(m, k)), dtype=torch.uint8, device="cuda")
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    yv = torch.full((1, n), float("nan"), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    sink = F.Graph()
    with sink:
        F.nvfp4_gemm(W, x, y, F.GemmTile(8, 128, 32), workspace=ws).submit(sink)
        F.gemv(W, x[:1], yv).submit(sink)
    assert torch.isnan(y).all()  # recorded, not run
    sink.replay()
    torch.cuda.synchronize()
    assert F.device_error() == 0
    exp, mag = expected_gemm(W.to_host(), x.float().cpu().numpy(), range(0, n))
    got = y.cpu().numpy().astype(np.float64)
    assert O.rel_frobenius(got, exp) <= REL_FROB_TOL
    hh = W.to_host()
    ref_v = O.nvfp4_gemv_f32(hh.packed, hh.scales, hh.row_scales, n, k, x[:1].float().cpu().numpy())
    assert O.rel_frobenius(yv.cpu().numpy(), ref_v) <= REL_FROB_TOL
