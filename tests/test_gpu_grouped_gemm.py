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
               192, y.data_ptr(), N.FPB_F32, None)
    assert e.value.status == 2
