"""Router top-k followed by the expert GEMVs on one stream, in one CUDA graph.

The GEMV kernels run under programmatic dependent launch.  In decode the
expert ids they read are written by the router top-k launched just before
them (moe.rs:15-68 then gemv/mod.rs:137-206), so the GEMVs must not read the
ids before the top-k has finished.  Each replay first overwrites the ids with
a stale expert, then runs top-k and the expert GEMV with no host
synchronisation in between; the outputs must be those of the fresh ids.
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


EXPERTS, RPE, COLS, TOP_K = 64, 512, 2048, 8


def _logits(round_):
    rng = np.random.default_rng(100 + round_)
    return rng.standard_normal((1, EXPERTS)).astype(np.float32)


@pytest.mark.parametrize("fmt", ["nvfp4", "fp8_blocks", "fp8_rows"])
def test_topk_then_expert_gemv_in_one_graph(F, torch, fmt):
    from firepit_b200 import _native as N
    w = F.synth_normal((EXPERTS * RPE, COLS), seed=21, stream_id=1, std=0.02)
    if fmt == "nvfp4":
        W = F.Nvfp4Matrix.quantize(w, rows_per_global=RPE)
        h = W.to_host()
        fn = "fpb_nvfp4_expert_gemv"
    else:
        block = (128, 128) if fmt == "fp8_blocks" else (0, 0)
        W = F.Fp8Matrix.quantize(w, F.Fp8Scaling(*block))
        h = W.to_host()
        wd = np.asarray(O.fp8_dequantize(h.bits.reshape(EXPERTS * RPE, COLS),
                                         h.scales if block == (0, 0) else
                                         h.scales.reshape(EXPERTS * RPE // 128, COLS // 128), *block),
                        np.float64).reshape(EXPERTS * RPE, COLS)
        fn = "fpb_fp8_expert_gemv"
    x = F.synth_normal((1, COLS), seed=0, stream_id=0, dtype=torch.bfloat16)
    xf = x.float().cpu().numpy()
    logits = torch.empty(1, EXPERTS, dtype=torch.float32, device="cuda")
    ids = torch.empty(1, TOP_K, dtype=torch.int32, device="cuda")
    wts = torch.empty(1, TOP_K, dtype=torch.float32, device="cuda")
    y = torch.empty(TOP_K, RPE, dtype=torch.float32, device="cuda")
    stale = 7

    def ops(stream):
        ids.fill_(stale)
        N.call("fpb_moe_topk", logits.data_ptr(), EXPERTS, None, 1, EXPERTS, TOP_K, TOP_K, ids.data_ptr(),
               wts.data_ptr(), stream)
        N.call(fn, W.handle, x.data_ptr(), N.FPB_BF16, ids.data_ptr(), TOP_K, RPE, 0, y.data_ptr(), N.FPB_F32,
               stream)

    logits.copy_(torch.from_numpy(_logits(0)))
    ops(torch.cuda.current_stream().cuda_stream)  # every code path initialised outside capture
    torch.cuda.synchronize()
    g = F.Graph()
    with g:
        g.run("chain", ops)
    for r in range(6):
        lg = _logits(r)
        logits.copy_(torch.from_numpy(lg))
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        ref_ids, _ = O.moe_topk(lg, TOP_K, TOP_K)
        assert np.array_equal(ids.cpu().numpy(), ref_ids), "top-k ids differ from the oracle"
        got = y.cpu().numpy()
        if fmt == "nvfp4":
            exp = O.nvfp4_expert_gemv_f32(h.packed, h.scales, h.row_scales, COLS, ref_ids[0], RPE, 0,
                                          np.repeat(xf, TOP_K, axis=0))
            assert O.rel_frobenius(got, exp) <= REL_FROB_TOL
        else:
            rows = np.concatenate([np.arange(e * RPE, (e + 1) * RPE) for e in ref_ids[0]])
            exp = (xf.astype(np.float64) @ wd[rows].T).reshape(TOP_K, RPE)
            assert O.rel_frobenius(got, exp) <= REL_FROB_TOL
    del g
