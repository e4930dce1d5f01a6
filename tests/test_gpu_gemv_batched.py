"""Several NVFP4 decode GEMVs in one launch (fpb_nvfp4_gemv_batched).

Each member must equal the single-matrix GEMV of the same operands (bit for
bit where both run the streaming kernel with the same unit height) and the
oracle's f32 kernel-order result (gemv/nvfp4.rs:34-59) within the relative
Frobenius tolerance of the other GEMV tests.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_FROB_TOL = 1e-3       # f32 output vs the oracle
REL_FROB_TOL_BF16 = 4e-3  # bf16 output rounding on top


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


@pytest.fixture(scope="module")
def F(torch):
    import firepit_b200
    return firepit_b200


def _matrix(F, rows, cols, seed):
    w = F.synth_normal((rows, cols), seed=seed, stream_id=1, std=0.02)
    m = F.Nvfp4Matrix.quantize(w)
    return m, m.to_host()


def _x(torch, batch, cols, seed, dtype):
    x = O.synth_normal(batch * cols, seed=seed, stream=2).reshape(batch, cols)
    xt = torch.from_numpy(x).cuda().to(dtype)
    return xt, xt.float().cpu().numpy()


@pytest.mark.parametrize("batch", [1, 4, 8])
@pytest.mark.parametrize("xdt,ydt", [("bf16", "f32"), ("f32", "f32"), ("bf16", "bf16")])
@pytest.mark.parametrize("cols", [2048, 4096, 640])
def test_batched_members_match_single_gemvs_and_oracle(F, torch, batch, xdt, ydt, cols):
    tx = torch.bfloat16 if xdt == "bf16" else torch.float32
    ty = torch.bfloat16 if ydt == "bf16" else torch.float32
    mats = [_matrix(F, r, cols, seed=s) for r, s in ((1024, 1), (4096, 2), (512, 3))]
    x0, x0f = _x(torch, batch, cols, 10, tx)
    x1, x1f = _x(torch, batch, cols, 11, tx)
    # (matrix, rows, x): whole matrices, a row range, a shared x, a 4-row sliver
    plan = [(0, range(0, 1024), 0), (1, range(0, 4096), 1), (2, range(128, 512), 0), (0, range(100, 364), 1),
            (1, range(4092, 4096), 0)]
    xs, xfs = [x0, x1], [x0f, x1f]
    members, ys = [], []
    for mi, rows, xi in plan:
        y = torch.full((batch, len(rows)), float("nan"), dtype=ty, device="cuda")
        members.append((mats[mi][0], xs[xi], y, rows))
        ys.append(y)
    tile = F.GemvTile(4, 4)  # the row ranges are multiples of 4, not of the default 16
    F.gemv_batched(members, tile).submit(F.Eager())
    tol = REL_FROB_TOL if ydt == "f32" else REL_FROB_TOL_BF16
    for (mi, rows, xi), y in zip(plan, ys):
        m, h = mats[mi]
        single = torch.full_like(y, float("nan"))
        F.gemv(m, xs[xi], single, tile, rows=rows).submit(F.Eager())
        got, one = y.float().cpu().numpy(), single.float().cpu().numpy()
        ref = O.nvfp4_gemv_f32(h.packed, h.scales, h.row_scales, m.rows, cols, xfs[xi])[:, rows.start:rows.stop]
        assert O.rel_frobenius(got, ref) <= tol, f"member {mi} {rows}"
        assert O.rel_frobenius(got, one) <= 1e-5 if ydt == "f32" else O.rel_frobenius(got, one) <= 8e-3


def test_batched_config0_sixteen_matrices(F, torch):
    """Sixteen BASELINE config-0 matrices (4096x4096, x bf16 N(0,1), y bf16)
    in one launch, each with its own x."""
    n, rows, cols = 16, 4096, 4096
    members, refs = [], []
    for i in range(n):
        m, h = _matrix(F, rows, cols, seed=100 + i)
        x = F.synth_normal((1, cols), seed=i, stream_id=0, dtype=torch.bfloat16)
        y = torch.full((1, rows), float("nan"), dtype=torch.bfloat16, device="cuda")
        members.append((m, x, y))
        refs.append((h, x.float().cpu().numpy()))
    F.gemv_batched(members).submit(F.Eager())
    for (m, x, y), (h, xf) in zip(members, refs):
        ref = O.nvfp4_gemv_f32(h.packed, h.scales, h.row_scales, rows, cols, xf)
        assert O.rel_frobenius(y.float().cpu().numpy(), ref) <= REL_FROB_TOL_BF16


def test_batched_fallback_shapes_and_errors(F, torch):
    from firepit_b200 import _native as N
    # cols % 128 != 0 and a batch above 8: one launch per member, same results
    for cols, batch in ((160, 2), (2048, 12)):
        mats = [_matrix(F, 96, cols, seed=cols + i) for i in range(3)]
        x, xf = _x(torch, batch, cols, 5, torch.bfloat16)
        ys = [torch.empty(batch, 96, device="cuda") for _ in mats]
        F.gemv_batched([(m, x, y) for (m, _), y in zip(mats, ys)], F.GemvTile(16, 1)).submit(F.Eager())
        for (m, h), y in zip(mats, ys):
            ref = O.nvfp4_gemv_f32(h.packed, h.scales, h.row_scales, 96, cols, xf)
            assert O.rel_frobenius(y.cpu().numpy(), ref) <= REL_FROB_TOL
    a, _ = _matrix(F, 64, 256, seed=1)
    b, _ = _matrix(F, 64, 512, seed=2)
    x = torch.zeros(1, 512, device="cuda")
    y = torch.zeros(1, 64, device="cuda")
    segs = (N.GemvSegment * 2)(N.GemvSegment(a.handle.value, 0, 0, x.data_ptr(), y.data_ptr()),
                               N.GemvSegment(b.handle.value, 0, 0, x.data_ptr(), y.data_ptr()))
    assert N.lib.fpb_nvfp4_gemv_batched(segs, 2, N.FPB_F32, N.FPB_F32, 1, None) == N.FPB_ERR_SHAPE
    many = (N.GemvSegment * 129)(*[N.GemvSegment(a.handle.value, 0, 0, x.data_ptr(), y.data_ptr())] * 129)
    assert N.lib.fpb_nvfp4_gemv_batched(many, 129, N.FPB_F32, N.FPB_F32, 1, None) == N.FPB_ERR_UNSUPPORTED
    bad = (N.GemvSegment * 1)(N.GemvSegment(a.handle.value, 32, 16, x.data_ptr(), y.data_ptr()))
    assert N.lib.fpb_nvfp4_gemv_batched(bad, 1, N.FPB_F32, N.FPB_F32, 1, None) == N.FPB_ERR_SHAPE
    torch.cuda.synchronize()
