"""The W4A4 GEMM batch (firepit_b200.nvfp4_gemm_batch, fpb_nvfp4_gemm_batch_create)
against the single-matrix W4A4 GEMM.

Every member must equal ``nvfp4_gemm_view(weight, rows, x, y)`` for the same
m > 16 bit for bit: the same NVFP4 codes of x (per-tensor global) and the
same tcgen05 products and epilogue order.  ``nvfp4_gemm`` itself is checked
against the oracle in test_gpu_gemm.py.
"""
import pytest

pytestmark = pytest.mark.gpu

K = 512


def _weight(F, rows, cols, seed):
    w = F.synth_normal((rows, cols), seed=seed, stream_id=1, std=0.02)
    p, s, g = F.quantize_nvfp4(w)
    return F.Nvfp4Matrix.from_device(p, s, g, rows, cols)


@pytest.mark.parametrize("m", [17, 100, 128])
@pytest.mark.parametrize("dtypes", [("bf16", "bf16"), ("f32", "f32"), ("bf16", "f32")])
def test_members_equal_single_gemm(m, dtypes):
    import torch

    import firepit_b200 as F
    dt = {"bf16": torch.bfloat16, "f32": torch.float32}
    xd, yd = dt[dtypes[0]], dt[dtypes[1]]
    ws = [_weight(F, 384, K, 10 + i) for i in range(3)]
    xs = [F.synth_normal((m, K), seed=20 + i, stream_id=0, dtype=xd) for i in range(2)]
    # members: whole matrices, a row range, and two members sharing one x
    members = [(ws[0], xs[0], None, None), (ws[1], xs[1], None, range(128, 384)), (ws[2], xs[0], None, None),
               (ws[0], xs[1], None, range(256, 384))]
    members = [(w, x, torch.empty(m, len(r) if r else w.rows, dtype=yd, device="cuda"), r) for w, x, _, r in members]
    batch = F.nvfp4_gemm_batch(members)
    batch.submit(F.Eager())
    for w, x, y, r in members:
        ref = torch.empty_like(y)
        F.nvfp4_gemm_view(w, r or range(0, w.rows), x, ref, F.GemmTile(1, 128, 32)).submit(F.Eager())
        torch.cuda.synchronize()
        assert torch.equal(y, ref)
    assert F.device_error() == 0


def test_graph_replay_and_new_inputs():
    """The batch binds its tensors: a CUDA graph of submit picks up new x
    values on replay."""
    import torch

    import firepit_b200 as F
    m = 64
    ws = [_weight(F, 256, K, 30 + i) for i in range(4)]
    x = F.synth_normal((m, K), seed=40, stream_id=0, dtype=torch.bfloat16)
    ys = [torch.empty(m, 256, dtype=torch.bfloat16, device="cuda") for _ in ws]
    batch = F.nvfp4_gemm_batch([(w, x, y) for w, y in zip(ws, ys)])
    batch.submit(F.Eager())
    torch.cuda.synchronize()
    g = F.Graph()
    with g:
        batch.submit(g)
    x.copy_(F.synth_normal((m, K), seed=41, stream_id=0, dtype=torch.bfloat16))
    g.replay()
    torch.cuda.synchronize()
    for w, y in zip(ws, ys):
        ref = torch.empty_like(y)
        F.nvfp4_gemm(w, x, ref, F.GemmTile(1, 128, 32)).submit(F.Eager())
        torch.cuda.synchronize()
        assert torch.equal(y, ref)


def test_batch_errors():
    import torch

    import firepit_b200 as F
    w = _weight(F, 256, K, 50)
    x = torch.zeros(129, K, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(F.ShapeError):
        F.nvfp4_gemm_batch([(w, x, torch.empty(129, 256, dtype=torch.bfloat16, device="cuda"))])  # m > 128
    w2 = _weight(F, 256, 320, 51)
    x2 = torch.zeros(8, 320, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(F.ShapeError):
        F.nvfp4_gemm_batch([(w2, x2, torch.empty(8, 256, dtype=torch.bfloat16, device="cuda"))])  # K % 256
    with pytest.raises(F.ShapeError):
        F.nvfp4_gemm_batch([(w, x[:8], torch.empty(8, 128, dtype=torch.bfloat16, device="cuda"), range(64, 192))])


@pytest.mark.parametrize("ydt", ["bf16", "f32"])
def test_ragged_view_takes_direct_stores(ydt):
    """A member whose y pitch is not 16-byte aligned (a 300-row view) makes
    the batch store every member directly; results are the same."""
    import torch

    import firepit_b200 as F
    yd = {"bf16": torch.bfloat16, "f32": torch.float32}[ydt]
    m = 40
    ws = [_weight(F, 384, K, 60 + i) for i in range(2)]
    x = F.synth_normal((m, K), seed=61, stream_id=0, dtype=torch.bfloat16)
    members = [(ws[0], x, torch.empty(m, 300, dtype=yd, device="cuda"), range(0, 300)),
               (ws[1], x, torch.empty(m, 384, dtype=yd, device="cuda"), None)]
    F.nvfp4_gemm_batch(members).submit(F.Eager())
    for w, xx, y, r in members:
        ref = torch.empty_like(y)
        F.nvfp4_gemm_view(w, r or range(0, w.rows), xx, ref, F.GemmTile(1, 1, 32)).submit(F.Eager())
        torch.cuda.synchronize()
        assert torch.equal(y, ref)
    assert F.device_error() == 0
