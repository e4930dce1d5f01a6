"""The quantizer entry point that allocates nothing.

fpb_nvfp4_quantize_noalloc serves callers that cannot allocate device
memory (their device memory is one arena reserved up front, or their serving
loop must not call cudaMalloc).  It keeps its scratch in a fixed array inside
the library, so this test checks that, called twice in a row through the C
ABI, it produces exactly what the ordinary entry point (given its own
scratch buffer) produces, and that the second call is not disturbed by what
the first left in the shared array.  Quantization is bit-exact, so the
comparison is exact.  This file is collected last on purpose.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _quantize(N, torch, w, rpg, noalloc):
    rows, cols = w.shape
    dtype = N.FPB_BF16 if w.dtype == torch.bfloat16 else N.FPB_F32
    packed = torch.empty(rows, cols // 2, dtype=torch.uint8, device="cuda")
    scales = torch.empty(rows, cols // 16, dtype=torch.uint8, device="cuda")
    globals_ = torch.empty(rows, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    if noalloc:
        N.call("fpb_nvfp4_quantize_noalloc", w.data_ptr(), dtype, rows, cols, rpg, packed.data_ptr(),
               scales.data_ptr(), globals_.data_ptr(), stream)
    else:
        scratch = torch.empty(rows // rpg, dtype=torch.float32, device="cuda")
        N.call("fpb_nvfp4_quantize", w.data_ptr(), dtype, rows, cols, rpg, packed.data_ptr(),
               scales.data_ptr(), globals_.data_ptr(), scratch.data_ptr(), stream)
    torch.cuda.synchronize()
    return packed.cpu().numpy(), scales.cpu().numpy(), globals_.cpu().numpy().view(np.uint32)


def test_noalloc_quantize_matches_the_allocating_entry_point_twice():
    import torch

    import firepit_b200 as F
    from firepit_b200 import _native as N

    # First call: large values and many row blocks; second call: small values
    # and fewer blocks, so stale maxima left in the shared array would show.
    cases = [(F.synth_normal((512, 2048), seed=1, stream_id=5, std=3.0), 32),
             (F.synth_normal((256, 1024), seed=2, stream_id=6, std=0.02).to(torch.bfloat16), 64)]
    for w, rpg in cases:
        got = _quantize(N, torch, w, rpg, noalloc=True)
        want = _quantize(N, torch, w, rpg, noalloc=False)
        for g, e in zip(got, want):
            assert np.array_equal(g, e)


def test_noalloc_quantize_rejects_more_blocks_than_its_scratch():
    import torch

    from firepit_b200 import _native as N

    w = torch.zeros(16385, 32, device="cuda")
    out = torch.empty(16385 * 16, dtype=torch.uint8, device="cuda")
    g = torch.empty(16385, device="cuda")
    st = N.lib.fpb_nvfp4_quantize_noalloc(w.data_ptr(), N.FPB_F32, 16385, 32, 1, out.data_ptr(), out.data_ptr(),
                                         g.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == N.FPB_ERR_UNSUPPORTED
    assert "scratch" in N.last_error()
