"""CPU-only checks of the C-ABI library: it loads, exports every declared
symbol, and its host-side logic (codecs, format validation, MoE bookkeeping)
matches the oracle and the reference's rules.  No kernel is launched."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

import firepit_b200 as F
from firepit_b200 import _native as N
from oracle import oracle as O

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> set:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(fpb_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    names = declared_symbols()
    assert len(names) >= 20
    lib = C.CDLL(str(N.LIB_PATH))
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding declares a signature for each of them
    assert names <= set(N.SIGNATURES), sorted(names - set(N.SIGNATURES))


def test_status_strings():
    for code in range(9):
        assert N.lib.fpb_status_string(code)
    assert N.lib.fpb_status_string(0) == b"ok"


def test_host_codecs_match_oracle():
    for c in range(16):
        assert N.lib.fpb_e2m1_to_f32(c) == O.e2m1_test(c)
    for b in range(256):
        assert N.lib.fpb_e4m3_to_f32(b) == O.e4m3(b)
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.standard_normal(3000) * 100, rng.standard_normal(3000) * 1e-3,
                         rng.uniform(-8, 8, 3000), [0.0, -0.0, 448.0, 464.0, 6.0, 5.0, 2 ** -10]])
    for x in xs.astype(np.float32):
        assert N.lib.fpb_f32_to_e4m3(float(x)) == O.lib.orc_f32_to_e4m3(float(x)), x
        assert N.lib.fpb_f32_to_e2m1(float(x)) == O.lib.orc_f32_to_e2m1(float(x)), x


def _validate(packed_len, scales, globals_, rows, cols):
    packed = np.zeros(max(packed_len, 1), np.uint8)
    scales = np.ascontiguousarray(scales, np.uint8)
    g = np.ascontiguousarray(globals_, np.float32)
    return N.lib.fpb_nvfp4_validate(packed.ctypes.data, packed_len, scales.ctypes.data, scales.size,
                                    g.ctypes.data, rows, cols)


def test_nvfp4_validation_mirrors_from_parts():
    """weights/nvfp4.rs:53-64 (every Err branch) and the oracle's restatement."""
    rows, cols = 4, 64
    ok_scales = np.full(rows * cols // 16, 0x38, np.uint8)
    assert _validate(rows * cols // 2, ok_scales, [1.0] * rows, rows, cols) == N.FPB_OK
    cases = [
        (rows * cols // 2, ok_scales, [1.0] * rows, 0, cols),          # rows == 0
        (rows * cols // 2, ok_scales, [1.0] * rows, rows, 48),         # cols % 32
        (rows * cols // 2 - 1, ok_scales, [1.0] * rows, rows, cols),   # packed length
        (rows * cols // 2, ok_scales[:-1], [1.0] * rows, rows, cols),  # scales length
        (rows * cols // 2, np.r_[ok_scales[:-1], 0x7F], [1.0] * rows, rows, cols),  # NaN scale
        (rows * cols // 2, np.r_[ok_scales[:-1], 0xFF], [1.0] * rows, rows, cols),  # -NaN scale
        (rows * cols // 2, ok_scales, [1.0, np.inf, 1.0, 1.0], rows, cols),          # inf global
        (rows * cols // 2, ok_scales, [1.0, np.nan, 1.0, 1.0], rows, cols),          # NaN global
        (rows * cols // 2, ok_scales, [1.0, -0.5, 1.0, 1.0], rows, cols),            # negative global
    ]
    for args in cases:
        assert _validate(*args) == N.FPB_ERR_FORMAT, args
        g = np.ascontiguousarray(args[2], np.float32)
        s = np.ascontiguousarray(args[1], np.uint8)
        assert O.lib.orc_nvfp4_validate(args[0], s.ctypes.data, s.size, g.ctypes.data, args[3], args[4]) != 0
    # negative (non-NaN) e4m3 scales are accepted, as in the reference
    assert _validate(rows * cols // 2, np.full(rows * cols // 16, 0xB8, np.uint8), [1.0] * rows, rows,
                     cols) == N.FPB_OK
    with pytest.raises(F.FormatError):
        F.HostNvfp4Matrix.from_parts(np.zeros(rows * cols // 2, np.uint8), np.r_[ok_scales[:-1], 0x7F], 1.0,
                                     rows, cols)
    m = F.HostNvfp4Matrix.from_parts(np.zeros(rows * cols // 2, np.uint8), ok_scales, 0.5, rows, cols)
    assert m.row_scales.tolist() == [0.5] * rows


def test_host_stack_keeps_per_part_globals():
    a = F.HostNvfp4Matrix.from_parts(np.zeros(64, np.uint8), np.zeros(8, np.uint8), 1.0, 2, 64)
    b = F.HostNvfp4Matrix.from_parts(np.ones(64, np.uint8), np.ones(8, np.uint8), 0.25, 2, 64)
    s = F.HostNvfp4Matrix.stack([a, b])
    assert s.rows == 4 and s.row_scales.tolist() == [1.0, 1.0, 0.25, 0.25]
    with pytest.raises(F.FormatError):
        F.HostNvfp4Matrix.stack([a, F.HostNvfp4Matrix.zeros(2, 32)])
    with pytest.raises(F.FormatError):
        F.HostNvfp4Matrix.stack([])


def test_moe_dims_validation():
    """kernels src/moe.rs:943-960."""
    assert F.MoeDims.new(2048, 512, 512, 256, 8)
    assert F.MoeDims.new(2048, 512, 512, 512, 10)
    for dims in [(0, 512, 512, 256, 8), (2048, 0, 512, 256, 8), (2048, 512, 0, 256, 8), (2048, 512, 512, 0, 8),
                 (2048, 512, 512, 256, 0), (2048, 512, 256, 256, 8), (2048, 512, 512, 4, 8),
                 (48, 512, 512, 256, 8), (2048, 96, 512, 256, 8)]:
        with pytest.raises(F.MoeDimensionError):
            F.MoeDims.new(*dims)


def test_prefill_layout_errors():
    dims = F.MoeDims.new(32, 32, 32, 4, 2)
    for ids, w, kind in [([], [], "Count"), ([0, 1, 2], [1, 1, 1], "Count"), ([0, 5], [1, 1], "Index"),
                         ([1, 1], [1, 1], "Duplicate"), ([0, 1], [-1, 1], "Weight"),
                         ([0, 1], [np.nan, 1], "Weight"), ([0, 1], [0, 0], "Weight")]:
        with pytest.raises(F.ExpertSelectionError) as e:
            F.PrefillLayout.parse(ids, w, dims, 4)
        assert e.value.kind == kind, (ids, w, str(e.value))
    with pytest.raises(F.ExpertSelectionError) as e:
        F.PrefillLayout.parse([0, 1], [1, 1], dims, 3)
    assert e.value.kind == "Tile"
    assert F.PrefillLayout.max_padded_rows(4096, F.MoeDims.new(2048, 512, 512, 512, 10), 32) == \
        4096 * 10 + 512 * 31


def test_expert_selection_validation():
    dims = F.MoeDims.new(32, 32, 32, 4, 2)
    for ids, w in [([0], [1.0]), ([0, 4], [1, 1]), ([2, 2], [1, 1]), ([0, 1], [1, np.inf])]:
        idx = np.array(ids + [0] * (2 - len(ids)), np.int32)
        ww = np.array(list(w) + [0] * (2 - len(w)), np.float32)
        count = len(ids)
        assert N.lib.fpb_expert_selection_validate(idx.ctypes.data, ww.ctypes.data, count, dims.experts,
                                                   dims.top_k) == N.FPB_ERR_SELECTION


def test_gpu_calls_fail_cleanly_without_a_device():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    out = C.c_void_p()
    packed = np.zeros(64, np.uint8)
    scales = np.zeros(8, np.uint8)
    g = np.zeros(2, np.float32)
    st = N.lib.fpb_nvfp4_matrix_create(packed.ctypes.data, scales.ctypes.data, g.ctypes.data, 2, 64, None,
                                       C.byref(out))
    assert st in (N.FPB_ERR_NO_DEVICE, N.FPB_ERR_CUDA)
    assert out.value is None


def test_comm_host_side():
    """NCCL loads at run time; the unique id needs no GPU; bad ranks are
    rejected before any NCCL call."""
    if not N.lib.fpb_comm_available():
        pytest.skip("libnccl.so.2 not present")
    uid = (C.c_uint8 * N.FPB_COMM_ID_BYTES)()
    assert N.lib.fpb_comm_unique_id(uid) == N.FPB_OK
    assert any(uid)
    h = C.c_void_p()
    assert N.lib.fpb_comm_init(uid, 2, 2, 0, C.byref(h)) == N.FPB_ERR_INVALID_ARGUMENT
    assert N.lib.fpb_comm_init(uid, 0, 0, 0, C.byref(h)) == N.FPB_ERR_INVALID_ARGUMENT
    assert N.lib.fpb_status_string(N.FPB_ERR_COMM) == b"communication error"


def test_multi_gpu_and_batch_entry_points_check_arguments_first():
    """The expert-parallel, peer-memory and gather entry points reject bad
    shapes and pointers on the host, before any CUDA call (no GPU needed)."""
    fake = 1 << 20  # a 16-byte-aligned address that is never dereferenced
    # fpb_ep_dispatch: cols % 64, experts not divisible by ranks, too many ranks
    args = [fake, N.FPB_BF16, 4, 96, fake, fake, 4, 4, 16, 2, fake, fake, fake, fake, None]
    assert N.lib.fpb_ep_dispatch(*args) == N.FPB_ERR_SHAPE
    args[3], args[8] = 64, 15
    assert N.lib.fpb_ep_dispatch(*args) == N.FPB_ERR_SHAPE
    args[8], args[9] = 64, 33
    assert N.lib.fpb_ep_dispatch(*args) == N.FPB_ERR_SHAPE
    args[9], args[0] = 2, fake + 8  # x not 16-byte aligned
    assert N.lib.fpb_ep_dispatch(*args) == N.FPB_ERR_INVALID_ARGUMENT
    assert N.lib.fpb_ep_dispatch_chunks(fake, N.FPB_BF16, 4, 64, fake, fake, 4, 4, 16, 2, fake, None, 0, fake,
                                        fake, None) == N.FPB_ERR_INVALID_ARGUMENT  # no chunk table
    assert N.lib.fpb_ep_unpack(fake, 0, 64, 4, fake, fake, None) == N.FPB_ERR_SHAPE
    assert N.lib.fpb_ep_record_bytes(2048, 16) == 1280
    # fpb_moe_gather_codes: cols % 64, then the factor stride's alignment
    assert N.lib.fpb_moe_gather_codes(fake, 16, fake, 4, 8, 96, fake, 128, None, 0, fake, fake,
                                      None) == N.FPB_ERR_SHAPE
    assert N.lib.fpb_moe_gather_codes(fake, 1280, fake + 1024, 1282, 8, 2048, fake, 128, None, 0, fake, fake,
                                      None) == N.FPB_ERR_INVALID_ARGUMENT
    # masked layout: the same selection checks as fpb_moe_layout
    assert N.lib.fpb_moe_layout_masked(fake, 0, 4, 4, 16, 128, 128, fake, fake, fake, fake, fake, fake, 1 << 20,
                                       None) == N.FPB_ERR_SELECTION
    assert N.lib.fpb_moe_combine_chunks(fake, N.FPB_BF16, 128, 64, fake, fake, 8, 4, 4, None, 8, N.FPB_F32,
                                        None) == N.FPB_ERR_INVALID_ARGUMENT
    # peer memory and the barrier
    p = C.c_void_p()
    assert N.lib.fpb_ipc_alloc(0, C.byref(p)) == N.FPB_ERR_INVALID_ARGUMENT
    assert N.lib.fpb_ipc_get_handle(None, None) == N.FPB_ERR_INVALID_ARGUMENT
    assert N.lib.fpb_peer_barrier(fake, fake, fake, 0, 0, 100, None) == N.FPB_ERR_INVALID_ARGUMENT
    assert N.lib.fpb_peer_barrier(fake, fake, fake, 2, 2, 100, None) == N.FPB_ERR_INVALID_ARGUMENT
    assert N.lib.fpb_peer_barrier(fake, fake, fake, 2, 0, 0, None) == N.FPB_ERR_INVALID_ARGUMENT
    assert N.lib.fpb_peer_all_reduce_max(fake, fake, fake, 2, 0, None, 100, None) == N.FPB_ERR_INVALID_ARGUMENT
