"""numpy binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py, as the checker and the timed CPU baseline.  The
product package never imports it.  Each function restates reference code;
the citations are in fp_oracle.h.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        build()
    return C.CDLL(str(LIB_PATH))


lib = _load()
_vp, _sz = C.c_void_p, C.c_size_t
for name, res, args in [
    ("orc_e2m1_test", C.c_float, [C.c_uint8]),
    ("orc_e2m1_modelopt", C.c_float, [C.c_uint8]),
    ("orc_e4m3", C.c_float, [C.c_uint8]),
    ("orc_f32_to_e2m1", C.c_uint8, [C.c_float]),
    ("orc_f32_to_e4m3", C.c_uint8, [C.c_float]),
    ("orc_f32_to_bf16", C.c_uint16, [C.c_float]),
    ("orc_bf16_to_f32", C.c_float, [C.c_uint16]),
    ("orc_synth_normal_one", C.c_float, [C.c_uint64, C.c_uint32, C.c_uint64]),
    ("orc_synth_normal", None, [C.c_uint64, C.c_uint32, C.c_uint64, _sz, C.c_float, C.c_float, _vp]),
    ("orc_philox4x32_10", None, [_vp, _vp, _vp]),
    ("orc_nvfp4_quantize", C.c_int, [_vp, _sz, _sz, _sz, _vp, _vp, _vp]),
    ("orc_nvfp4_dequantize", None, [_vp, _vp, _vp, _sz, _sz, _vp]),
    ("orc_nvfp4_validate", C.c_int, [_sz, _vp, _sz, _vp, _sz, _sz]),
    ("orc_nvfp4_gemv_f32", None, [_vp, _vp, _vp, _sz, _sz, _vp, _sz, _vp]),
    ("orc_nvfp4_gemv_f64", None, [_vp, _vp, _vp, _sz, _sz, _vp, _sz, _vp, _vp]),
    ("orc_nvfp4_expert_gemv_f32", None, [_vp, _vp, _vp, _sz, _vp, _sz, _sz, _sz, _vp, _vp]),
    ("orc_fp8_quantize", C.c_int, [_vp, _sz, _sz, _sz, _sz, _vp, _vp]),
    ("orc_fp8_dequantize", None, [_vp, _vp, _sz, _sz, _sz, _sz, _vp]),
    ("orc_fp8_gemm_f64", None, [_vp, _vp, _sz, _vp, _vp, _sz, _sz, _sz, _sz, _vp, _vp]),
    ("orc_moe_topk", None, [_vp, _sz, _vp, _sz, _sz, _sz, _sz, _vp, _vp]),
    ("orc_moe_layout", C.c_int, [_vp, _sz, _sz, _sz, _sz, _sz, _sz, _vp, _vp, _vp, _vp, _vp]),
    ("orc_swiglu", None, [_vp, _sz, _sz, _vp]),
    ("orc_moe_combine", None, [_vp, _sz, _vp, _vp, _sz, _sz, _sz, _vp, _vp, C.c_float, _vp, _vp]),
    ("orc_gamma_tilde", C.c_double, [_sz]),
    ("orc_inner_product_excess", C.c_double, [_vp, _vp, _vp, _sz, _sz]),
    ("orc_num_threads", C.c_int, []),
    ("orc_set_num_threads", None, [C.c_int]),
]:
    fn = getattr(lib, name)
    fn.restype = res
    fn.argtypes = args


def _p(a: np.ndarray) -> int:
    assert a.flags.c_contiguous
    return a.ctypes.data


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ---- codecs -------------------------------------------------------------------
def e2m1_test(code: int) -> float:
    return lib.orc_e2m1_test(code)


def e2m1_modelopt(code: int) -> float:
    return lib.orc_e2m1_modelopt(code)


def e4m3(bits: int) -> float:
    return lib.orc_e4m3(bits)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bit patterns (RNE)."""
    x = f32(x)
    u = x.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---- synthetic data ---------------------------------------------------------------
def synth_normal(count: int, seed: int, stream: int, mean: float = 0.0, std: float = 1.0,
                 offset: int = 0) -> np.ndarray:
    out = np.empty(count, np.float32)
    lib.orc_synth_normal(seed, stream, offset, count, mean, std, _p(out))
    return out


# ---- NVFP4 ----------------------------------------------------------------------------
def nvfp4_quantize(w: np.ndarray, rows_per_global: int | None = None):
    w = f32(w)
    rows, cols = w.shape
    rpg = rows if rows_per_global is None else rows_per_global
    packed = np.empty(rows * cols // 2, np.uint8)
    scales = np.empty(rows * cols // 16, np.uint8)
    globals_ = np.empty(rows, np.float32)
    rc = lib.orc_nvfp4_quantize(_p(w), rows, cols, rpg, _p(packed), _p(scales), _p(globals_))
    if rc != 0:
        raise ValueError("orc_nvfp4_quantize: invalid input")
    return packed, scales, globals_


def nvfp4_dequantize(packed, scales, row_globals, rows: int, cols: int) -> np.ndarray:
    out = np.empty((rows, cols), np.float32)
    lib.orc_nvfp4_dequantize(_p(packed), _p(scales), _p(f32(row_globals)), rows, cols, _p(out))
    return out


def nvfp4_gemv_f32(packed, scales, row_globals, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    x = f32(x).reshape(-1, cols)
    y = np.empty((x.shape[0], rows), np.float32)
    lib.orc_nvfp4_gemv_f32(_p(packed), _p(scales), _p(f32(row_globals)), rows, cols, _p(x), x.shape[0], _p(y))
    return y


def nvfp4_gemv_f64(packed, scales, row_globals, rows: int, cols: int, x: np.ndarray):
    x = f32(x).reshape(-1, cols)
    e = np.empty((x.shape[0], rows), np.float64)
    m = np.empty((x.shape[0], rows), np.float64)
    lib.orc_nvfp4_gemv_f64(_p(packed), _p(scales), _p(f32(row_globals)), rows, cols, _p(x), x.shape[0],
                           _p(e), _p(m))
    return e, m


def nvfp4_expert_gemv_f32(packed, scales, row_globals, cols: int, ids, rows_per_expert: int,
                          input_stride: int, x: np.ndarray) -> np.ndarray:
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    x = f32(x).reshape(-1, cols)
    y = np.empty((ids.size, rows_per_expert), np.float32)
    lib.orc_nvfp4_expert_gemv_f32(_p(packed), _p(scales), _p(f32(row_globals)), cols, _p(ids), ids.size,
                                  rows_per_expert, input_stride, _p(x), _p(y))
    return y


# ---- error model ----------------------------------------------------------------------
# ---- FP8 E4M3 --------------------------------------------------------------------------
def fp8_quantize(w: np.ndarray, block_n: int = 0, block_k: int = 0):
    """bits u8 [rows, cols] and f32 scales ([rows] when block_n = block_k = 0,
    else [rows/block_n, cols/block_k])."""
    w = f32(w)
    rows, cols = w.shape
    bits = np.empty((rows, cols), np.uint8)
    n_scales = rows if block_n == 0 and block_k == 0 else (rows // block_n) * (cols // block_k)
    scales = np.empty(n_scales, np.float32)
    if lib.orc_fp8_quantize(_p(w), rows, cols, block_n, block_k, _p(bits), _p(scales)) != 0:
        raise ValueError("orc_fp8_quantize: invalid input")
    return bits, scales


def fp8_dequantize(bits, scales, block_n: int = 0, block_k: int = 0) -> np.ndarray:
    bits = np.ascontiguousarray(bits, np.uint8)
    rows, cols = bits.shape
    out = np.empty((rows, cols), np.float32)
    lib.orc_fp8_dequantize(_p(bits), _p(f32(scales)), rows, cols, block_n, block_k, _p(out))
    return out


def fp8_gemm_f64(a_bits, a_scales, w_bits, w_scales, block_n: int = 0, block_k: int = 0):
    a_bits = np.ascontiguousarray(a_bits, np.uint8)
    w_bits = np.ascontiguousarray(w_bits, np.uint8)
    m, k = a_bits.shape
    n = w_bits.shape[0]
    e = np.empty((m, n), np.float64)
    mag = np.empty((m, n), np.float64)
    lib.orc_fp8_gemm_f64(_p(a_bits), _p(f32(a_scales)), m, _p(w_bits), _p(f32(w_scales)), n, k, block_n, block_k,
                         _p(e), _p(mag))
    return e, mag


# ---- MoE ---------------------------------------------------------------------------------
def moe_topk(logits, k: int, width: int, shared_gate=None):
    logits = f32(logits)
    tokens, experts = logits.shape
    ids = np.empty((tokens, width), np.int32)
    w = np.empty((tokens, width), np.float32)
    g = None if shared_gate is None else f32(shared_gate).reshape(-1)
    lib.orc_moe_topk(_p(logits), experts, None if g is None else _p(g), tokens, experts, k, width, _p(ids), _p(w))
    return ids, w


def moe_layout(ids, kk: int, experts: int, tile_rows: int, cap: int):
    ids = np.ascontiguousarray(ids, np.int32)
    tokens, width = ids.shape
    token_rows = np.empty(cap, np.int32)
    tile_experts = np.empty(cap // tile_rows, np.int32)
    inverse = np.empty((tokens, width), np.int32)
    ranges = np.empty((experts, 2), np.int64)
    padded = np.zeros(1, np.int32)
    rc = lib.orc_moe_layout(_p(ids), tokens, width, kk, experts, tile_rows, cap, _p(token_rows), _p(tile_experts),
                            _p(inverse), _p(ranges), _p(padded))
    if rc != 0:
        raise ValueError("orc_moe_layout: invalid ids or capacity")
    return token_rows, tile_experts, inverse, ranges, int(padded[0])


def swiglu(gate_up):
    gate_up = f32(gate_up)
    rows, two_i = gate_up.shape
    out = np.empty((rows, two_i // 2), np.float32)
    lib.orc_swiglu(_p(gate_up), rows, two_i // 2, _p(out))
    return out


def moe_combine(routed, inverse, weights, slots: int, residual=None, gamma=None, eps: float = 1e-6):
    routed = f32(routed)
    inverse = np.ascontiguousarray(inverse, np.int32)
    weights = f32(weights)
    tokens, width = inverse.shape
    cols = routed.shape[1]
    out = np.empty((tokens, cols), np.float32)
    normed = np.empty((tokens, cols), np.float32) if residual is not None else None
    lib.orc_moe_combine(_p(routed), cols, _p(inverse), _p(weights), tokens, width, slots,
                        None if residual is None else _p(f32(residual)), None if gamma is None else _p(f32(gamma)),
                        eps, _p(out), None if normed is None else _p(normed))
    return (out, normed) if residual is not None else out


def gamma_tilde(n: int) -> float:
    return lib.orc_gamma_tilde(n)


def inner_product_excess(actual, expected, magnitude, n: int) -> float:
    a = f32(actual).reshape(-1)
    e = np.ascontiguousarray(expected, np.float64).reshape(-1)
    m = np.ascontiguousarray(magnitude, np.float64).reshape(-1)
    return lib.orc_inner_product_excess(_p(a), _p(e), _p(m), a.size, n)


def rel_frobenius(actual, expected) -> float:
    a = np.asarray(actual, np.float64).reshape(-1)
    e = np.asarray(expected, np.float64).reshape(-1)
    den = np.linalg.norm(e)
    return float(np.linalg.norm(a - e) / (den if den > 0 else 1.0))


def num_threads() -> int:
    return lib.orc_num_threads()


def set_num_threads(n: int) -> None:
    lib.orc_set_num_threads(int(n))
