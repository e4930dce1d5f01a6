"""The reference's deterministic NVFP4 test matrices, restated.

crates/firepit-kernels/tests/nvfp4_oracle.rs:241-321 builds its cases from
integer formulas of the element index and a proptest seed.  The same
formulas are evaluated here for a fixed list of seeds (the reference draws
them at random; these cover small, large and 64-bit values).
"""
from __future__ import annotations

import numpy as np

MASK64 = (1 << 64) - 1
PART_ROWS = 128                                  # nvfp4_oracle.rs:22
SCALES = [0x00, 0x01, 0x30, 0x38, 0x3B, 0x7E]    # nvfp4_oracle.rs:244
GLOBALS = [1.0, 3.2152449e-5, 0.75]              # nvfp4_oracle.rs:245
SEEDS = [0, 1, 2, 3, 5, 7, 11, 29, 255, 1023, 65537, 0xDEADBEEF, 0x123456789ABCDEF0,
         0xFFFFFFFFFFFFFFFF, 0x8000000000000001, 0x5A5A5A5A5A5A5A5A]


def _mix(i: np.ndarray, mul: int, seed: int) -> np.ndarray:
    """((i * mul) wrapping) ^ seed on u64, as the Rust tests compute it."""
    i = i.astype(np.uint64)
    return (i * np.uint64(mul)) ^ np.uint64(seed & MASK64)


def pack_codes(codes: np.ndarray) -> np.ndarray:
    """Pairs of codes -> bytes, first code in the low nibble (checkpoint.rs:414-418)."""
    c = codes.astype(np.uint8).reshape(-1, 2)
    return (c[:, 0] | (c[:, 1] << 4)).astype(np.uint8)


def kernels_case(k_blocks: int, seed: int):
    """nvfp4_kernels_match_dequantized_f64_oracle (nvfp4_oracle.rs:241-267)."""
    cols = (k_blocks + 1) * 128
    rows = 2 * PART_ROWS
    i = np.arange(rows * cols)
    codes = (_mix(i, 29, seed) % np.uint64(16)).astype(np.uint8)
    g = np.arange(rows * cols // 16)
    scales = np.array(SCALES, np.uint8)[(_mix(g, 7, seed) % np.uint64(len(SCALES))).astype(np.int64)]
    s = seed & MASK64
    globals_ = [GLOBALS[s % 3], GLOBALS[(s // 3) % 3]]
    k = np.arange(cols)
    x = (_mix(k, 13, seed) % np.uint64(41)).astype(np.float32) / np.float32(37.0) - np.float32(0.5)
    return _assemble(codes, scales, globals_, rows, cols) + (x.astype(np.float32), s % 2)


EXTREME_CASES = [  # nvfp4_oracle.rs:276-295: (codes, scales, globals, amplitude)
    ([0x7, 0xF, 0x0, 0x8], [0x7E, 0x7E], [2.0 ** -100, 1.0], 1.0),
    ([0x1, 0x9, 0x1, 0x9], [0x01, 0x01], [2.0 ** 100, 1.0], 2.0 ** 20),
    ([0x7, 0x9, 0xF, 0x1], [0x7E, 0x01], [1.0, 0.75], 2.0 ** 20),
]


def extreme_case(case: int, seed: int):
    """nvfp4_extreme_finite_values_match_f64_oracle (nvfp4_oracle.rs:269-321)."""
    codes_t, scales_t, globals_, amp = EXTREME_CASES[case]
    cols, rows = 256, 2 * PART_ROWS
    i = np.arange(rows * cols)
    codes = np.array(codes_t, np.uint8)[(_mix(i, 7, seed) % np.uint64(4)).astype(np.int64)]
    g = np.arange(rows * cols // 16).astype(np.uint64)
    scales = np.array(scales_t, np.uint8)[((g ^ np.uint64(seed & MASK64)) % np.uint64(2)).astype(np.int64)]
    k = np.arange(cols)
    x = np.where(((k + (seed & MASK64) % 3) % 3) == 0, -amp, amp).astype(np.float32)
    return _assemble(codes, scales, globals_, rows, cols) + (x, (seed & MASK64) % 2)


def _assemble(codes, scales, globals_, rows, cols):
    packed = pack_codes(codes)
    row_globals = np.repeat(np.array(globals_, np.float32), PART_ROWS)
    return packed, scales.astype(np.uint8), row_globals, rows, cols


# ---- FP8 (crates/firepit-kernels/tests/fp8_oracle.rs) ----------------------------------------
FP8_VALUES = [(0xB8, -1.0), (0x38, 1.0), (0x30, 0.5), (0xC0, -2.0), (0x40, 2.0), (0x39, 1.125), (0x3B, 1.375),
              (0x35, 0.8125)]                       # fp8_oracle.rs:122-131
FP8_SCALES = [0.8125, 1.203125, 2.25]               # fp8_oracle.rs:132


def _wrapping_add_mod(i: np.ndarray, seed: int, mod: int) -> np.ndarray:
    """((i + seed) wrapping on u64) % mod."""
    return ((i.astype(np.uint64) + np.uint64(seed & MASK64)) % np.uint64(mod)).astype(np.int64)


def fp8_kernels_case(n_blocks: int, k_blocks: int, seed: int):
    """fp8_gemv_and_gemm_match_dequantized_f64_oracle (fp8_oracle.rs:119-170):
    bits [rows, cols], 128x128 block scales, the input row, rows, cols."""
    rows, cols = (n_blocks + 1) * 128, (k_blocks + 1) * 128
    i = np.arange(rows * cols)
    table = np.array([b for b, _ in FP8_VALUES], np.uint8)
    bits = table[(_mix(i, 17, seed) % np.uint64(len(FP8_VALUES))).astype(np.int64)].reshape(rows, cols)
    nsc = (rows // 128) * (cols // 128)
    scales = np.array(FP8_SCALES, np.float32)[_wrapping_add_mod(np.arange(nsc), seed, len(FP8_SCALES))]
    x = ((_mix(np.arange(cols), 13, seed) % np.uint64(41)).astype(np.float32) / np.float32(37.0)
         - np.float32(0.5)).astype(np.float32)
    return bits, scales, x, rows, cols


FP8_EXTREME_CASES = [  # fp8_oracle.rs:251-268: (scale, encodings, amplitude)
    (float(np.uint32(0x0001 << 16).view(np.float32)), [0x7E, 0xFE, 0x7E, 0xFE], 2.0 ** 20),
    (float(np.uint32(0x7F7F << 16).view(np.float32)), [0x01, 0x81, 0x01, 0x81], 0.5),
    (1.0 / 128.0, [0x7E, 0xFE, 0x01, 0x81], 2.0 ** 20),
]


def fp8_extreme_case(case: int, seed: int):
    """fp8_extreme_finite_values_match_f64_oracle (fp8_oracle.rs:247-300):
    rows 128, cols 256, one scale per 128x128 block."""
    scale, enc, amp = FP8_EXTREME_CASES[case]
    rows, cols = 128, 256
    i = np.arange(rows * cols)
    bits = np.array(enc, np.uint8)[(_mix(i, 7, seed) % np.uint64(4)).astype(np.int64)].reshape(rows, cols)
    x = np.where(_wrapping_add_mod(np.arange(cols), seed, 3) == 0, -amp, amp).astype(np.float32)
    return bits, np.full(2, scale, np.float32), x, rows, cols
