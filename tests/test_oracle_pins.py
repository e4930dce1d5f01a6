"""Pins the CPU oracle before it is trusted as the checker.

* decode tables: every e2m1 code and every e4m3 byte against the reference's
  own formulas (kernels tests/nvfp4_oracle.rs:21-42, firepit
  src/checkpoint.rs:338-390) and against torch's independent e4m3 decoder;
* the ModelOpt / Qwen dequant fixture of the reference (bit patterns from
  real checkpoints, tests/golden/dequant_samples.json): every sample must be
  reachable through the oracle's decode tables with one global per tensor;
* the quantizer (no reference counterpart, parity unpinned): rounding and
  saturation properties of RN_e2m1 / RN_e4m3 and round-trip bounds;
* the MoE prefill layout against a stable sort (kernels src/moe.rs:865-941).
"""
import json
import math
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


# ---- restated reference formulas -------------------------------------------------------
def ref_e2m1(code: int) -> float:  # kernels tests/nvfp4_oracle.rs:21-31
    m = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0][code & 7]
    return -m if code & 8 else m


def ref_e4m3(bits: int) -> float:  # kernels tests/nvfp4_oracle.rs:33-42
    sign = -1.0 if bits & 0x80 else 1.0
    e, f = (bits >> 3) & 0xF, bits & 7
    return sign * f * 2.0 ** -9 if e == 0 else sign * (1 + f / 8) * 2.0 ** (e - 7)


def test_e2m1_all_codes():
    for c in range(16):
        assert np.float32(O.e2m1_test(c)).tobytes() == np.float32(ref_e2m1(c)).tobytes()
        want = 0.0 if c == 8 else ref_e2m1(c)  # ModelOpt table, checkpoint.rs:386-390
        assert np.float32(O.e2m1_modelopt(c)).tobytes() == np.float32(want).tobytes()
    assert math.copysign(1.0, O.e2m1_test(8)) == -1.0
    assert math.copysign(1.0, O.e2m1_modelopt(8)) == 1.0


def test_e4m3_all_bytes_match_formula_and_torch():
    torch = pytest.importorskip("torch")
    raw = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    for b in range(256):
        assert O.e4m3(b) == ref_e4m3(b)
        if b & 0x7F == 0x7F:  # NaN in e4m3fn; the reference formula has no NaN case
            assert math.isnan(raw[b])
        else:
            assert O.e4m3(b) == raw[b], hex(b)


# ---- quantizer rounding --------------------------------------------------------------
def _grid_e4m3():
    vals = sorted({O.e4m3(b) for b in range(0x7F)})
    return vals


def test_e4m3_rounding_midpoints_and_saturation():
    vals = _grid_e4m3()
    for i, v in enumerate(vals):
        assert O.e4m3(O.lib.orc_f32_to_e4m3(v)) == v
        assert O.lib.orc_f32_to_e4m3(-v) == (O.lib.orc_f32_to_e4m3(v) | 0x80)
        if i + 1 < len(vals):
            mid = np.float32((v + vals[i + 1]) / 2)
            got = O.e4m3(O.lib.orc_f32_to_e4m3(float(mid)))
            lo_code, hi_code = O.lib.orc_f32_to_e4m3(v), O.lib.orc_f32_to_e4m3(vals[i + 1])
            assert got == (v if lo_code % 2 == 0 else vals[i + 1]), (v, vals[i + 1])
            del hi_code
    for big in (448.0, 449.0, 463.9, 464.0, 480.0, 1e6, float("inf")):
        assert O.lib.orc_f32_to_e4m3(big) == 0x7E
    assert O.lib.orc_f32_to_e4m3(2.0 ** -10) == 0x00  # half of the smallest subnormal: ties to even
    assert O.lib.orc_f32_to_e4m3(2.0 ** -10 * 1.0001) == 0x01


def test_e2m1_rounding_midpoints_and_saturation():
    grid = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    for c, v in enumerate(grid):
        assert O.lib.orc_f32_to_e2m1(v) == c
        assert O.lib.orc_f32_to_e2m1(-v) == c | 8
    ties = {0.25: 0.0, 0.75: 1.0, 1.25: 1.0, 1.75: 2.0, 2.5: 2.0, 3.5: 4.0, 5.0: 4.0}
    for x, want in ties.items():
        assert O.e2m1_test(O.lib.orc_f32_to_e2m1(x)) == want, x
    for big in (6.0, 7.0, 1e30, float("inf")):
        assert O.lib.orc_f32_to_e2m1(big) == 7


def test_random_values_round_to_nearest():
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.standard_normal(4000) * 3, rng.uniform(-7, 7, 4000)]).astype(np.float32)
    grid = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
    for x in xs:
        got = abs(O.e2m1_test(O.lib.orc_f32_to_e2m1(float(x))))
        best = np.min(np.abs(grid - min(abs(x), 6.0)))
        assert abs(got - min(abs(x), 6.0)) <= best + 1e-12


def test_nvfp4_quantize_round_trip_bounds():
    w = O.synth_normal(64 * 256, seed=3, stream=1, std=0.02).reshape(64, 256)
    packed, scales, g = O.nvfp4_quantize(w)
    amax = np.abs(w).max()
    assert g[0] == np.float32(amax) / np.float32(2688.0)
    assert all((s & 0x7F) != 0x7F for s in scales)
    dq = O.nvfp4_dequantize(packed, scales, g, 64, 256)
    s_dec = np.array([O.e4m3(int(s)) for s in scales], np.float64).reshape(64, 16)
    step = np.repeat(s_dec * float(g[0]), 16, axis=1)  # one e2m1 unit of each group
    # Largest e2m1 gap is 2 units (between 4 and 6): half of it bounds the error,
    # plus the satfinite clamp when the scale rounded down.
    err = np.abs(dq.astype(np.float64) - w)
    assert np.all(err <= step * 1.0 + 1e-30)
    # A quantized matrix round-trips: its dequantized values are all on the grid.
    codes = np.stack([packed & 0xF, packed >> 4], axis=1).reshape(64, 256)
    assert np.all(dq == np.vectorize(O.e2m1_modelopt)(codes).astype(np.float32) *
                  (np.repeat(s_dec, 16, axis=1).astype(np.float32) * g[0]))


def test_nvfp4_quantize_zero_and_nonfinite():
    packed, scales, g = O.nvfp4_quantize(np.zeros((2, 32), np.float32))
    assert not packed.any() and not scales.any() and not g.any()
    bad = np.zeros((2, 32), np.float32)
    bad[1, 3] = np.inf
    with pytest.raises(ValueError):
        O.nvfp4_quantize(bad)


# ---- ModelOpt / Qwen fixture structure -------------------------------------------------
def _f32(bits: int) -> float:
    return float(np.uint32(bits).view(np.float32))


def _decoded_products(global_scale: np.float32) -> set:
    """All values RN(E2M1[c] * RN(e4m3(s) * g)) for valid c, s (checkpoint.rs:420)."""
    e = np.array([O.e2m1_modelopt(c) for c in range(16)], np.float32)
    s = np.array([O.e4m3(b) for b in range(256) if (b & 0x7F) != 0x7F], np.float32)
    sg = (s * global_scale).astype(np.float32)
    return set((e[:, None] * sg[None, :]).astype(np.float32).view(np.uint32).ravel().tolist())


def _nvfp4_structure_ok(samples) -> bool:
    vals = [np.uint32(s["bits"]).view(np.float32) for s in samples]
    nz = [v for v in vals if v != 0]
    if not nz:
        return True
    v0 = np.float32(abs(nz[0]))
    e_vals = [0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    s_vals = [O.e4m3(b) for b in range(1, 0x7F)]
    for e in e_vals:
        for s in s_vals:
            g0 = np.float32(v0 / np.float32(e) / np.float32(s))
            for g in _ulp_neighbours(g0, 2):
                # quick reject on the first value before building the full table
                if np.float32(np.float32(e) * np.float32(np.float32(s) * g)) != v0:
                    continue
                table = _decoded_products(g)
                if all(int(np.float32(v).view(np.uint32)) in table for v in vals):
                    return True
    return False


def _ulp_neighbours(x: np.float32, n: int) -> list:
    out, up, down = [np.float32(x)], np.float32(x), np.float32(x)
    for _ in range(n):
        up = np.nextafter(up, np.float32(np.inf))
        down = np.nextafter(down, np.float32(-np.inf))
        out += [up, down]
    return out


def _fp8_scalar_structure_ok(samples) -> bool:
    vals = [np.uint32(s["bits"]).view(np.float32) for s in samples]
    nz = [v for v in vals if v != 0]
    if not nz:
        return True
    v0 = np.float32(abs(nz[0]))
    codes = np.array([O.e4m3(b) for b in range(256) if (b & 0x7F) != 0x7F], np.float32)
    for w in codes[codes > 0]:
        s0 = np.float32(v0 / w)
        for s in (np.nextafter(s0, np.float32(-np.inf)), s0, np.nextafter(s0, np.float32(np.inf))):
            s = np.float32(s)
            prods = set((codes * s).astype(np.float32).view(np.uint32).tolist())
            if all(int(np.float32(v).view(np.uint32)) in prods for v in vals):
                return True
    return False


def test_modelopt_dequant_fixture_is_reachable_by_the_decode_tables():
    data = json.loads((GOLDEN / "dequant_samples.json").read_text())
    by_tensor: dict = {}
    for s in data["nvfp4_or_fp8_modelopt"]:
        by_tensor.setdefault(s["tensor"], []).append(s)
    nvfp4 = 0
    for name, samples in by_tensor.items():
        ok4 = _nvfp4_structure_ok(samples)
        nvfp4 += ok4
        assert ok4 or _fp8_scalar_structure_ok(samples), name
    assert nvfp4 >= 2  # the routed/shared expert projections are NVFP4


def test_fp8_block_fixture_is_reachable_by_e4m3_times_bf16():
    data = json.loads((GOLDEN / "dequant_samples.json").read_text())
    codes = [O.e4m3(b) for b in range(256) if (b & 0x7F) != 0x7F]
    for s in data["fp8_block"]:
        v = np.uint32(s["bits"]).view(np.float32)
        if v == 0:
            continue
        found = False
        for w in codes:
            if w == 0:
                continue
            q = np.float32(v / np.float32(w))
            b = O.bf16_bits(np.array([q], np.float32))[0]
            for d in (-1, 0, 1):
                sc = O.bf16_to_f32(np.array([int(b) + d], np.uint16))[0]
                if np.float32(np.float32(w) * sc) == v:
                    found = True
                    break
            if found:
                break
        assert found, s


# ---- MoE layout -----------------------------------------------------------------------------
def sorted_layout(indices, experts, top_k, tile_rows):
    """kernels src/moe.rs:865-901: the layout from a stable sort by expert."""
    entries = [(int(e), t, j) for t in range(len(indices) // top_k)
               for j, e in enumerate(indices[t * top_k:(t + 1) * top_k])]
    entries.sort(key=lambda x: x[0])
    token_rows, tile_experts = [], []
    inverse = [0] * len(indices)
    ranges = []
    cursor = 0
    for expert in range(experts):
        start, count = len(token_rows), 0
        while cursor < len(entries) and entries[cursor][0] == expert:
            _, token, slot = entries[cursor]
            inverse[token * top_k + slot] = len(token_rows)
            token_rows.append(token)
            cursor += 1
            count += 1
        padded = -(-count // tile_rows) * tile_rows
        token_rows += [-1] * (start + padded - len(token_rows))
        tile_experts += [expert] * (padded // tile_rows)
        ranges.append((start, count))
    return token_rows, tile_experts, inverse, ranges


@pytest.mark.parametrize("experts,top_k,tokens,tile_rows",
                         [(4, 1, 1, 1), (8, 3, 17, 4), (64, 8, 300, 32), (257, 9, 1000, 32), (5, 5, 40, 64)])
def test_counting_layout_matches_a_stable_sort_by_expert(experts, top_k, tokens, tile_rows):
    """kernels src/moe.rs:903-941, with the same LCG."""
    import firepit_b200 as F
    state = 0x9E3779B97F4A7C15

    def nxt(bound):
        nonlocal state
        state = (state * 6364136223846793005 + 1442695040888963407) & ((1 << 64) - 1)
        return (state >> 33) % bound

    indices = []
    for _ in range(tokens):
        ids = []
        while len(ids) < top_k:
            i = nxt(experts)
            if i not in ids:
                ids.append(i)
        indices += ids
    dims = F.MoeDims.new(32, 32, 32, experts, top_k)
    layout = F.PrefillLayout.parse(indices, [0.5] * len(indices), dims, tile_rows)
    tr, te, inv, rg = sorted_layout(indices, experts, top_k, tile_rows)
    assert layout.token_rows.tolist() == tr
    assert layout.tile_experts.tolist() == te
    assert layout.inverse.tolist() == inv
    assert layout.ranges == rg
    assert layout.tokens == tokens
