"""FP8 host logic and oracle pins (no GPU).

* The e4m3 value table of the reference's FP8 tests (fp8_oracle.rs:122-131)
  decodes to the listed values through the oracle and the library's codec.
* HostFp8Matrix validation returns the reference's errors
  (weights/fp8.rs:30-112).
* The oracle's quantizer (no reference counterpart) is pinned by properties:
  every quantized value is within half an e4m3 step of the input, grid values
  are fixed points, and the scale is amax/448.
"""
import numpy as np
import pytest

import refcases as R
from oracle import oracle as O


def test_fp8_value_table_decodes():
    import firepit_b200 as F
    for bits, value in R.FP8_VALUES:
        assert O.lib.orc_e4m3(bits) == np.float32(value)
        assert F._native.lib.fpb_e4m3_to_f32(bits) == np.float32(value)


def test_fp8_validation_errors():
    import firepit_b200 as F
    bits = np.zeros(256 * 256, np.uint8)
    m = F.HostFp8Matrix.from_parts(bits, np.ones(4, np.float32), 256, 256, 128, 128)
    assert m.scaling == F.Fp8Scaling.blocks(128, 128)
    with pytest.raises(F.FormatError, match="invalid FP8 scale grid"):
        F.HostFp8Matrix.from_parts(bits, np.ones(3, np.float32), 256, 256, 128, 128)
    with pytest.raises(F.FormatError, match="invalid FP8 scale grid"):
        F.HostFp8Matrix.from_parts(bits, np.ones(4, np.float32), 256, 256, 96, 128)
    with pytest.raises(F.FormatError, match="one value per row"):
        F.HostFp8Matrix.with_row_scales(bits, np.ones(255, np.float32), 256, 256)
    with pytest.raises(F.FormatError, match="invalid FP8 matrix or scales"):
        F.HostFp8Matrix.from_parts(bits, np.array([1, 1, np.inf, 1], np.float32), 256, 256, 128, 128)
    with pytest.raises(F.FormatError, match="invalid FP8 matrix or scales"):
        F.HostFp8Matrix.with_row_scales(np.zeros(256 * 48, np.uint8), np.ones(256, np.float32), 256, 48)
    with pytest.raises(F.FormatError, match="invalid FP8 matrix or scales"):
        F.HostFp8Matrix.with_row_scales(bits[:-1], np.ones(256, np.float32), 256, 256)
    z = F.HostFp8Matrix.zeros(128, 256, F.Fp8Scaling.rows())
    s = F.HostFp8Matrix.stack([z, z])
    assert s.rows == 256 and s.scales.size == 256
    with pytest.raises(F.FormatError, match="differ"):
        F.HostFp8Matrix.stack([z, F.HostFp8Matrix.zeros(128, 256, F.Fp8Scaling.blocks(128, 128))])


@pytest.mark.parametrize("block", [(128, 128), (0, 0), (64, 32)])
def test_fp8_oracle_quantizer_properties(block):
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((256, 256)) * 0.02).astype(np.float32)
    w[3, :] = 0.0
    bits, scales = O.fp8_quantize(w, *block)
    deq = O.fp8_dequantize(bits, scales, *block)
    bn, bk = block if block != (0, 0) else (1, 256)
    for b in range(scales.size):
        r0, c0 = (b // (256 // bk)) * bn, (b % (256 // bk)) * bk
        blk = w[r0:r0 + bn, c0:c0 + bk]
        assert scales[b] == np.float32(np.abs(blk).max()) / np.float32(448.0)
    # |w/s - e4m3(w/s)| <= half a step: step = 2^(e-3) for normals, 2^-9 for subnormals
    full = np.repeat(np.repeat(scales.reshape(256 // bn, 256 // bk), bn, 0), bk, 1)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(full > 0, w / full, 0).astype(np.float32)
    qd = np.array([O.lib.orc_e4m3(int(v)) for v in bits.reshape(-1)], np.float32).reshape(256, 256)
    step = np.where(np.abs(q) >= 2.0 ** -6, 2.0 ** (np.floor(np.log2(np.maximum(np.abs(q), 1e-30))) - 3), 2.0 ** -9)
    assert np.all(np.abs(q - qd) <= step / 2 + 1e-12)
    assert np.all(deq[3, :] == 0.0) and np.all(bits[3, :] == 0)
    # grid values are fixed points: quantize(dequantize(q)) == q, same scales
    bits2, scales2 = O.fp8_quantize(deq, *block)
    assert np.array_equal(scales2, scales) and np.array_equal(bits2, bits)
