"""Checkpoint loading on the CPU: the C library's safetensors reader, the
quantization configs and the weight loaders (crates/firepit/src/
checkpoint.rs, config.rs, model.rs:447-660).

Fixtures are written by the `safetensors` package (an independent writer).
The dequantization checks restate the reference's own tests
(checkpoint.rs:342-420: fp8_to_f32, ModelOpt's E2M1 table with +0 for code
0b1000, value = E2M1[c] * (scale * global); FP8 blocks: weight * bf16 scale)
and compare them bit for bit with the oracle on the loaded matrices."""
import json
import struct

import numpy as np
import pytest

torch = pytest.importorskip("torch")
st_torch = pytest.importorskip("safetensors.torch")

import firepit_b200 as F  # noqa: E402
from firepit_b200 import checkpoint as CK  # noqa: E402
from oracle import oracle as O  # noqa: E402

# ModelOpt's e2m1_values (checkpoint.rs:384-387): 0b1000 decodes as +0.
E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, 0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], np.float32)


def fp8_to_f32(bits: np.ndarray) -> np.ndarray:
    """checkpoint.rs:342-352."""
    bits = bits.astype(np.int64)
    sign = np.where(bits & 0x80, -1.0, 1.0).astype(np.float32)
    e = (bits >> 3) & 0x0F
    f = (bits & 0x07).astype(np.float32)
    sub = sign * f * np.float32(2.0 ** -9)
    norm = sign * (np.float32(1.0) + f / np.float32(8.0)) * np.exp2((e - 7).astype(np.float32))
    return np.where(e == 0, sub, norm).astype(np.float32)


def _rng(seed):
    return np.random.default_rng(seed)


def _nvfp4_parts(rows, cols, seed):
    r = _rng(seed)
    packed = r.integers(0, 256, rows * cols // 2, dtype=np.uint8)
    scales = r.integers(0, 0x7F, rows * cols // 16, dtype=np.uint8)  # finite e4m3 (no 0x7F / 0xFF NaN)
    glob = np.float32(r.uniform(1e-4, 1e-2))
    return packed, scales, glob


def _write(path, tensors: dict, metadata=None):
    st_torch.save_file(tensors, str(path), metadata=metadata)


def _t_u8(a, shape):
    return torch.from_numpy(np.ascontiguousarray(a).reshape(shape).copy())


def _t_e4m3(a, shape):
    return _t_u8(a, shape).view(torch.float8_e4m3fn)


def _t_bf16_bits(bits, shape):
    return torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16).reshape(shape).copy()).view(
        torch.bfloat16)


@pytest.fixture
def nvfp4_file(tmp_path):
    rows, cols = 64, 256
    packed, scales, glob = _nvfp4_parts(rows, cols, 1)
    path = tmp_path / "nvfp4.safetensors"
    _write(path, {
        "layer.mlp.down_proj.weight": _t_u8(packed, (rows, cols // 2)),
        "layer.mlp.down_proj.weight_scale": _t_e4m3(scales, (rows, cols // 16)),
        "layer.mlp.down_proj.weight_scale_2": torch.tensor(glob, dtype=torch.float32),
        "norm.weight": torch.arange(8, dtype=torch.float32).to(torch.bfloat16),
        "ids": torch.arange(-3, 3, dtype=torch.int32),
    }, metadata={"format": "pt", "note": "café \"quoted\""})
    return path, rows, cols, packed, scales, glob


def test_safetensors_reader_matches_the_writer(nvfp4_file):
    path, rows, cols, packed, scales, glob = nvfp4_file
    with CK.SafetensorsFile(path) as f:
        assert set(f.names()) == {"layer.mlp.down_proj.weight", "layer.mlp.down_proj.weight_scale",
                                  "layer.mlp.down_proj.weight_scale_2", "norm.weight", "ids"}
        assert f.metadata("format") == "pt"
        assert f.metadata("note") == "café \"quoted\""
        assert f.metadata("absent") is None
        assert f.has_tensor("ids") and not f.has_tensor("nope")
        assert f.info("layer.mlp.down_proj.weight") == ("U8", (rows, cols // 2), rows * cols // 2)
        shape, b = f.tensor_nvfp4("layer.mlp.down_proj.weight")
        assert shape == (rows, cols // 2) and np.array_equal(b, packed)
        shape, s = f.tensor_fp8("layer.mlp.down_proj.weight_scale")
        assert shape == (rows, cols // 16) and np.array_equal(s, scales)
        assert np.float32(f.scalar_f32("layer.mlp.down_proj.weight_scale_2")) == glob
        shape, v = f.tensor("norm.weight")  # BF16 as f32 (checkpoint.rs:193-212)
        assert shape == (8,) and np.array_equal(v, np.arange(8, dtype=np.float32))
        shape, i = f.tensor_i32("ids")
        assert shape == (6,) and np.array_equal(i, np.arange(-3, 3))
        rs, row = f.row("norm.weight", 0)
        assert rs == () and row.tolist() == [0.0]


def test_safetensors_reader_errors(nvfp4_file, tmp_path):
    path = nvfp4_file[0]
    with CK.SafetensorsFile(path) as f:
        with pytest.raises(CK.CheckpointError, match="unknown tensor nope"):
            f.info("nope")
        with pytest.raises(CK.CheckpointError, match="expected F32, got U8"):
            f.scalar_f32("layer.mlp.down_proj.weight")
        with pytest.raises(CK.CheckpointError, match="expected an F32 scalar"):
            _write(tmp_path / "v.safetensors", {"v": torch.zeros(2)})
            CK.SafetensorsFile(tmp_path / "v.safetensors").scalar_f32("v")
        with pytest.raises(CK.CheckpointError, match="unsupported dtype U8"):
            f.tensor("layer.mlp.down_proj.weight")
        with pytest.raises(CK.CheckpointError, match="row 9 out of 8"):
            f.row("norm.weight", 9)
    with pytest.raises(OSError):
        CK.SafetensorsFile(tmp_path / "missing.safetensors")
    data = path.read_bytes()
    (tmp_path / "trunc.safetensors").write_bytes(data[:-1])
    with pytest.raises(CK.CheckpointError, match="disagree"):
        CK.SafetensorsFile(tmp_path / "trunc.safetensors")

    def raw(header: bytes, body: bytes = b""):
        p = tmp_path / "raw.safetensors"
        p.write_bytes(struct.pack("<Q", len(header)) + header + body)
        return p

    with pytest.raises(CK.CheckpointError, match="header length"):
        p = tmp_path / "long.safetensors"
        p.write_bytes(struct.pack("<Q", 1 << 40) + b"{}")
        CK.SafetensorsFile(p)
    for bad, msg in [(b"{", "header JSON"), (b"[]", "not an object"), (b'{"a": 1}', "no dtype"),
                     (b'{"a": {"dtype": "Q9", "shape": [1], "data_offsets": [0, 1]}}', "unsupported dtype"),
                     (b'{"a": {"dtype": "U8", "shape": [2], "data_offsets": [0, 1]}}', "disagree"),
                     (b'{"a": {"dtype": "U8", "shape": [-1], "data_offsets": [0, 1]}}', "bad shape"),
                     (b'{"__metadata__": {"k": 1}}', "not a string"), (b'{} x', "trailing")]:
        with pytest.raises(CK.CheckpointError, match=msg):
            CK.SafetensorsFile(raw(bad, b"\0" * 4))
    # escapes, surrogate pairs and padding are accepted
    hdr = json.dumps({"näme\U0001F600": {"dtype": "U8", "shape": [2, 2], "data_offsets": [0, 4]}},
                     ensure_ascii=True).encode() + b"    "
    with CK.SafetensorsFile(raw(hdr, bytes([1, 2, 3, 4]))) as f:
        assert f.names() == ["näme\U0001F600"]
        assert f.tensor_nvfp4("näme\U0001F600")[1].tolist() == [1, 2, 3, 4]


def test_nvfp4_load_and_modelopt_dequant_bits(nvfp4_file, tmp_path):
    path, rows, cols, packed, scales, glob = nvfp4_file
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps(
        {"weight_map": {n: path.name for n in CK.SafetensorsFile(path).names()}}))
    ck = CK.Checkpoint.open(tmp_path)
    name = "layer.mlp.down_proj.weight"
    h = CK.load_weight(ck, name, (rows, cols), CK.WeightFormat.NVFP4)
    assert isinstance(h, F.HostNvfp4Matrix)
    assert np.array_equal(h.packed, packed) and np.array_equal(h.scales, scales)
    assert np.all(h.row_scales == glob)
    # checkpoint.rs:402-420, element by element
    col = np.arange(cols)
    pair = packed.reshape(rows, cols // 2)[:, col // 2]
    code = np.where(col % 2 == 0, pair & 0xF, pair >> 4)
    scale = fp8_to_f32(scales.reshape(rows, cols // 16)[:, col // 16])
    ref = E2M1[code] * (scale * glob)
    got = O.nvfp4_dequantize(h.packed, h.scales, h.row_scales, rows, cols)
    assert np.array_equal(ref.view(np.uint32), got.reshape(rows, cols).view(np.uint32))
    # the format must agree with the stored scale tensors
    with pytest.raises(CK.CheckpointError, match="contradict"):
        CK.load_weight(ck, name, (rows, cols), CK.WeightFormat.FP8_TENSOR)
    with pytest.raises(CK.CheckpointError, match="invalid"):
        CK.load_weight(ck, name, (rows, cols * 2), CK.WeightFormat.NVFP4)


def test_fp8_block_and_tensor_loads(tmp_path):
    rows, cols, bn, bk = 256, 384, 128, 128
    r = _rng(2)
    bits = r.integers(0, 256, rows * cols, dtype=np.uint8)
    bits[(bits & 0x7F) == 0x7F] = 0x11  # no NaN encodings
    sinv = O.bf16_bits(r.uniform(1e-4, 1e-1, (rows // bn) * (cols // bk)).astype(np.float32))
    _write(tmp_path / "a.safetensors", {
        "m.q_proj.weight": _t_e4m3(bits, (rows, cols)),
        "m.q_proj.weight_scale_inv": _t_bf16_bits(sinv, (rows // bn, cols // bk)),
        "m.o_proj.weight": _t_e4m3(bits, (rows, cols)),
        "m.o_proj.weight_scale": torch.tensor(0.25, dtype=torch.float32),
    })
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {
        "m.q_proj.weight": "a.safetensors", "m.q_proj.weight_scale_inv": "a.safetensors",
        "m.o_proj.weight": "a.safetensors", "m.o_proj.weight_scale": "a.safetensors",
        "m.k_proj.weight": "b.safetensors"}}))
    ck = CK.Checkpoint.open(tmp_path)
    h = CK.load_weight(ck, "m.q_proj.weight", (rows, cols), CK.WeightFormat.fp8_blocks(bn, bk))
    assert isinstance(h, F.HostFp8Matrix) and (h.scaling.block_n, h.scaling.block_k) == (bn, bk)
    # checkpoint.rs:375-379: weight * bf16 scale, in f32
    sgrid = CK.bf16_bits_to_f32(sinv).reshape(rows // bn, cols // bk)
    ref = fp8_to_f32(bits.reshape(rows, cols)) * np.repeat(np.repeat(sgrid, bn, 0), bk, 1)
    got = O.fp8_dequantize(h.bits.reshape(rows, cols), h.scales.reshape(rows // bn, cols // bk), bn, bk)
    assert np.array_equal(ref.astype(np.float32).view(np.uint32), np.asarray(got, np.float32).view(np.uint32))
    t = CK.load_weight(ck, "m.o_proj.weight", (rows, cols), CK.WeightFormat.FP8_TENSOR)
    assert t.scaling.is_rows and np.all(t.scales == np.float32(0.25))
    with pytest.raises(CK.CheckpointError, match="which is not downloaded"):
        ck.stored("m.k_proj.weight")
    with pytest.raises(CK.CheckpointError, match="unknown tensor"):
        ck.stored("m.v_proj.weight")
    assert ck.stored("m.q_proj.weight") == ("F8_E4M3", (rows, cols))


def test_expert_stacking_keeps_per_row_globals(tmp_path):
    rows, cols = 32, 128
    tensors, parts = {}, []
    for e in range(3):
        packed, scales, glob = _nvfp4_parts(rows, cols, 10 + e)
        base = f"model.layers.0.mlp.experts.{e}.down_proj"
        tensors[f"{base}.weight"] = _t_u8(packed, (rows, cols // 2))
        tensors[f"{base}.weight_scale"] = _t_e4m3(scales, (rows, cols // 16))
        tensors[f"{base}.weight_scale_2"] = torch.tensor(glob, dtype=torch.float32)
        parts.append((packed, scales, glob))
    _write(tmp_path / "s.safetensors", tensors)
    (tmp_path / "model.safetensors.index.json").write_text(
        json.dumps({"weight_map": {n: "s.safetensors" for n in tensors}}))
    ck = CK.Checkpoint.open(tmp_path)
    names = [f"model.layers.0.mlp.experts.{e}.down_proj.weight" for e in range(3)]
    h = CK.load_experts(ck, names, (rows, cols), CK.WeightFormat.NVFP4)
    assert h.rows == 3 * rows
    for e, (packed, scales, glob) in enumerate(parts):
        assert np.all(h.row_scales[e * rows:(e + 1) * rows] == glob)
        assert np.array_equal(h.packed[e * rows * cols // 2:(e + 1) * rows * cols // 2], packed)
    with pytest.raises(CK.CheckpointError, match="mix formats"):
        CK.stack_weights([h, CK.HostBf16Weight(np.zeros((1, cols), np.uint16), 1, cols)])


def test_expert_loader_names_the_corrupt_expert(tmp_path):
    """One expert with a NaN block scale (0x7f) among several: the error names
    that expert's tensor, as a per-expert load would."""
    rows, cols = 32, 128
    tensors = {}
    for e in range(4):
        packed, scales, glob = _nvfp4_parts(rows, cols, 20 + e)
        if e == 2:
            scales = scales.copy()
            scales[5] = 0x7F
        base = f"model.layers.0.mlp.experts.{e}.down_proj"
        tensors[f"{base}.weight"] = _t_u8(packed, (rows, cols // 2))
        tensors[f"{base}.weight_scale"] = _t_e4m3(scales, (rows, cols // 16))
        tensors[f"{base}.weight_scale_2"] = torch.tensor(glob, dtype=torch.float32)
    _write(tmp_path / "s.safetensors", tensors)
    (tmp_path / "model.safetensors.index.json").write_text(
        json.dumps({"weight_map": {n: "s.safetensors" for n in tensors}}))
    ck = CK.Checkpoint.open(tmp_path)
    names = [f"model.layers.0.mlp.experts.{e}.down_proj.weight" for e in range(4)]
    with pytest.raises(CK.FormatError, match=r"experts\.2\.down_proj\.weight"):
        CK.load_experts(ck, names, (rows, cols), CK.WeightFormat.NVFP4)


def test_quantization_configs(tmp_path):
    q = CK.Quantization.parse({"quantization_config": {
        "quant_method": "fp8", "fmt": "e4m3", "activation_scheme": "dynamic", "weight_block_size": [128, 128],
        "modules_to_not_convert": ["lm_head"]}}, None)
    assert q.format("model.layers.0.mlp.gate_proj.weight") == CK.WeightFormat.fp8_blocks(128, 128)
    assert q.format("lm_head.weight") == CK.WeightFormat.BF16
    for bad in ([128], [100, 128], [128, 96], [0, 128]):
        with pytest.raises(CK.CheckpointError):
            CK.Fp8Config.parse({"fmt": "e4m3", "activation_scheme": "dynamic", "weight_block_size": bad,
                                "modules_to_not_convert": []})
    with pytest.raises(CK.CheckpointError, match="unsupported FP8 quantization"):
        CK.Fp8Config.parse({"fmt": "e5m2", "activation_scheme": "dynamic"})
    mo = {"producer": {"name": "modelopt"}, "quantization": {"quant_algo": "MIXED_PRECISION", "quantized_layers": {
        "model.layers.0.mlp.experts": {"quant_algo": "W4A16_NVFP4", "group_size": 16},
        "model.layers.0.self_attn.q_proj": {"quant_algo": "FP8"}}}}
    q = CK.Quantization.parse({"quantization_config": {"quant_method": "modelopt"}}, mo)
    assert q.format("model.layers.0.mlp.experts.17.up_proj.weight") == CK.WeightFormat.NVFP4
    assert q.format("model.layers.0.self_attn.q_proj.weight") == CK.WeightFormat.FP8_TENSOR
    assert q.format("model.layers.0.self_attn.k_proj.weight") == CK.WeightFormat.BF16
    with pytest.raises(CK.CheckpointError, match="disagree"):
        CK.Quantization.parse({"quantization_config": {"quant_method": "fp8"}}, mo)
    with pytest.raises(CK.CheckpointError, match="unsupported ModelOpt layer"):
        CK.ModelOptConfig.parse({"producer": {"name": "modelopt"}, "quantization": {
            "quant_algo": "MIXED_PRECISION", "quantized_layers": {"x": {"quant_algo": "W4A16_NVFP4",
                                                                        "group_size": 32}}}})
    assert CK.Quantization.parse({}, None) is None
    (tmp_path / "config.json").write_text(json.dumps({"quantization_config": {"quant_method": "modelopt"}}))
    (tmp_path / "hf_quant_config.json").write_text(json.dumps(mo))
    assert CK.Quantization.open(tmp_path).format("model.layers.0.mlp.experts.3.down_proj.weight") == \
        CK.WeightFormat.NVFP4


def test_verify_formats(nvfp4_file, tmp_path):
    path = nvfp4_file[0]
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps(
        {"weight_map": {n: path.name for n in CK.SafetensorsFile(path).names()}}))
    ck = CK.Checkpoint.open(tmp_path)
    mo = CK.Quantization(CK.ModelOptConfig({"layer.mlp.down_proj": CK.WeightFormat.NVFP4}))
    report = CK.verify_formats(ck, mo)
    assert [r[0] for r in report] == ["layer.mlp.down_proj.weight", "norm.weight"]
    assert report[0][1] == CK.WeightFormat.NVFP4 and report[1][1] == CK.WeightFormat.BF16
    with pytest.raises(CK.CheckpointError, match="contradict"):
        CK.verify_formats(ck, None)
