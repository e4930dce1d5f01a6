"""Weights loaded from safetensors checkpoints through to the kernels: a
ModelOpt-format NVFP4 projection and its stacked experts into the decode GEMV,
a Qwen-format FP8 block-scaled projection into the FP8 GEMM, each against the
oracle on the loaded parts (crates/firepit/src/model.rs:554-660 then
gemv/mod.rs:74-123, gemm/mod.rs:424-442)."""
import json

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu
REL_FROB_TOL = 1e-3


@pytest.fixture(scope="module")
def torch():
    import torch as t
    return t


@pytest.fixture(scope="module")
def F(torch):
    import firepit_b200
    return firepit_b200


def _save(torch, path, tensors):
    from safetensors.torch import save_file
    save_file(tensors, str(path))


def test_modelopt_nvfp4_checkpoint_to_gemv(F, torch, tmp_path):
    rows, cols, experts = 1024, 2048, 3
    tensors, names = {}, []
    for e in range(experts):
        w = F.synth_normal((rows, cols), seed=e, stream_id=1, std=0.02)
        h = F.Nvfp4Matrix.quantize(w, rows).to_host()  # one global per expert, as ModelOpt stores it
        base = f"model.layers.0.mlp.experts.{e}.down_proj"
        tensors[f"{base}.weight"] = torch.from_numpy(h.packed.reshape(rows, cols // 2).copy())
        tensors[f"{base}.weight_scale"] = torch.from_numpy(h.scales.reshape(rows, cols // 16).copy()).view(
            torch.float8_e4m3fn)
        tensors[f"{base}.weight_scale_2"] = torch.tensor(float(h.row_scales[0]), dtype=torch.float32)
        names.append(f"{base}.weight")
    _save(torch, tmp_path / "experts.safetensors", tensors)
    (tmp_path / "model.safetensors.index.json").write_text(
        json.dumps({"weight_map": {n: "experts.safetensors" for n in tensors}}))
    ck = F.Checkpoint.open(tmp_path)
    stacked = F.load_experts(ck, names, (rows, cols), F.WeightFormat.NVFP4)
    m = stacked.upload()
    x = O.bf16_to_f32(O.bf16_bits(O.synth_normal(cols, seed=0, stream=0)))
    xt = torch.from_numpy(x.reshape(1, cols)).cuda().to(torch.bfloat16)
    y = torch.full((1, experts * rows), float("nan"), dtype=torch.float32, device="cuda")
    F.gemv(m, xt, y).submit(F.Eager())
    assert F.device_error() == 0
    y_ref = O.nvfp4_gemv_f32(stacked.packed, stacked.scales, stacked.row_scales, experts * rows, cols, x)[0]
    assert O.rel_frobenius(y.cpu().numpy()[0], y_ref) <= REL_FROB_TOL
    e64, mag = O.nvfp4_gemv_f64(stacked.packed, stacked.scales, stacked.row_scales, experts * rows, cols, x)
    assert O.inner_product_excess(y.cpu().numpy(), e64, mag, cols + 2) <= 1.0


def test_qwen_fp8_checkpoint_to_gemm(F, torch, tmp_path):
    m_rows, rows, cols = 256, 1024, 2048
    w = F.synth_normal((rows, cols), seed=3, stream_id=1, std=0.02)
    bits, scales = F.quantize_fp8(w, F.Fp8Scaling(128, 128))
    # weight_scale_inv is stored in bf16: round the scales to bf16 first
    sb = O.bf16_bits(scales.cpu().numpy().astype(np.float32))
    _save(torch, tmp_path / "a.safetensors", {
        "model.layers.0.mlp.gate_proj.weight": bits.view(rows, cols).cpu().view(torch.float8_e4m3fn),
        "model.layers.0.mlp.gate_proj.weight_scale_inv": torch.from_numpy(
            sb.view(np.int16).reshape(rows // 128, cols // 128).copy()).view(torch.bfloat16)})
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {
        "model.layers.0.mlp.gate_proj.weight": "a.safetensors",
        "model.layers.0.mlp.gate_proj.weight_scale_inv": "a.safetensors"}}))
    (tmp_path / "config.json").write_text(json.dumps({"quantization_config": {
        "quant_method": "fp8", "fmt": "e4m3", "activation_scheme": "dynamic", "weight_block_size": [128, 128],
        "modules_to_not_convert": []}}))
    q = F.Quantization.open(tmp_path)
    ck = F.Checkpoint.open(tmp_path)
    name = "model.layers.0.mlp.gate_proj.weight"
    h = F.load_weight(ck, name, (rows, cols), q.format(name))
    W = h.upload()
    x = F.synth_normal((m_rows, cols), seed=4, stream_id=2, dtype=torch.bfloat16)
    y = torch.full((m_rows, rows), float("nan"), dtype=torch.float32, device="cuda")
    F.fp8_gemm(W, x, y).submit(F.Eager())
    assert F.device_error() == 0
    a_bits, a_s = O.fp8_quantize(x.float().cpu().numpy())
    e, mag = O.fp8_gemm_f64(a_bits, a_s, h.bits.reshape(rows, cols), h.scales, 128, 128)
    got = y.cpu().numpy().astype(np.float64)
    assert O.rel_frobenius(got, e) <= REL_FROB_TOL
    assert np.all(np.abs(got - e) <= (O.gamma_tilde(cols + 1) + 2.0 ** -16) * mag + 1e-300)
