"""Checkpoint loading for the quantized-matmul path.

Mirrors the reference's host-side loader of NVFP4 / FP8 weights:

* ``SafetensorsFile`` / ``Checkpoint`` — crates/firepit/src/checkpoint.rs:57-339
  (one safetensors shard; a directory with ``model.safetensors.index.json``).
  The file format is parsed by the C library (``fpb_safetensors_*``).
* ``WeightFormat``, ``Fp8Config``, ``ModelOptConfig``, ``Quantization`` —
  crates/firepit/src/config.rs:11-160 (which format each weight is stored in,
  from ``config.json``'s ``quantization_config`` and ModelOpt's
  ``hf_quant_config.json``).
* ``check_companions``, ``load_weight``, ``stack_weights``, ``verify_formats``
  — crates/firepit/src/model.rs:447-515, 554-660 (scale tensors that must or
  must not accompany a weight, building ``HostNvfp4Matrix`` /
  ``HostFp8Matrix`` from the stored parts, stacking projections or experts
  with per-row globals kept).

On-disk formats: ModelOpt NVFP4 stores ``<name>.weight`` as U8 [N, K/2] (two
e2m1 codes per byte, even column in the low nibble), ``.weight_scale`` as
F8_E4M3 [N, K/16] and ``.weight_scale_2`` as an F32 scalar (the global);
ModelOpt FP8 stores F8_E4M3 [N, K] with an F32 scalar ``.weight_scale``;
Qwen FP8 stores F8_E4M3 [N, K] with BF16 [N/bn, K/bk] ``.weight_scale_inv``.
"""
from __future__ import annotations

import ctypes as C
import json
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import _native as N
from .fp8 import HostFp8Matrix
from .gemm import DEFAULT_GEMM_TILE
from .gemv import DEFAULT_GEMV_TILE
from .weights import NVFP4_GROUP, Q8_BLOCK, FormatError, HostNvfp4Matrix

# Stored dtype names, indexed by the C ABI's FPB_ST_* codes.
DTYPES = ("BOOL", "U8", "I8", "F8_E5M2", "F8_E4M3", "I16", "U16", "F16", "BF16", "I32", "U32", "F32", "F64",
          "I64", "U64")
_CODE = {name: i for i, name in enumerate(DTYPES)}
_MAX_DIMS = 16


class CheckpointError(FormatError):
    """The reference loader's ``Err(..)`` (missing tensors, wrong dtypes or shapes)."""


def _raise(status: int) -> None:
    if status == N.FPB_ERR_IO:
        raise OSError(N.last_error())
    raise CheckpointError(N.last_error())


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 -> f32 (exact): the bf16 bits are the upper half of the f32."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


class SafetensorsFile:
    """checkpoint.rs:57-213."""

    def __init__(self, path: str | os.PathLike):
        self.path = str(path)
        h = C.c_void_p()
        st = N.lib.fpb_safetensors_open(os.fsencode(self.path), C.byref(h))
        if st != N.FPB_OK:
            _raise(st)
        self._h = h

    @classmethod
    def open(cls, path) -> "SafetensorsFile":
        return cls(path)

    def close(self) -> None:
        if getattr(self, "_h", None):
            N.lib.fpb_safetensors_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:  # pragma: no cover - interpreter shutdown
            pass

    def names(self) -> list[str]:
        return [N.lib.fpb_safetensors_name(self._h, i).decode() for i in range(N.lib.fpb_safetensors_count(self._h))]

    def metadata(self, key: str) -> str | None:
        """checkpoint.rs:78-84."""
        v = N.lib.fpb_safetensors_metadata(self._h, key.encode())
        return None if v is None else v.decode()

    def has_tensor(self, name: str) -> bool:
        """checkpoint.rs:86-88."""
        return bool(N.lib.fpb_safetensors_has(self._h, name.encode()))

    def info(self, name: str) -> tuple[str, tuple[int, ...], int]:
        """(dtype, shape, byte size) of a stored tensor (checkpoint.rs:187-191)."""
        dt, nd, nb = C.c_int(), C.c_int(), C.c_size_t()
        shape = (C.c_int64 * _MAX_DIMS)()
        st = N.lib.fpb_safetensors_info(self._h, name.encode(), C.byref(dt), shape, _MAX_DIMS, C.byref(nd),
                                        C.byref(nb))
        if st != N.FPB_OK:
            _raise(st)
        return DTYPES[dt.value], tuple(int(shape[i]) for i in range(nd.value)), int(nb.value)

    def _read(self, name: str, dtype: str, byte_begin: int, nbytes: int) -> np.ndarray:
        out = np.empty(nbytes, dtype=np.uint8)
        st = N.lib.fpb_safetensors_read(self._h, name.encode(), _CODE[dtype], byte_begin,
                                        out.ctypes.data if nbytes else None, nbytes)
        if st != N.FPB_OK:
            _raise(st)
        return out

    def bytes(self, name: str, dtype: str) -> tuple[tuple[int, ...], np.ndarray]:
        """checkpoint.rs:158-167: raw bytes after checking the stored dtype."""
        stored, shape, nbytes = self.info(name)
        if stored != dtype:
            raise CheckpointError(f"{name}: expected {dtype}, got {stored}")
        return shape, self._read(name, dtype, 0, nbytes)

    def tensor(self, name: str) -> tuple[tuple[int, ...], np.ndarray]:
        """checkpoint.rs:90-97 with read (:193-212): BF16 or F32 data as f32."""
        dtype, shape, nbytes = self.info(name)
        return shape, self._as_f32(name, dtype, self._read_any(name, dtype, 0, nbytes))

    def tensor_i32(self, name: str):
        """checkpoint.rs:99-109."""
        shape, b = self.bytes(name, "I32")
        return shape, b.view("<i4").copy()

    def tensor_bf16(self, name: str):
        """checkpoint.rs:111-121: bf16 bits (uint16)."""
        shape, b = self.bytes(name, "BF16")
        return shape, b.view("<u2").copy()

    def tensor_fp8(self, name: str):
        """checkpoint.rs:123-129: e4m3 bits (uint8)."""
        return self.bytes(name, "F8_E4M3")

    def tensor_nvfp4(self, name: str):
        """checkpoint.rs:131-137: packed e2m1 pairs (uint8)."""
        return self.bytes(name, "U8")

    def scalar_f32(self, name: str) -> float:
        """checkpoint.rs:139-145."""
        shape, b = self.bytes(name, "F32")
        if shape != () or b.size != 4:
            raise CheckpointError(f"{name}: expected an F32 scalar, got shape {list(shape)}")
        return float(b.view("<f4")[0])

    def row(self, name: str, row: int) -> tuple[tuple[int, ...], np.ndarray]:
        """checkpoint.rs:169-185: one row of a BF16 / F32 tensor as f32."""
        dtype, shape, _ = self.info(name)
        if not shape:
            raise CheckpointError("scalar tensor has no rows")
        rows, row_shape = shape[0], shape[1:]
        if row >= rows:
            raise CheckpointError(f"{name}: row {row} out of {rows}")
        width = int(np.prod(row_shape, dtype=np.int64)) if row_shape else 1
        size = {"BF16": 2, "F32": 4}.get(dtype)
        if size is None:
            raise CheckpointError(f"unsupported dtype {dtype}")
        return row_shape, self._as_f32(name, dtype, self._read(name, dtype, row * width * size, width * size))

    def _read_any(self, name, dtype, begin, nbytes):
        if dtype not in ("BF16", "F32"):
            raise CheckpointError(f"unsupported dtype {dtype}")
        return self._read(name, dtype, begin, nbytes)

    @staticmethod
    def _as_f32(name, dtype, b: np.ndarray) -> np.ndarray:
        if dtype == "BF16":
            return bf16_bits_to_f32(b.view("<u2"))
        return b.view("<f4").copy()


class Checkpoint:
    """checkpoint.rs:195-339: tensors of a sharded checkpoint directory."""

    def __init__(self, shard_of: dict[str, str], shards: dict[str, SafetensorsFile]):
        self.shard_of, self.shards = shard_of, shards

    @classmethod
    def open(cls, directory) -> "Checkpoint":
        d = Path(directory)
        with open(d / "model.safetensors.index.json") as f:
            index = json.load(f)
        weight_map = index.get("weight_map")
        if not isinstance(weight_map, dict):
            raise CheckpointError("index has no weight_map")
        shard_of = {name: shard for name, shard in weight_map.items() if isinstance(shard, str)}
        shards = {shard: SafetensorsFile(d / shard) for shard in sorted(set(shard_of.values()))
                  if (d / shard).exists()}
        return cls(shard_of, shards)

    def _shard(self, name: str) -> SafetensorsFile:
        shard = self.shard_of.get(name)
        if shard is None:
            raise CheckpointError(f"unknown tensor {name}")
        f = self.shards.get(shard)
        if f is None:
            raise CheckpointError(f"{name} is in {shard}, which is not downloaded")
        return f

    def tensor(self, name):
        return self._shard(name).tensor(name)

    def tensor_bf16(self, name):
        return self._shard(name).tensor_bf16(name)

    def tensor_fp8(self, name):
        return self._shard(name).tensor_fp8(name)

    def tensor_nvfp4(self, name):
        return self._shard(name).tensor_nvfp4(name)

    def scalar_f32(self, name) -> float:
        return self._shard(name).scalar_f32(name)

    def row(self, name, row):
        return self._shard(name).row(name, row)

    def contains(self, name: str) -> bool:
        return name in self.shard_of

    def names(self):
        return iter(self.shard_of)

    def stored(self, name: str) -> tuple[str, tuple[int, ...]]:
        """checkpoint.rs:245-248."""
        dtype, shape, _ = self._shard(name).info(name)
        return dtype, shape

    def stacked_bf16(self, first: str, second: str, rows: int, cols: int):
        """checkpoint.rs:250-265: gate and up stacked along rows."""
        gshape, gate = self.tensor_bf16(first)
        ushape, up = self.tensor_bf16(second)
        if gshape != (rows, cols) or ushape != gshape:
            raise CheckpointError("stacked matrix shape mismatch")
        return (2 * rows, cols), np.concatenate([gate, up])


# ---- formats (config.rs) -----------------------------------------------------------
@dataclass(frozen=True)
class WeightFormat:
    """config.rs:11-17: ``bf16``, ``fp8_blocks`` (block_n, block_k), ``fp8_tensor`` or ``nvfp4``."""

    kind: str
    block_n: int = 0
    block_k: int = 0

    BF16 = None  # filled in below
    FP8_TENSOR = None
    NVFP4 = None

    @classmethod
    def fp8_blocks(cls, block_n: int, block_k: int) -> "WeightFormat":
        return cls("fp8_blocks", block_n, block_k)


WeightFormat.BF16 = WeightFormat("bf16")
WeightFormat.FP8_TENSOR = WeightFormat("fp8_tensor")
WeightFormat.NVFP4 = WeightFormat("nvfp4")


@dataclass
class Fp8Config:
    """config.rs:19-80 (Qwen FP8 ``quantization_config``)."""

    block_n: int
    block_k: int
    excluded: frozenset

    @classmethod
    def parse(cls, value: dict) -> "Fp8Config":
        if value.get("fmt") != "e4m3" or value.get("activation_scheme") != "dynamic":
            raise CheckpointError("unsupported FP8 quantization configuration")
        blocks = value.get("weight_block_size")
        if not isinstance(blocks, list):
            raise CheckpointError("missing FP8 block size")
        if len(blocks) != 2:
            raise CheckpointError("FP8 block size must have two dimensions")
        for b, what in zip(blocks, ("rows", "columns")):
            if not isinstance(b, int) or isinstance(b, bool) or b < 0:
                raise CheckpointError(f"invalid FP8 block {what}")
        block_n, block_k = blocks
        if (block_n == 0 or block_k == 0 or block_n % DEFAULT_GEMM_TILE.n != 0
                or block_k % (DEFAULT_GEMV_TILE.blocks * Q8_BLOCK) != 0):
            raise CheckpointError("unsupported FP8 block shape")
        excluded = value.get("modules_to_not_convert")
        if not isinstance(excluded, list):
            raise CheckpointError("missing excluded FP8 modules")
        if not all(isinstance(m, str) for m in excluded):
            raise CheckpointError("invalid excluded FP8 module")
        return cls(block_n, block_k, frozenset(excluded))

    def format(self, module: str) -> WeightFormat:
        if module in self.excluded:
            return WeightFormat.BF16
        return WeightFormat.fp8_blocks(self.block_n, self.block_k)


@dataclass
class ModelOptConfig:
    """config.rs:82-122 (ModelOpt ``hf_quant_config.json``, MIXED_PRECISION)."""

    layers: dict

    @classmethod
    def parse(cls, value: dict) -> "ModelOptConfig":
        q = value.get("quantization") or {}
        if (value.get("producer") or {}).get("name") != "modelopt" or q.get("quant_algo") != "MIXED_PRECISION":
            raise CheckpointError("unsupported ModelOpt quantization configuration")
        layers_v = q.get("quantized_layers")
        if not isinstance(layers_v, dict):
            raise CheckpointError("missing ModelOpt quantized layers")
        layers = {}
        for module, layer in layers_v.items():
            algo = layer.get("quant_algo") if isinstance(layer, dict) else None
            group = layer.get("group_size") if isinstance(layer, dict) else None
            if algo == "FP8" and group is None:
                layers[module] = WeightFormat.FP8_TENSOR
            elif algo == "W4A16_NVFP4" and group == NVFP4_GROUP:
                layers[module] = WeightFormat.NVFP4
            else:
                raise CheckpointError(f"{module}: unsupported ModelOpt layer quantization")
        return cls(layers)

    def format(self, module: str) -> WeightFormat:
        base, sep, _ = module.partition(".experts.")
        key = f"{base}.experts" if sep else module
        return self.layers.get(key, WeightFormat.BF16)


class Quantization:
    """config.rs:124-160."""

    def __init__(self, config):
        self.config = config

    @classmethod
    def parse(cls, config: dict, modelopt: dict | None) -> "Quantization | None":
        qc = config.get("quantization_config")
        method = None
        if qc is not None:
            method = qc.get("quant_method") if isinstance(qc, dict) else None
            if not isinstance(method, str):
                raise CheckpointError("invalid quantization method")
        if method is None and modelopt is None:
            return None
        if method == "fp8" and modelopt is None:
            return cls(Fp8Config.parse(qc))
        if method == "modelopt" and modelopt is not None:
            return cls(ModelOptConfig.parse(modelopt))
        raise CheckpointError("quantization method and ModelOpt configuration disagree")

    @classmethod
    def open(cls, directory) -> "Quantization | None":
        """The quantization part of ModelConfig::open (config.rs:190-200)."""
        d = Path(directory)
        with open(d / "config.json") as f:
            config = json.load(f)
        modelopt = None
        if (d / "hf_quant_config.json").exists():
            with open(d / "hf_quant_config.json") as f:
                modelopt = json.load(f)
        return cls.parse(config, modelopt)

    def format(self, weight: str) -> WeightFormat:
        module = weight[:-len(".weight")] if weight.endswith(".weight") else weight
        return self.config.format(module)


def weight_format(quantization: "Quantization | None", weight: str) -> WeightFormat:
    """ModelConfig::format: bf16 for an unquantized checkpoint."""
    return quantization.format(weight) if quantization is not None else WeightFormat.BF16


# ---- weights (model.rs) -------------------------------------------------------------
def _companion(name: str, suffix: str) -> str:
    return name.replace(".weight", suffix)


def check_companions(checkpoint: Checkpoint, name: str, fmt: WeightFormat) -> None:
    """model.rs:447-460: the scale tensors present must match the format."""
    present = tuple(checkpoint.contains(_companion(name, s))
                    for s in (".weight_scale_inv", ".weight_scale", ".weight_scale_2"))
    expected = {"bf16": (False, False, False), "fp8_blocks": (True, False, False),
                "fp8_tensor": (False, True, False), "nvfp4": (False, True, True)}[fmt.kind]
    if present != expected:
        raise CheckpointError(f"{name}: scale tensors contradict {fmt}")


@dataclass
class HostBf16Weight:
    """HostBf16Tensor of a dense weight: bf16 bits [rows, cols]."""

    bits: np.ndarray
    rows: int
    cols: int


def load_weight(checkpoint: Checkpoint, name: str, shape: tuple[int, int], fmt: WeightFormat):
    """HostWeight::load (model.rs:554-617)."""
    rows, cols = shape
    check_companions(checkpoint, name, fmt)
    shape_error = f"{name}: invalid {fmt} data or scale shape"
    if fmt.kind == "bf16":
        s, data = checkpoint.tensor_bf16(name)
        if s != (rows, cols):
            raise CheckpointError(shape_error)
        return HostBf16Weight(data, rows, cols)
    if fmt.kind == "fp8_blocks":
        s, bits = checkpoint.tensor_fp8(name)
        ss, scales = checkpoint.tensor_bf16(_companion(name, ".weight_scale_inv"))
        if s != (rows, cols) or ss != (rows // fmt.block_n, cols // fmt.block_k):
            raise CheckpointError(shape_error)
        return HostFp8Matrix.from_parts(bits, bf16_bits_to_f32(scales), rows, cols, fmt.block_n, fmt.block_k)
    if fmt.kind == "fp8_tensor":
        s, bits = checkpoint.tensor_fp8(name)
        if s != (rows, cols):
            raise CheckpointError(shape_error)
        scale = checkpoint.scalar_f32(_companion(name, ".weight_scale"))
        return HostFp8Matrix.with_row_scales(bits, np.full(rows, scale, np.float32), rows, cols)
    if fmt.kind == "nvfp4":
        s, packed = checkpoint.tensor_nvfp4(name)
        ss, scales = checkpoint.tensor_fp8(_companion(name, ".weight_scale"))
        if s != (rows, cols // 2) or ss != (rows, cols // NVFP4_GROUP):
            raise CheckpointError(shape_error)
        return HostNvfp4Matrix.from_parts(packed, scales, checkpoint.scalar_f32(_companion(name, ".weight_scale_2")),
                                          rows, cols)
    raise CheckpointError(f"unknown weight format {fmt}")


def stack_weights(parts: list):
    """HostWeight::stack (model.rs:619-660): rows concatenated, one format."""
    if not parts:
        raise CheckpointError("no weights to stack")
    kind = type(parts[0])
    if any(type(p) is not kind for p in parts):
        raise CheckpointError("stacked weights mix formats")
    if kind is HostBf16Weight:
        cols = parts[0].cols
        if any(p.cols != cols for p in parts):
            raise CheckpointError("stacked dense weights differ in columns")
        return HostBf16Weight(np.concatenate([p.bits for p in parts]), sum(p.rows for p in parts), cols)
    if kind is HostFp8Matrix:
        return HostFp8Matrix.stack(parts)
    return HostNvfp4Matrix.stack(parts)


def load_experts(checkpoint: Checkpoint, names: list[str], shape: tuple[int, int], fmt: WeightFormat):
    """Experts stacked along rows, each keeping its own scales and global
    (the stacking of the MoE expert weights, model.rs:619-660).  NVFP4
    experts are read straight into the stacked arrays and validated once
    (the same checks as loading each and stacking)."""
    if fmt.kind != "nvfp4" or not names:
        return stack_weights([load_weight(checkpoint, n, shape, fmt) for n in names])
    rows, cols = shape
    e = len(names)
    packed = np.empty(e * rows * cols // 2, np.uint8)
    scales = np.empty(e * rows * cols // NVFP4_GROUP, np.uint8)
    row_globals = np.empty(e * rows, np.float32)
    pb, sb = rows * cols // 2, rows * cols // NVFP4_GROUP
    for i, name in enumerate(names):
        check_companions(checkpoint, name, fmt)
        scale_name = _companion(name, ".weight_scale")
        f, fs = checkpoint._shard(name), checkpoint._shard(scale_name)
        dt, s, nb = f.info(name)
        sdt, ss, snb = fs.info(scale_name)
        if s != (rows, cols // 2) or ss != (rows, cols // NVFP4_GROUP):
            raise CheckpointError(f"{name}: invalid {fmt} data or scale shape")
        if dt != "U8":
            raise CheckpointError(f"{name}: expected U8, got {dt}")
        if sdt != "F8_E4M3":
            raise CheckpointError(f"{scale_name}: expected F8_E4M3, got {sdt}")
        for fh, n, dtype, dst in ((f, name, "U8", packed[i * pb:(i + 1) * pb]),
                                  (fs, scale_name, "F8_E4M3", scales[i * sb:(i + 1) * sb])):
            st = N.lib.fpb_safetensors_read(fh._h, n.encode(), _CODE[dtype], 0, dst.ctypes.data, dst.size)
            if st != N.FPB_OK:
                _raise(st)
        row_globals[i * rows:(i + 1) * rows] = checkpoint.scalar_f32(_companion(name, ".weight_scale_2"))
    st = N.lib.fpb_nvfp4_validate(packed.ctypes.data, packed.size, scales.ctypes.data, scales.size,
                                  row_globals.ctypes.data, e * rows, cols)
    if st != N.FPB_OK:
        # Name the checkpoint tensor at fault, as loading each expert on its
        # own would (HostWeight::load per expert, model.rs:619-660).
        for i, name in enumerate(names):
            st_i = N.lib.fpb_nvfp4_validate(packed[i * pb:].ctypes.data, pb, scales[i * sb:].ctypes.data, sb,
                                            row_globals[i * rows:].ctypes.data, rows, cols)
            if st_i != N.FPB_OK:
                raise FormatError(f"{name}: {N.last_error()}")
        raise FormatError(N.last_error())
    return HostNvfp4Matrix(packed, scales, row_globals, e * rows, cols)


def verify_formats(checkpoint: Checkpoint, quantization: "Quantization | None") -> list[tuple[str, WeightFormat, str,
                                                                                              tuple[int, ...]]]:
    """The per-weight part of verify_checkpoint (model.rs:469-500): each
    ``.weight``'s companions and stored dtype agree with its format."""
    report = []
    for name in sorted(n for n in checkpoint.names() if n.endswith(".weight")):
        fmt = weight_format(quantization, name)
        check_companions(checkpoint, name, fmt)
        dtype, shape = checkpoint.stored(name)
        ok = {"bf16": dtype not in ("U8", "F8_E4M3"), "fp8_blocks": dtype == "F8_E4M3",
              "fp8_tensor": dtype == "F8_E4M3", "nvfp4": dtype == "U8"}[fmt.kind]
        if not ok:
            raise CheckpointError(f"{name}: {dtype} data contradicts {fmt}")
        report.append((name, fmt, dtype, shape))
    return report
