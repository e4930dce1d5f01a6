"""FP8 E4M3 weights and the prefill FP8 GEMM.

Mirrors crates/firepit-kernels/src/weights/fp8.rs (``Fp8Scaling``,
``HostFp8Matrix``, ``Fp8Matrix``) and the FP8 entry points of
src/gemm/mod.rs:417-697 (``fp8_gemm``, ``fp8_gemm_view``,
``fp8_grouped_gemm_view``) with the reference's shape asserts.  On B200 the
activations are quantized to e4m3 with one f32 scale per token (amax/448) and
both operands go through the tcgen05 tensor cores (kind::f8f6f4); block scales
are applied per 128-column K block in f32.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _native as N
from .gemm import GemmTile
from .gemv import ShapeError, _dtype_code
from .sink import Eager, Sink
from .weights import FormatError, current_stream_handle


@dataclass(frozen=True)
class Fp8Scaling:
    """weights/fp8.rs:8-12: ``Blocks(block_n, block_k)`` or ``Rows`` (block_n = block_k = 0)."""

    block_n: int = 0
    block_k: int = 0

    @classmethod
    def blocks(cls, block_n: int, block_k: int) -> "Fp8Scaling":
        return cls(block_n, block_k)

    @classmethod
    def rows(cls) -> "Fp8Scaling":
        return cls(0, 0)

    @property
    def is_rows(self) -> bool:
        return self.block_n == 0 and self.block_k == 0


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


@dataclass
class HostFp8Matrix:
    """weights/fp8.rs:21-27: e4m3 bits, f32 scales, shape and scaling."""

    bits: np.ndarray    # uint8 [rows * cols]
    scales: np.ndarray  # float32 [rows/block_n * cols/block_k] or [rows]
    rows: int
    cols: int
    scaling: Fp8Scaling

    @classmethod
    def _checked(cls, bits, scales, rows, cols, scaling: Fp8Scaling) -> "HostFp8Matrix":
        bits = np.ascontiguousarray(bits, dtype=np.uint8).reshape(-1)
        scales = np.ascontiguousarray(scales, dtype=np.float32).reshape(-1)
        st = N.lib.fpb_fp8_validate(bits.size, _ptr(scales) if scales.size else None, scales.size, rows, cols,
                                    scaling.block_n, scaling.block_k)
        if st != N.FPB_OK:
            raise FormatError(N.last_error())
        return cls(bits, scales, rows, cols, scaling)

    @classmethod
    def from_parts(cls, bits, scales, rows: int, cols: int, block_n: int, block_k: int) -> "HostFp8Matrix":
        """weights/fp8.rs:30-54."""
        if block_n == 0 or block_k == 0:
            raise FormatError("invalid FP8 scale grid")
        return cls._checked(bits, scales, rows, cols, Fp8Scaling.blocks(block_n, block_k))

    @classmethod
    def with_row_scales(cls, bits, scales, rows: int, cols: int) -> "HostFp8Matrix":
        """weights/fp8.rs:56-66."""
        return cls._checked(bits, scales, rows, cols, Fp8Scaling.rows())

    @classmethod
    def zeros(cls, rows: int, cols: int, scaling: Fp8Scaling) -> "HostFp8Matrix":
        """weights/fp8.rs:68-77."""
        bits = np.zeros(rows * cols, np.uint8)
        if scaling.is_rows:
            return cls.with_row_scales(bits, np.zeros(rows, np.float32), rows, cols)
        n = (rows // scaling.block_n) * (cols // scaling.block_k) if scaling.block_n and scaling.block_k else 0
        return cls.from_parts(bits, np.zeros(n, np.float32), rows, cols, scaling.block_n, scaling.block_k)

    @staticmethod
    def stack(parts: list["HostFp8Matrix"]) -> "HostFp8Matrix":
        """weights/fp8.rs:101-112."""
        if not parts:
            raise FormatError("no FP8 matrices to stack")
        first = parts[0]
        if any((p.cols, p.scaling) != (first.cols, first.scaling) for p in parts):
            raise FormatError("stacked FP8 matrices differ in columns or scaling")
        return HostFp8Matrix(np.concatenate([p.bits for p in parts]), np.concatenate([p.scales for p in parts]),
                             sum(p.rows for p in parts), first.cols, first.scaling)

    def upload(self, stream=None) -> "Fp8Matrix":
        """weights/fp8.rs:114-131 (synchronises the stream)."""
        h = C.c_void_p()
        s = current_stream_handle() if stream is None else stream
        N.call("fpb_fp8_matrix_create", _ptr(self.bits), _ptr(self.scales), self.rows, self.cols,
               self.scaling.block_n, self.scaling.block_k, s, C.byref(h))
        return Fp8Matrix(h, self.rows, self.cols, self.scaling)


class Fp8Matrix:
    """Device FP8 matrix (weights/fp8.rs:14-19); owns its storage."""

    def __init__(self, handle: C.c_void_p, rows: int, cols: int, scaling: Fp8Scaling):
        self._h = handle
        self.rows, self.cols, self.scaling = rows, cols, scaling

    @property
    def handle(self) -> C.c_void_p:
        if self._h is None:
            raise ValueError("FP8 matrix was destroyed")
        return self._h

    def destroy(self) -> None:
        if getattr(self, "_h", None) is not None:
            N.lib.fpb_fp8_matrix_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass

    @classmethod
    def from_device(cls, bits, scales, rows: int, cols: int, scaling: Fp8Scaling, stream=None) -> "Fp8Matrix":
        h = C.c_void_p()
        s = current_stream_handle() if stream is None else stream
        N.call("fpb_fp8_matrix_create_device", bits.data_ptr(), scales.data_ptr(), rows, cols, scaling.block_n,
               scaling.block_k, s, C.byref(h))
        return cls(h, rows, cols, scaling)

    @classmethod
    def quantize(cls, w, scaling: Fp8Scaling = Fp8Scaling(128, 128), stream=None) -> "Fp8Matrix":
        bits, scales = quantize_fp8(w, scaling, stream)
        return cls.from_device(bits, scales, w.shape[0], w.shape[1], scaling, stream)

    def to_host(self, stream=None) -> HostFp8Matrix:
        bits = np.empty(self.rows * self.cols, np.uint8)
        n = self.rows if self.scaling.is_rows else (self.rows // self.scaling.block_n) * (
            self.cols // self.scaling.block_k)
        scales = np.empty(n, np.float32)
        s = current_stream_handle() if stream is None else stream
        N.call("fpb_fp8_matrix_download", self.handle, _ptr(bits), _ptr(scales), s)
        return HostFp8Matrix(bits, scales, self.rows, self.cols, self.scaling)


def quantize_fp8(w, scaling: Fp8Scaling = Fp8Scaling.rows(), stream=None):
    """Device quantize (scale = amax/448 per block, or per row / token):
    returns (bits u8 [rows, cols], scales f32) as torch tensors."""
    import torch
    if w.dim() != 2 or not w.is_cuda or not w.is_contiguous():
        raise ValueError("quantize_fp8 expects a contiguous 2-D CUDA tensor")
    rows, cols = w.shape
    n = rows if scaling.is_rows else (rows // max(scaling.block_n, 1)) * (cols // max(scaling.block_k, 1))
    bits = torch.empty(rows, cols, dtype=torch.uint8, device=w.device)
    scales = torch.empty(max(n, 1), dtype=torch.float32, device=w.device)
    s = current_stream_handle(w.device) if stream is None else stream
    N.call("fpb_fp8_quantize", w.data_ptr(), _dtype_code(w), rows, cols, scaling.block_n, scaling.block_k,
           bits.data_ptr(), scales.data_ptr(), s)
    return bits, scales[:n]


def _check(weight: Fp8Matrix, tile: GemmTile, rows: range, m: int, x, y) -> None:
    """gemm/mod.rs:431-441 and :468-486, :586-601."""
    if not (tile.m > 0 and tile.n > 0 and tile.k > 0):
        raise ShapeError(f"invalid GEMM tile {tile}")
    if not (m > 0 and m % tile.m == 0):
        raise ShapeError(f"m = {m} is not a positive multiple of tile.m = {tile.m}")
    if tuple(x.shape) != (m, weight.cols):
        raise ShapeError(f"x shape {tuple(x.shape)} != ({m}, {weight.cols})")
    if not (rows.start < rows.stop <= weight.rows and len(rows) % tile.n == 0 and weight.cols % tile.k == 0):
        raise ShapeError(f"rows {rows} / cols {weight.cols} do not fit tile {tile}")
    sc = weight.scaling
    if not sc.is_rows:
        if rows.start % sc.block_n or rows.stop % sc.block_n:
            raise ShapeError(f"rows {rows} not aligned to block_n {sc.block_n}")
        if sc.block_n % tile.n or sc.block_k % tile.k:
            raise ShapeError(f"block {sc.block_n}x{sc.block_k} not a multiple of tile {tile}")
    if tuple(y.shape) != (m, len(rows)) or not (x.is_contiguous() and y.is_contiguous()):
        raise ShapeError(f"y shape {tuple(y.shape)} != ({m}, {len(rows)}) or not contiguous")


class Fp8Gemm:
    """``act="e4m3"`` (default): activations quantized per
    token to e4m3, tcgen05 kind::f8f6f4.  ``act="hilo"``: the reference's
    numerics (gemm/mod.rs:87-100, 155-168), f32 activations as bf16 hi + lo
    on tcgen05 kind::f16; any block sizes that divide the matrix."""

    def __init__(self, weight: Fp8Matrix, x, y, tile: GemmTile, rows: range | None = None, workspace=None,
                 act: str = "e4m3"):
        if act not in ("e4m3", "hilo"):
            raise ValueError(f"act must be 'e4m3' or 'hilo', not {act!r}")
        self.act = act
        self.weight, self.x, self.y, self.tile = weight, x, y, tile
        self.rows = rows if rows is not None else range(0, weight.rows)
        _check(weight, tile, self.rows, x.shape[0], x, y)
        self.workspace = workspace

    def submit(self, sink: Sink | None = None) -> None:
        import torch
        sink = sink or Eager()
        m = self.x.shape[0]
        fn = "fpb_fp8_gemm"
        if self.act == "hilo":
            fn = "fpb_fp8_gemm_hilo"
            need = int(N.lib.fpb_fp8_gemm_hilo_workspace_bytes(m, len(self.rows), self.weight.cols,
                                                                _dtype_code(self.x), int(not self.weight.scaling.is_rows)))
        else:
            # activations + the stream-K partial sums of this row range
            need = int(N.lib.fpb_fp8_gemm_workspace_bytes(m, self.weight.cols)) + int(
                N.lib.fpb_fp8_gemm_split_bytes(m, self.weight.cols, len(self.rows)))
        ws = self.workspace
        if ws is None or ws.numel() * ws.element_size() < need:
            ws = torch.empty(need, dtype=torch.uint8, device=self.x.device)
            self.workspace = ws

        def launch(stream):
            N.call(fn, self.weight.handle, self.rows.start, self.rows.stop, self.x.data_ptr(),
                   _dtype_code(self.x), m, self.y.data_ptr(), _dtype_code(self.y), ws.data_ptr(), need, stream)

        sink.run("fp8_gemm", launch)


def fp8_gemm(weight: Fp8Matrix, x, y, tile: GemmTile = GemmTile(64, 128, 32), workspace=None,
             act: str = "e4m3") -> Fp8Gemm:
    """gemm/mod.rs:424-442."""
    return Fp8Gemm(weight, x, y, tile, None, workspace, act)


def fp8_gemm_view(weight: Fp8Matrix, rows: range, x, y, tile: GemmTile = GemmTile(64, 128, 32),
                  workspace=None, act: str = "e4m3") -> Fp8Gemm:
    """gemm/mod.rs:579-608."""
    return Fp8Gemm(weight, x, y, tile, rows, workspace, act)


def fp8_grouped_gemm_q(weight: Fp8Matrix, a_bits, a_scales, tile_experts, rows_per_expert: int, y,
                       stream=None) -> None:
    padded = a_bits.shape[0]
    if tuple(y.shape) != (padded, rows_per_expert) or not y.is_contiguous():
        raise ShapeError(f"y shape {tuple(y.shape)} != ({padded}, {rows_per_expert})")
    if tile_experts.numel() * 128 != padded:
        raise ShapeError(f"{tile_experts.numel()} tile experts for {padded} rows (128-row tiles)")
    s = current_stream_handle(y.device) if stream is None else stream
    N.call("fpb_fp8_grouped_gemm_q", weight.handle, a_bits.data_ptr(), a_scales.data_ptr(), padded,
           tile_experts.data_ptr(), rows_per_expert, y.data_ptr(), _dtype_code(y), s)


class Fp8GroupedGemmView:
    """gemm/mod.rs:650-697: x holds the layout's padded rows, row tile t uses
    expert layout.tile_experts[t]."""

    def __init__(self, weight: Fp8Matrix, x, y, layout, experts: int, rows_per_expert: int, tile: GemmTile):
        if tile.m != layout.tile_rows or layout.tile_rows != 128:
            raise ShapeError("the tensor-core grouped GEMM needs a layout built with tile_rows = 128")
        if weight.rows != experts * rows_per_expert:
            raise ShapeError(f"weight rows {weight.rows} != {experts} x {rows_per_expert}")
        if tuple(x.shape) != (layout.padded_rows(), weight.cols):
            raise ShapeError(f"x shape {tuple(x.shape)} != ({layout.padded_rows()}, {weight.cols})")
        if rows_per_expert % tile.n or rows_per_expert % 128:
            raise ShapeError(f"rows_per_expert {rows_per_expert} does not fit tile {tile}")
        sc = weight.scaling
        if not sc.is_rows and (rows_per_expert % sc.block_n or sc.block_n % tile.n or sc.block_k % tile.k):
            raise ShapeError(f"block {sc.block_n}x{sc.block_k} does not fit rows_per_expert / tile")
        self.weight, self.x, self.y, self.layout, self.rpe = weight, x, y, layout, rows_per_expert
        self._tile_experts = None

    def submit(self, sink: Sink | None = None) -> None:
        import torch
        sink = sink or Eager()
        if self._tile_experts is None:
            self._tile_experts = torch.from_numpy(self.layout.tile_experts).to(self.x.device)

        def launch(stream):
            bits, scales = quantize_fp8(self.x, Fp8Scaling.rows(), stream)
            fp8_grouped_gemm_q(self.weight, bits, scales, self._tile_experts, self.rpe, self.y, stream)

        sink.run("fp8_grouped_gemm", launch)


def fp8_grouped_gemm_view(weight: Fp8Matrix, x, y, layout, experts: int, rows_per_expert: int,
                          tile: GemmTile = GemmTile(128, 128, 32)) -> Fp8GroupedGemmView:
    """gemm/mod.rs:650-680."""
    return Fp8GroupedGemmView(weight, x, y, layout, experts, rows_per_expert, tile)
