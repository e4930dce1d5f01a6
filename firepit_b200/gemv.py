"""Decode GEMV entry points (crates/firepit-kernels/src/gemv/mod.rs).

``gemv(weight, x, y, tile).submit(sink)`` and
``expert_gemv_weight_view(weight, x, selection, y, rows_per_expert,
input_stride, tile).submit(sink)`` keep the reference's builder shape.  The
tile argument is validated the way the reference asserts it
(``GemvTile::fits``); the B200 kernel picks its own tiling.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import _native as N
from .sink import Eager, Sink
from .weights import Q8_BLOCK, Nvfp4Matrix, current_stream_handle


class ShapeError(ValueError):
    """The reference's ``assert!`` on shapes and tiles."""


@dataclass(frozen=True)
class GemvTile:
    """gemv/mod.rs:16-20."""

    rows: int
    blocks: int

    def fits(self, rows: int, cols: int) -> bool:
        """gemv/mod.rs:60-64."""
        return rows % self.rows == 0 and cols % Q8_BLOCK == 0 and (cols // Q8_BLOCK) % self.blocks == 0


DEFAULT_GEMV_TILE = GemvTile(rows=16, blocks=4)  # gemv/mod.rs:22-25
FP8_TARGET_ROW_TILES = 64
FP8_MAX_ROW_TILE = 128


def _next_pow2(v: int) -> int:
    return 1 << (v - 1).bit_length() if v > 1 else 1


def fp8_tile(rows: int, cols: int, block_n: int, block_k: int, groups: int) -> GemvTile:
    """gemv/mod.rs:30-54: about 64 row tiles, at most 128 rows, power of two."""
    if not (rows > 0 and cols > 0 and block_n > 0 and block_k > 0 and groups > 0):
        raise ShapeError("fp8_tile: sizes must be positive")
    target = _next_pow2(min(max(-(-rows * groups // FP8_TARGET_ROW_TILES), 1), FP8_MAX_ROW_TILE))
    t_rows, t_blocks = target, DEFAULT_GEMV_TILE.blocks
    while rows % t_rows != 0 or block_n % t_rows != 0:
        t_rows //= 2
    while (cols // Q8_BLOCK) % t_blocks != 0 or block_k % (t_blocks * Q8_BLOCK) != 0:
        t_blocks //= 2
    return GemvTile(t_rows, t_blocks)


def row_scaled_tile(rows: int, cols: int, groups: int) -> GemvTile:
    """gemv/mod.rs:56-58."""
    return fp8_tile(rows, cols, rows, cols, groups)


def _dtype_code(t) -> int:
    import torch
    if t.dtype == torch.float32:
        return N.FPB_F32
    if t.dtype == torch.bfloat16:
        return N.FPB_BF16
    raise TypeError(f"unsupported dtype {t.dtype}")


def _is_fp8(weight) -> bool:
    return getattr(weight, "scaling", None) is not None


def _check_fp8_tile(weight, tile: GemvTile) -> None:
    """gemv/fp8.rs:205-229: block scales must be whole tiles."""
    sc = weight.scaling
    if not sc.is_rows and (sc.block_n % tile.rows != 0 or sc.block_k % (tile.blocks * Q8_BLOCK) != 0):
        raise ShapeError(f"GEMV tile {tile} does not divide the FP8 blocks {sc.block_n}x{sc.block_k}")


class Gemv:
    """gemv/mod.rs:66-123: the weight-format dispatch, ``Weight::Nvfp4``
    (gemv/nvfp4.rs) or ``Weight::Fp8`` (gemv/fp8.rs:186-246)."""

    def __init__(self, weight, x, y, tile: GemvTile, rows: range | None = None):
        self.weight, self.x, self.y, self.tile = weight, x, y, tile
        self.rows = rows if rows is not None else range(0, weight.rows)
        n = len(self.rows)
        batch = x.shape[0]
        if batch <= 0 or not tile.fits(n, weight.cols):
            raise ShapeError(f"GEMV tile {tile} does not fit {n}x{weight.cols}")
        if _is_fp8(weight):
            _check_fp8_tile(weight, tile)
        if x.numel() != batch * weight.cols:
            raise ShapeError(f"x has {x.numel()} elements, expected {batch}x{weight.cols}")
        if y.numel() != batch * n:
            raise ShapeError(f"y has {y.numel()} elements, expected {batch}x{n}")
        if not (x.is_contiguous() and y.is_contiguous()):
            raise ShapeError("x and y must be contiguous")

    def submit(self, sink: Sink | None = None) -> None:
        sink = sink or Eager()
        batch = self.x.shape[0]

        fn = "fpb_fp8_gemv" if _is_fp8(self.weight) else "fpb_nvfp4_gemv"

        def launch(stream):
            N.call(fn, self.weight.handle, self.rows.start, self.rows.stop,
                   self.x.data_ptr(), _dtype_code(self.x), self.y.data_ptr(), _dtype_code(self.y),
                   batch, stream)

        sink.run("gemv", launch)


def gemv(weight, x, y, tile: GemvTile = DEFAULT_GEMV_TILE, rows: range | None = None) -> Gemv:
    """gemv/mod.rs:74-87.  x: [batch, cols] (the reference's [B, K/32, 32]
    is the same memory), y: [batch, rows]."""
    return Gemv(weight, x, y, tile, rows)


class BatchedGemv:
    """Several NVFP4 decode GEMVs in one launch (fpb_nvfp4_gemv_batched).

    The reference saves decode launches by stacking the projections that
    read one input into a single matrix at load time (firepit
    src/model.rs:407-444); here each ``(weight, x, y[, rows])`` keeps its own
    handle and input, and every member's result equals ``gemv(weight, x, y,
    rows=rows)``.  All members share the column count, dtypes and batch."""

    def __init__(self, members, tile: GemvTile = DEFAULT_GEMV_TILE):
        if not members:
            raise ShapeError("batched GEMV: no members")
        self.gemvs = [Gemv(m[0], m[1], m[2], tile, m[3] if len(m) > 3 else None) for m in members]
        first = self.gemvs[0]
        for g in self.gemvs:
            if _is_fp8(g.weight):
                raise ShapeError("batched GEMV: NVFP4 weights only")
            if g.weight.cols != first.weight.cols or g.x.shape[0] != first.x.shape[0]:
                raise ShapeError("batched GEMV: members differ in columns or batch")
            if g.x.dtype != first.x.dtype or g.y.dtype != first.y.dtype:
                raise ShapeError("batched GEMV: members differ in dtypes")
        arr = (N.GemvSegment * len(self.gemvs))()
        for i, g in enumerate(self.gemvs):
            arr[i] = N.GemvSegment(g.weight.handle.value, g.rows.start, g.rows.stop, g.x.data_ptr(),
                                   g.y.data_ptr())
        self._segs = arr

    def submit(self, sink: Sink | None = None) -> None:
        sink = sink or Eager()
        first = self.gemvs[0]

        def launch(stream):
            N.call("fpb_nvfp4_gemv_batched", self._segs, len(self.gemvs), _dtype_code(first.x),
                   _dtype_code(first.y), first.x.shape[0], stream)

        sink.run("gemv_batched", launch)


def gemv_batched(members, tile: GemvTile = DEFAULT_GEMV_TILE) -> BatchedGemv:
    """members: ``(weight, x, y)`` or ``(weight, x, y, rows)`` tuples."""
    return BatchedGemv(members, tile)


class PlanesGemvBatch(BatchedGemv):
    """The members of a ``BatchedGemv`` on the tensor cores
    (fpb_nvfp4_gemv_batch_*): x as 8 NVFP4 digit planes against each
    member's weight rows with tcgen05, every member in one launch.  The
    member tensors are bound at construction (a device table is built and
    the stream synchronised), so ``submit`` reads nothing on the host and can
    be recorded by a Graph sink; results equal ``gemv`` up to f32 rounding.
    Needs cols % 256 == 0, cols <= 4096 and rows starting at multiples of
    128 (ShapeError otherwise: use ``gemv_batched``)."""

    def __init__(self, members, tile: GemvTile = DEFAULT_GEMV_TILE, y_peers=None):
        """y_peers (optional): per member, the device pointers of the copies
        its result goes to instead of its y (fpb_nvfp4_gemv_batch_create_peers:
        e.g. this rank's slice in every rank's gathered output)."""
        super().__init__(members, tile)
        first = self.gemvs[0]
        h = C.c_void_p()
        stream = current_stream_handle(first.x.device)
        if y_peers is None:
            st = N.lib.fpb_nvfp4_gemv_batch_create(self._segs, len(self.gemvs), _dtype_code(first.x),
                                                    _dtype_code(first.y), first.x.shape[0], stream, C.byref(h))
        else:
            n_peer = len(y_peers[0])
            if len(y_peers) != len(self.gemvs) or any(len(p) != n_peer for p in y_peers):
                raise ShapeError("batched GEMV: one list of peer copies per member, all of one length")
            arr = (C.c_void_p * (len(self.gemvs) * n_peer))(*[int(v) for p in y_peers for v in p])
            self._peers = arr
            st = N.lib.fpb_nvfp4_gemv_batch_create_peers(self._segs, len(self.gemvs), _dtype_code(first.x),
                                                          _dtype_code(first.y), first.x.shape[0], arr, n_peer,
                                                          stream, C.byref(h))
        if st == N.FPB_ERR_UNSUPPORTED or st == N.FPB_ERR_SHAPE:
            raise ShapeError(N.last_error())
        N.check(st, "fpb_nvfp4_gemv_batch_create")
        self._batch = h

    def submit(self, sink: Sink | None = None) -> None:
        sink = sink or Eager()
        sink.run("gemv_batch_planes", lambda stream: N.call("fpb_nvfp4_gemv_batch_run", self._batch, stream))

    def __del__(self):
        h = getattr(self, "_batch", None)
        if h is not None and h.value:
            try:
                N.lib.fpb_nvfp4_gemv_batch_destroy(h)
            except Exception:
                pass
            self._batch = None


def gemv_batch_planes(members, tile: GemvTile = DEFAULT_GEMV_TILE, y_peers=None) -> PlanesGemvBatch:
    """members: ``(weight, x, y)`` or ``(weight, x, y, rows)`` tuples; y_peers
    as in ``PlanesGemvBatch``."""
    return PlanesGemvBatch(members, tile, y_peers)


class ExpertGemvView:
    """gemv/mod.rs:126-206 for ``Weight::Nvfp4`` or ``Weight::Fp8``
    (gemv/fp8.rs:248-281)."""

    def __init__(self, weight, x, selection, y, rows_per_expert: int, input_stride: int,
                 tile: GemvTile):
        dims = selection.dims
        if weight.rows != dims.experts * rows_per_expert:
            raise ShapeError("expert GEMV: weight rows != experts * rows_per_expert")
        if not tile.fits(rows_per_expert, weight.cols):
            raise ShapeError(f"GEMV tile {tile} does not fit {rows_per_expert}x{weight.cols}")
        if _is_fp8(weight):
            _check_fp8_tile(weight, tile)
            if not weight.scaling.is_rows and rows_per_expert % weight.scaling.block_n != 0:
                raise ShapeError("expert GEMV: rows per expert not a multiple of the FP8 block rows")
        self.weight, self.x, self.selection, self.y = weight, x, selection, y
        self.rows_per_expert, self.input_stride = rows_per_expert, input_stride
        self.slots = selection.slots

    def submit(self, sink: Sink | None = None) -> None:
        sink = sink or Eager()

        fn = "fpb_fp8_expert_gemv" if _is_fp8(self.weight) else "fpb_nvfp4_expert_gemv"

        def launch(stream):
            N.call(fn, self.weight.handle, self.x.data_ptr(), _dtype_code(self.x),
                   self.selection.indices.data_ptr(), self.slots, self.rows_per_expert, self.input_stride,
                   self.y.data_ptr(), _dtype_code(self.y), stream)

        sink.run("expert_gemv", launch)


def expert_gemv_weight_view(weight, x, selection, y, rows_per_expert: int, input_stride: int,
                            tile: GemvTile = DEFAULT_GEMV_TILE) -> ExpertGemvView:
    """gemv/mod.rs:137-156."""
    return ExpertGemvView(weight, x, selection, y, rows_per_expert, input_stride, tile)


__all__ = ["GemvTile", "DEFAULT_GEMV_TILE", "fp8_tile", "row_scaled_tile", "gemv", "Gemv", "gemv_batched",
           "BatchedGemv",
           "expert_gemv_weight_view", "ExpertGemvView", "ShapeError", "current_stream_handle"]
