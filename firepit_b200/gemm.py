"""Prefill GEMM entry points (crates/firepit-kernels/src/gemm/nvfp4.rs).

``nvfp4_gemm(weight, x, y, tile).submit(sink)`` and
``nvfp4_gemm_view(weight, rows, x, y, tile).submit(sink)`` keep the
reference's builder shape and its shape asserts (gemm/nvfp4.rs:119-206).  Two
activation modes: ``act="nvfp4"`` (default) quantizes the
activations to NVFP4 on the fly and both operands go through the block-scaled
tensor cores (tcgen05.mma kind::mxf4nvf4); ``act="hilo"`` is the reference's
own numerics (gemm/nvfp4.rs:33-50): f32 activations as bf16 hi + lo times the
weights dequantized to bf16, on tcgen05 kind::f16.  The tile argument is
validated; the kernel tiles 128 x 128.
"""
from __future__ import annotations

from dataclasses import dataclass

from . import _native as N
from .gemv import ShapeError, _dtype_code
from .sink import Eager, Sink
from .weights import Q8_BLOCK, Nvfp4Matrix


@dataclass(frozen=True)
class GemmTile:
    """gemm/mod.rs:208-213."""

    m: int
    n: int
    k: int


DEFAULT_GEMM_TILE = GemmTile(64, 128, 32)          # gemm/mod.rs:215-219
DEFAULT_GROUPED_GEMM_TILE = GemmTile(32, 128, 32)  # gemm/mod.rs:221-225


def workspace_bytes(m: int, k: int) -> int:
    return int(N.lib.fpb_nvfp4_gemm_workspace_bytes(m, k))


def _check_tile(weight: Nvfp4Matrix, tile: GemmTile, rows: range, m: int) -> None:
    """gemm/nvfp4.rs:119-122 and gemm/mod.rs:588-605."""
    if not (tile.m > 0 and tile.n > 0 and tile.k % Q8_BLOCK == 0):
        raise ShapeError(f"invalid GEMM tile {tile}")
    if not (m > 0 and m % tile.m == 0):
        raise ShapeError(f"m = {m} is not a positive multiple of tile.m = {tile.m}")
    if not (rows.start < rows.stop <= weight.rows and len(rows) % tile.n == 0 and weight.cols % tile.k == 0):
        raise ShapeError(f"rows {rows} / cols {weight.cols} do not fit tile {tile}")


class Nvfp4Gemm:
    def __init__(self, weight: Nvfp4Matrix, x, y, tile: GemmTile, rows: range | None = None, workspace=None,
                 act: str = "nvfp4"):
        if act not in ("nvfp4", "hilo"):
            raise ValueError(f"act must be 'nvfp4' or 'hilo', not {act!r}")
        self.act = act
        self.weight, self.x, self.y, self.tile = weight, x, y, tile
        self.rows = rows if rows is not None else range(0, weight.rows)
        m = x.shape[0]
        _check_tile(weight, tile, self.rows, m)
        if tuple(x.shape) != (m, weight.cols):
            raise ShapeError(f"x shape {tuple(x.shape)} != ({m}, {weight.cols})")
        if tuple(y.shape) != (m, len(self.rows)) or not (x.is_contiguous() and y.is_contiguous()):
            raise ShapeError(f"y shape {tuple(y.shape)} != ({m}, {len(self.rows)}) or not contiguous")
        self.workspace = workspace

    def submit(self, sink: Sink | None = None) -> None:
        import torch
        sink = sink or Eager()
        m = self.x.shape[0]
        if self.act == "hilo":
            fn = "fpb_nvfp4_gemm_hilo"
            need = int(N.lib.fpb_nvfp4_gemm_hilo_workspace_bytes(m, len(self.rows), self.weight.cols,
                                                                  _dtype_code(self.x)))
        else:
            fn = "fpb_nvfp4_gemm"
            need = workspace_bytes(m, self.weight.cols)
        ws = self.workspace
        if ws is None or ws.numel() * ws.element_size() < need:
            ws = torch.empty(need, dtype=torch.uint8, device=self.x.device)
            self.workspace = ws

        def launch(stream):
            N.call(fn, self.weight.handle, self.rows.start, self.rows.stop, self.x.data_ptr(),
                   _dtype_code(self.x), m, self.y.data_ptr(), _dtype_code(self.y), ws.data_ptr(), need, stream)

        sink.run("nvfp4_gemm", launch)


def nvfp4_gemm(weight: Nvfp4Matrix, x, y, tile: GemmTile = DEFAULT_GEMM_TILE, workspace=None,
               act: str = "nvfp4") -> Nvfp4Gemm:
    """gemm/nvfp4.rs:131-143."""
    return Nvfp4Gemm(weight, x, y, tile, None, workspace, act)


def nvfp4_gemm_view(weight: Nvfp4Matrix, rows: range, x, y, tile: GemmTile = DEFAULT_GEMM_TILE,
                    workspace=None, act: str = "nvfp4") -> Nvfp4Gemm:
    """gemm/nvfp4.rs:166-182."""
    return Nvfp4Gemm(weight, x, y, tile, rows, workspace, act)


class Nvfp4GemmBatch:
    """Several NVFP4 GEMMs under BASELINE config 2's W4A4 rule in one launch
    (fpb_nvfp4_gemm_batch_create / fpb_nvfp4_gemv_batch_run): each member
    ``(weight, x, y[, rows])`` has its own weight rows and x [m, K] (f32 or
    bf16, m <= 128), and y [m, len(rows)] (f32 or bf16) gets what
    ``nvfp4_gemm_view(weight, rows, x, y)`` gives for m > 16: x quantized to
    NVFP4 per tensor (the same codes as ``quantize_act``), the tcgen05 GEMM
    over every member's 128-row weight tiles together, so that a few tokens
    against many matrices (a layer's projections, the experts of a decode
    batch) keep every SM busy.  Members sharing one x tensor quantize it
    once.  The tensors are bound at construction (a device table is built
    and the stream synchronised); ``submit`` can be recorded by a Graph sink.
    Needs K % 256 == 0 and rows starting at multiples of 128 (ShapeError)."""

    def __init__(self, members):
        import ctypes as C

        from .weights import current_stream_handle
        if not members:
            raise ShapeError("GEMM batch: no members")
        arr = (N.GemvSegment * len(members))()
        first_x, first_y = members[0][1], members[0][2]
        m = first_x.shape[0]
        for i, mem in enumerate(members):
            w, x, y = mem[0], mem[1], mem[2]
            rows = mem[3] if len(mem) > 3 and mem[3] is not None else range(0, w.rows)
            if not isinstance(w, Nvfp4Matrix):
                raise ShapeError("GEMM batch: NVFP4 weights only")
            if x.dim() != 2 or x.shape != (m, w.cols) or y.shape != (m, len(rows)):
                raise ShapeError(f"GEMM batch: member {i} shapes x {tuple(x.shape)} y {tuple(y.shape)}")
            if x.dtype != first_x.dtype or y.dtype != first_y.dtype:
                raise ShapeError("GEMM batch: members differ in dtypes")
            if not (x.is_contiguous() and y.is_contiguous()):
                raise ShapeError("GEMM batch: x and y must be contiguous")
            arr[i] = N.GemvSegment(w.handle.value, rows.start, rows.stop, x.data_ptr(), y.data_ptr())
        self._segs, self._members = arr, list(members)
        h = C.c_void_p()
        st = N.lib.fpb_nvfp4_gemm_batch_create(arr, len(members), _dtype_code(first_x), _dtype_code(first_y), m,
                                               current_stream_handle(first_x.device), C.byref(h))
        if st in (N.FPB_ERR_UNSUPPORTED, N.FPB_ERR_SHAPE):
            raise ShapeError(N.last_error())
        N.check(st, "fpb_nvfp4_gemm_batch_create")
        self._batch = h

    def submit(self, sink: Sink | None = None) -> None:
        sink = sink or Eager()
        sink.run("nvfp4_gemm_batch", lambda stream: N.call("fpb_nvfp4_gemv_batch_run", self._batch, stream))

    def __del__(self):
        h = getattr(self, "_batch", None)
        if h is not None and h.value:
            try:
                N.lib.fpb_nvfp4_gemv_batch_destroy(h)
            except Exception:
                pass
            self._batch = None


def nvfp4_gemm_batch(members) -> Nvfp4GemmBatch:
    """members: ``(weight, x, y)`` or ``(weight, x, y, rows)`` tuples."""
    return Nvfp4GemmBatch(members)


def quantize_act(x, stream=None):
    """NVFP4-quantizes activations [m, k]: (packed u8 [m, k/2], tiled factors,
    global f32 [1]) as device tensors."""
    import torch
    from .weights import current_stream_handle
    m, k = x.shape
    packed = torch.empty(m, k // 2, dtype=torch.uint8, device=x.device)
    sf = torch.empty(int(N.lib.fpb_nvfp4_act_sf_bytes(m, k)), dtype=torch.uint8, device=x.device)
    scal = torch.empty(2, dtype=torch.float32, device=x.device)
    s = current_stream_handle(x.device) if stream is None else stream
    N.call("fpb_nvfp4_quantize_act", x.data_ptr(), _dtype_code(x), m, k, packed.data_ptr(), sf.data_ptr(),
           scal.data_ptr(), scal[1:].data_ptr(), s)
    return packed, sf, scal[:1]


def device_error(reset: bool = True) -> int:
    import ctypes as C
    v = C.c_int(0)
    N.call("fpb_device_error", C.byref(v), 1 if reset else 0)
    return v.value


def nvfp4_grouped_gemm_q(weight: Nvfp4Matrix, a_packed, a_sf, a_global, tile_experts, rows_per_expert: int, y,
                         stream=None, token_rows=None) -> None:
    """Grouped GEMM on quantized activations (fpb_nvfp4_grouped_gemm_q).

    a_packed: [padded_rows, K/2] u8; a_sf: tiled factors; a_global: f32 [1];
    tile_experts: device int32 [padded_rows / 128]; y: [padded_rows, rows_per_expert].
    token_rows (device int32 [padded_rows], optional): the layout's tokens;
    padding rows' outputs are then unspecified.
    """
    from .weights import current_stream_handle
    padded_rows = a_packed.shape[0]
    if tuple(y.shape) != (padded_rows, rows_per_expert) or not y.is_contiguous():
        raise ShapeError(f"y shape {tuple(y.shape)} != ({padded_rows}, {rows_per_expert})")
    if tile_experts.numel() * 128 != padded_rows:
        raise ShapeError(f"{tile_experts.numel()} tile experts for {padded_rows} rows (128-row tiles)")
    s = current_stream_handle(y.device) if stream is None else stream
    N.call("fpb_nvfp4_grouped_gemm_q", weight.handle, a_packed.data_ptr(), a_sf.data_ptr(), a_global.data_ptr(),
           padded_rows, tile_experts.data_ptr(), None if token_rows is None else token_rows.data_ptr(),
           rows_per_expert, y.data_ptr(), _dtype_code(y), s)


def nvfp4_grouped_gemm_swiglu_q(weight: Nvfp4Matrix, a_packed, a_sf, a_global, tile_experts, inter: int, h,
                                amax=None, stream=None, token_rows=None):
    """The gate/up grouped GEMM fused with SwiGLU (fpb_nvfp4_grouped_gemm_swiglu_q).

    weight: experts of 2 * inter rows (gate rows, then up rows); h: [padded_rows,
    inter] f32/bf16.  Returns ``amax`` (device int32 [1]): max |h| as float bits,
    the input of ``rows_quantize(..., amax=...)``.  token_rows as in
    ``nvfp4_grouped_gemm_q`` (padding rows also left out of the amax).  The
    weight needs ``weight.prepare_glu(inter)`` once (done here on first use,
    which synchronises: make that first use outside any graph capture).
    """
    import torch
    from .weights import current_stream_handle
    padded_rows = a_packed.shape[0]
    if tuple(h.shape) != (padded_rows, inter) or not h.is_contiguous():
        raise ShapeError(f"h shape {tuple(h.shape)} != ({padded_rows}, {inter})")
    if tile_experts.numel() * 128 != padded_rows:
        raise ShapeError(f"{tile_experts.numel()} tile experts for {padded_rows} rows (128-row tiles)")
    if amax is None:
        amax = torch.zeros(1, dtype=torch.int32, device=h.device)
    s = current_stream_handle(h.device) if stream is None else stream
    weight.prepare_glu(inter, s)
    N.call("fpb_nvfp4_grouped_gemm_swiglu_q", weight.handle, a_packed.data_ptr(), a_sf.data_ptr(),
           a_global.data_ptr(), padded_rows, tile_experts.data_ptr(),
           None if token_rows is None else token_rows.data_ptr(), inter, h.data_ptr(), _dtype_code(h),
           amax.data_ptr(), s)
    return amax


def rows_quantize(x, valid_rows=None, amax=None, stream=None, token_rows=None, out=None):
    """NVFP4-quantizes rows x [rows, cols] (fpb_rows_quantize): (packed, tiled
    factors, global f32 [1]).  ``amax`` (device int32 [1], float bits) gives
    the |x| maximum to derive the global from; ``valid_rows`` (device int32
    [1]) limits the rows written; with ``token_rows`` padding rows (-1) are
    skipped.  ``out``: optional (packed, sf) buffers to write into."""
    import torch
    from .weights import current_stream_handle
    rows, cols = x.shape
    if out is None:
        packed = torch.empty(rows, cols // 2, dtype=torch.uint8, device=x.device)
        sf = torch.empty(int(N.lib.fpb_nvfp4_act_sf_bytes(rows, cols)), dtype=torch.uint8, device=x.device)
    else:
        packed, sf = out
    scal = torch.zeros(2, dtype=torch.float32, device=x.device)
    flags = 0 if token_rows is None else N.FPB_QUANT_SKIP_PADDING
    if amax is not None:
        scal[1:].view(torch.int32).copy_(amax.view(torch.int32).reshape(1))
        flags |= N.FPB_QUANT_AMAX_GIVEN
    s = current_stream_handle(x.device) if stream is None else stream
    N.call("fpb_rows_quantize", x.data_ptr(), _dtype_code(x), rows,
           None if valid_rows is None else valid_rows.data_ptr(),
           None if token_rows is None else token_rows.data_ptr(), cols, packed.data_ptr(), sf.data_ptr(),
           scal.data_ptr(), scal[1:].data_ptr(), flags, s)
    return packed, sf, scal[:1]


class Nvfp4GroupedGemmView:
    """gemm/nvfp4.rs:209-264: x holds the layout's padded_rows gathered rows,
    row tile t is multiplied by expert layout.tile_experts[t]."""

    def __init__(self, weight: Nvfp4Matrix, x, y, layout, experts: int, rows_per_expert: int, tile: GemmTile):
        if tile.m != layout.tile_rows:
            raise ShapeError(f"tile.m {tile.m} != layout tile_rows {layout.tile_rows}")
        if layout.tile_rows != 128:
            raise ShapeError("the tensor-core grouped GEMM needs a layout built with tile_rows = 128")
        if weight.rows != experts * rows_per_expert:
            raise ShapeError(f"weight rows {weight.rows} != {experts} x {rows_per_expert}")
        if tuple(x.shape) != (layout.padded_rows(), weight.cols):
            raise ShapeError(f"x shape {tuple(x.shape)} != ({layout.padded_rows()}, {weight.cols})")
        if rows_per_expert % tile.n or rows_per_expert % 128 or weight.cols % tile.k:
            raise ShapeError(f"rows_per_expert {rows_per_expert} / cols {weight.cols} do not fit tile {tile}")
        self.weight, self.x, self.y, self.layout, self.rpe = weight, x, y, layout, rows_per_expert
        self._tile_experts = None

    def submit(self, sink: Sink | None = None) -> None:
        import torch
        sink = sink or Eager()
        if self._tile_experts is None:
            self._tile_experts = torch.from_numpy(self.layout.tile_experts).to(self.x.device)

        def launch(stream):
            packed, sf, ga = quantize_act(self.x, stream)
            nvfp4_grouped_gemm_q(self.weight, packed, sf, ga, self._tile_experts, self.rpe, self.y, stream)

        sink.run("nvfp4_grouped_gemm", launch)


def nvfp4_grouped_gemm_view(weight: Nvfp4Matrix, x, y, layout, experts: int, rows_per_expert: int,
                            tile: GemmTile = GemmTile(128, 128, 32)) -> Nvfp4GroupedGemmView:
    """gemm/nvfp4.rs:218-243."""
    return Nvfp4GroupedGemmView(weight, x, y, layout, experts, rows_per_expert, tile)
