"""MoE routing bookkeeping (crates/firepit-kernels/src/moe.rs).

``MoeDims`` (moe.rs:163-259), ``ExpertSelection`` (moe.rs:278-395) and
``PrefillLayout`` (moe.rs:397-542).  Validation and the counting sort run in
the C library (host code, no GPU needed); device copies come from torch.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _native as N


class MoeDimensionError(ValueError):
    """moe.rs:150-160."""


class ExpertSelectionError(ValueError):
    """moe.rs:262-276; ``.kind`` is Count / Index / Duplicate / Weight / Tile."""

    def __init__(self, message: str):
        super().__init__(message)
        self.kind = message.rsplit(":", 1)[-1].strip() if ":" in message else message


def _next_pow2(v: int) -> int:
    return 1 << (v - 1).bit_length() if v > 1 else 1


@dataclass(frozen=True)
class MoeDims:
    hidden: int
    intermediate: int
    shared_intermediate: int
    experts: int
    top_k: int

    @classmethod
    def new(cls, hidden: int, intermediate: int, shared_intermediate: int, experts: int, top_k: int) -> "MoeDims":
        """moe.rs:172-225."""
        if N.lib.fpb_moe_dims_validate(hidden, intermediate, shared_intermediate, experts, top_k) != N.FPB_OK:
            raise MoeDimensionError(N.last_error())
        return cls(hidden, intermediate, shared_intermediate, experts, top_k)

    def with_shared_expert(self) -> "MoeDims":
        """moe.rs:227-233: the shared expert is one more expert and one more slot."""
        return MoeDims(self.hidden, self.intermediate, self.shared_intermediate, self.experts + 1, self.top_k + 1)

    def width(self) -> int:
        """moe.rs:242-244: padded slot count."""
        return _next_pow2(self.top_k)


class ExpertSelection:
    """Device ids/weights of one token's chosen experts (moe.rs:278-395)."""

    def __init__(self, indices, weights, dims: MoeDims, slots: int):
        self.indices, self.weights, self.dims, self.slots = indices, weights, dims, slots

    @classmethod
    def parse(cls, indices, weights, dims: MoeDims, device="cuda") -> "ExpertSelection":
        """moe.rs:327-377: validate on the host, pad to ``dims.width()``."""
        import torch
        idx = np.ascontiguousarray(indices, dtype=np.int32)
        w = np.ascontiguousarray(weights, dtype=np.float32)
        if idx.size != dims.top_k or w.size != dims.top_k:
            raise ExpertSelectionError("invalid expert selection: Count")
        if N.lib.fpb_expert_selection_validate(idx.ctypes.data, w.ctypes.data, idx.size, dims.experts,
                                               dims.top_k) != N.FPB_OK:
            raise ExpertSelectionError(N.last_error())
        width = dims.width()
        pi = np.zeros(width, np.int32)
        pw = np.zeros(width, np.float32)
        pi[: idx.size] = idx
        pw[: w.size] = w
        return cls(torch.from_numpy(pi).to(device), torch.from_numpy(pw).to(device), dims, dims.top_k)


@dataclass
class PrefillLayout:
    """moe.rs:397-542: the expert-sorted, tile-padded row layout."""

    tokens: int
    tile_rows: int
    token_rows: np.ndarray    # int32 [padded_rows], -1 = padding
    tile_experts: np.ndarray  # int32 [padded_rows / tile_rows]
    inverse: np.ndarray       # int32 [tokens * top_k]
    ranges: list              # (start, count) per expert

    @staticmethod
    def max_padded_rows(tokens: int, dims: MoeDims, tile_rows: int) -> int:
        out = C.c_size_t()
        if N.lib.fpb_prefill_layout_max_padded_rows(tokens, dims.experts, dims.top_k, tile_rows,
                                                    C.byref(out)) != N.FPB_OK:
            raise ExpertSelectionError(N.last_error())
        return out.value

    @classmethod
    def parse(cls, indices, weights, dims: MoeDims, tile_rows: int) -> "PrefillLayout":
        """moe.rs:430-450 (weights checked) then from_indices (moe.rs:452-516)."""
        return cls._build(indices, weights, dims, tile_rows)

    @classmethod
    def from_indices(cls, indices, dims: MoeDims, tile_rows: int) -> "PrefillLayout":
        return cls._build(indices, None, dims, tile_rows)

    @classmethod
    def _build(cls, indices, weights, dims: MoeDims, tile_rows: int) -> "PrefillLayout":
        idx = np.ascontiguousarray(indices, dtype=np.int32).reshape(-1)
        w = None if weights is None else np.ascontiguousarray(weights, dtype=np.float32).reshape(-1)
        if w is not None and w.size != idx.size:
            raise ExpertSelectionError("invalid expert selection: Count")
        count = idx.size
        cap = count + min(dims.experts, count) * max(tile_rows - 1, 0) if tile_rows > 0 else count
        token_rows = np.empty(max(cap, 1), np.int32)
        tile_experts = np.empty(max(cap, 1), np.int32)
        inverse = np.empty(max(count, 1), np.int32)
        ranges = np.empty(2 * dims.experts, np.uint64)
        padded, tiles = C.c_size_t(), C.c_size_t()
        st = N.lib.fpb_prefill_layout_host(
            idx.ctypes.data if count else None, None if w is None else w.ctypes.data, count, dims.experts,
            dims.top_k, tile_rows, token_rows.ctypes.data, token_rows.size, C.byref(padded),
            tile_experts.ctypes.data, tile_experts.size, C.byref(tiles), inverse.ctypes.data,
            ranges.ctypes.data)
        if st != N.FPB_OK:
            msg = N.last_error()
            if st == N.FPB_ERR_SELECTION:
                raise ExpertSelectionError(msg)
            raise N.FpbError(st, "fpb_prefill_layout_host", msg)
        return cls(count // dims.top_k, tile_rows, token_rows[: padded.value].copy(),
                   tile_experts[: tiles.value].copy(), inverse[:count].copy(),
                   [(int(ranges[2 * e]), int(ranges[2 * e + 1])) for e in range(dims.experts)])

    def padded_rows(self) -> int:
        return int(self.token_rows.size)

    def padding_rows(self) -> int:
        return int(self.token_rows.size - self.inverse.size)


# ---- device routing, layout, gather, SwiGLU, combine (moe.rs:15-147, 519-859) ----------------
def _stream(t, stream):
    from .weights import current_stream_handle
    return current_stream_handle(t.device) if stream is None else stream


def _dt(t) -> int:
    from .gemv import _dtype_code
    return _dtype_code(t)


def topk_device(logits, k: int, width: int, shared_gate=None, stream=None):
    """top_k_prefill (moe.rs:15-68) on the device: ids int32 / weights f32 [T, width]."""
    import torch
    tokens, experts = logits.shape
    ids = torch.empty(tokens, width, dtype=torch.int32, device=logits.device)
    w = torch.empty(tokens, width, dtype=torch.float32, device=logits.device)
    gate = None if shared_gate is None else shared_gate.data_ptr()
    N.call("fpb_moe_topk", logits.data_ptr(), logits.stride(0), gate, tokens, experts, k, width, ids.data_ptr(),
           w.data_ptr(), _stream(logits, stream))
    return ids, w


def _selection_select(self, router: MoeDims, logits, shared_gate, sink=None) -> None:
    """ExpertSelection::select (moe.rs:305-326): device top-k of one token's
    router logits [experts] with the shared expert in slot top_k."""
    from .sink import Eager
    if self.dims != router.with_shared_expert():
        raise MoeDimensionError("selection dims differ from the router's with the shared expert")
    if tuple(logits.shape) != (router.experts,) or tuple(shared_gate.shape) != (1, 1):
        raise ExpertSelectionError("invalid expert selection: Count")
    width = self.dims.width()
    sink = sink or Eager()

    def launch(stream):
        N.call("fpb_moe_topk", logits.data_ptr(), router.experts, shared_gate.data_ptr(), 1, router.experts,
               router.top_k, width, self.indices.data_ptr(), self.weights.data_ptr(), stream)

    sink.run("top_k_prefill", launch)


def _selection_empty(cls, dims: MoeDims, device="cuda") -> ExpertSelection:
    """ExpertSelection::empty (moe.rs:288-303)."""
    import torch
    width = dims.width()
    return cls(torch.zeros(width, dtype=torch.int32, device=device),
               torch.zeros(width, dtype=torch.float32, device=device), dims, dims.top_k)


def _selection_top_k(cls, logits, shared_gate, router: MoeDims, device="cuda") -> ExpertSelection:
    """ExpertSelection::top_k (moe.rs:328-337)."""
    sel = _selection_empty(cls, router.with_shared_expert(), device)
    sel.select(router, logits, shared_gate)
    return sel


ExpertSelection.select = _selection_select
ExpertSelection.empty = classmethod(_selection_empty)
ExpertSelection.top_k = classmethod(_selection_top_k)


def layout_scratch(tokens: int, slots: int, experts: int, device):
    """Device scratch for ``fpb_moe_layout`` (per-CTA expert counts), as bytes."""
    import torch
    n = int(N.lib.fpb_moe_layout_scratch_bytes(tokens, slots, experts))
    return torch.empty(n, dtype=torch.uint8, device=device)


class PrefillPlan:
    """PrefillPlan (moe.rs:519-671) with every array on the device.

    ``top_k`` runs the router top-k and the expert-sorted layout on the GPU
    (the reference downloads the ids and sorts on the host).  Arrays are sized
    for the largest possible padding (``cap`` rows); ``padded_rows_dev`` holds
    the actual row count and row tiles past it carry expert -1.
    """

    def __init__(self, dims: MoeDims, tokens: int, tile_rows: int, cap: int, indices, weights, token_rows,
                 tile_experts, inverse, ranges, padded_rows_dev):
        self.dims, self.tokens, self.tile_rows, self.cap = dims, tokens, tile_rows, cap
        self.indices, self.weights = indices, weights
        self.token_rows, self.tile_experts, self.inverse = token_rows, tile_experts, inverse
        self.ranges, self.padded_rows_dev = ranges, padded_rows_dev

    @staticmethod
    def capacity(tokens: int, dims: MoeDims, tile_rows: int) -> int:
        rows = PrefillLayout.max_padded_rows(tokens, dims, tile_rows)
        return (rows + tile_rows - 1) // tile_rows * tile_rows

    @classmethod
    def _alloc(cls, dims: MoeDims, tokens: int, tile_rows: int, device):
        import torch
        cap = cls.capacity(tokens, dims, tile_rows)
        width = dims.width()
        return dict(cap=cap, token_rows=torch.empty(cap, dtype=torch.int32, device=device),
                    tile_experts=torch.empty(cap // tile_rows, dtype=torch.int32, device=device),
                    inverse=torch.empty(tokens, width, dtype=torch.int32, device=device),
                    ranges=torch.empty(dims.experts, 2, dtype=torch.int64, device=device),
                    padded_rows_dev=torch.zeros(1, dtype=torch.int32, device=device),
                    scratch=layout_scratch(tokens, dims.top_k, dims.experts, device))

    @classmethod
    def top_k(cls, logits, shared_gate, router: MoeDims, tile_rows: int, stream=None) -> "PrefillPlan":
        """PrefillPlan::top_k (moe.rs:545-585), all on the device."""
        if logits.dim() != 2 or logits.shape[0] <= 0 or logits.shape[1] != router.experts or (
                shared_gate is not None and tuple(shared_gate.shape) != (logits.shape[0], 1)):
            raise ExpertSelectionError("invalid expert selection: Count")
        dims = router.with_shared_expert() if shared_gate is not None else router
        tokens = logits.shape[0]
        ids, w = topk_device(logits, router.top_k, dims.width(), shared_gate, stream)
        a = cls._alloc(dims, tokens, tile_rows, logits.device)
        N.call("fpb_moe_layout", ids.data_ptr(), tokens, dims.width(), dims.top_k, dims.experts, tile_rows, a["cap"],
               a["token_rows"].data_ptr(), a["tile_experts"].data_ptr(), a["inverse"].data_ptr(),
               a["ranges"].data_ptr(), a["padded_rows_dev"].data_ptr(), a["scratch"].data_ptr(),
               a["scratch"].numel(), _stream(logits, stream))
        return cls(dims, tokens, tile_rows, a["cap"], ids, w, a["token_rows"], a["tile_experts"], a["inverse"],
                   a["ranges"], a["padded_rows_dev"])

    @classmethod
    def parse(cls, indices, weights, dims: MoeDims, tile_rows: int, device="cuda") -> "PrefillPlan":
        """PrefillPlan::parse (moe.rs:587-613): host checks and sort, device copies."""
        import torch
        layout = PrefillLayout.parse(indices, weights, dims, tile_rows)
        tokens, width = layout.tokens, dims.width()
        a = cls._alloc(dims, tokens, tile_rows, device)
        ids = np.zeros((tokens, width), np.int32)
        ws = np.zeros((tokens, width), np.float32)
        ids[:, :dims.top_k] = np.asarray(indices, np.int32).reshape(tokens, dims.top_k)
        ws[:, :dims.top_k] = np.asarray(weights, np.float32).reshape(tokens, dims.top_k)
        tr = np.full(a["cap"], -1, np.int32)
        tr[:layout.padded_rows()] = layout.token_rows
        te = np.full(a["cap"] // tile_rows, -1, np.int32)
        te[:layout.tile_experts.size] = layout.tile_experts
        inv = np.zeros((tokens, width), np.int32)
        inv[:, :dims.top_k] = layout.inverse.reshape(tokens, dims.top_k)
        rg = np.array(layout.ranges, np.int64).reshape(dims.experts, 2)
        dev = lambda v: torch.from_numpy(v).to(device)  # noqa: E731
        return cls(dims, tokens, tile_rows, a["cap"], dev(ids), dev(ws), dev(tr), dev(te), dev(inv), dev(rg),
                   dev(np.array([layout.padded_rows()], np.int32)))

    def padded_rows(self) -> int:
        """Synchronises: the device-built layout's row count."""
        return int(self.padded_rows_dev.item())

    def layout(self) -> PrefillLayout:
        """Host copy of the layout (synchronises)."""
        p = self.padded_rows()
        ranges = self.ranges.cpu().numpy()
        return PrefillLayout(self.tokens, self.tile_rows, self.token_rows[:p].cpu().numpy(),
                             self.tile_experts[:p // self.tile_rows].cpu().numpy(),
                             self.inverse[:, :self.dims.top_k].cpu().numpy().reshape(-1),
                             [(int(s), int(c)) for s, c in ranges])


def gather_prefill_view(sorted_out, x, plan: PrefillPlan, stream=None) -> None:
    """gather_prefill_view (moe.rs:71-89, 705-733): row r of sorted_out is
    token plan.token_rows[r] of x, or zeros."""
    rows = sorted_out.shape[0]
    if rows > plan.cap or tuple(x.shape) != (plan.tokens, sorted_out.shape[1]):
        raise ValueError("gather_prefill_view: shapes")
    N.call("fpb_moe_gather", x.data_ptr(), _dt(x), plan.tokens, x.shape[1], plan.token_rows.data_ptr(), rows,
           sorted_out.data_ptr(), _dt(sorted_out), _stream(x, stream))


def gather_quantize(x, plan: PrefillPlan, stream=None, per_token: bool = True):
    """Gather fused with the NVFP4 activation quantize: (packed [cap, H/2],
    tiled factors, global f32 [1]) for the grouped NVFP4 GEMM.  per_token:
    encode each token row once and copy its codes to the rows that route it
    (H % 64 == 0; the bytes equal encoding every gathered row)."""
    import torch
    tokens, h = x.shape
    packed = torch.empty(plan.cap, h // 2, dtype=torch.uint8, device=x.device)
    sf = torch.empty(int(N.lib.fpb_nvfp4_act_sf_bytes(plan.cap, h)), dtype=torch.uint8, device=x.device)
    scal = torch.empty(2, dtype=torch.float32, device=x.device)
    ws, ws_bytes = None, 0
    if per_token:
        ws_bytes = int(N.lib.fpb_moe_gather_quantize_workspace_bytes(tokens, h))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    N.call("fpb_moe_gather_quantize", x.data_ptr(), _dt(x), tokens, h, plan.token_rows.data_ptr(), plan.cap,
           plan.padded_rows_dev.data_ptr(), packed.data_ptr(), sf.data_ptr(), scal.data_ptr(), scal[1:].data_ptr(), 0,
           None if ws is None else ws.data_ptr(), ws_bytes, _stream(x, stream))
    return packed, sf, scal[:1]


def swiglu(out, gate_up, stream=None) -> None:
    """swiglu (swiglu.rs:5-20): out [rows, I] = silu(gate) * up of gate_up [rows, 2I]."""
    rows, two_i = gate_up.shape
    if tuple(out.shape) != (rows, two_i // 2):
        raise ValueError("swiglu: shapes")
    N.call("fpb_swiglu", gate_up.data_ptr(), _dt(gate_up), rows, two_i // 2, out.data_ptr(), _dt(out),
           _stream(gate_up, stream))


def swiglu_quantize(gate_up, stream=None, valid_rows=None):
    """SwiGLU fused with the NVFP4 activation quantize (for the down GEMM);
    ``valid_rows``: device int32 row count (a plan's ``padded_rows_dev``)."""
    import torch
    rows, two_i = gate_up.shape
    inter = two_i // 2
    packed = torch.empty(rows, inter // 2, dtype=torch.uint8, device=gate_up.device)
    sf = torch.empty(int(N.lib.fpb_nvfp4_act_sf_bytes(rows, inter)), dtype=torch.uint8, device=gate_up.device)
    scal = torch.empty(2, dtype=torch.float32, device=gate_up.device)
    N.call("fpb_swiglu_quantize", gate_up.data_ptr(), _dt(gate_up), rows,
           None if valid_rows is None else valid_rows.data_ptr(), inter, packed.data_ptr(), sf.data_ptr(),
           scal.data_ptr(), scal[1:].data_ptr(), 0, _stream(gate_up, stream))
    return packed, sf, scal[:1]


def combine_prefill(out, routed, plan: PrefillPlan, stream=None) -> None:
    """combine_prefill (moe.rs:91-109, 779-800): out[t] = sum over slots of
    weight * routed[inverse[t, slot]]."""
    N.call("fpb_moe_combine", routed.data_ptr(), _dt(routed), routed.shape[0], routed.shape[1], plan.inverse.data_ptr(),
           plan.weights.data_ptr(), plan.tokens, plan.dims.width(), plan.dims.top_k, out.data_ptr(), _dt(out),
           _stream(routed, stream))


def _identity_inverse(selection: ExpertSelection):
    import torch
    inv = getattr(selection, "_inverse", None)
    if inv is None:
        inv = torch.arange(selection.dims.width(), dtype=torch.int32, device=selection.indices.device)
        selection._inverse = inv
    return inv


def combine(out, routed, selection: ExpertSelection, stream=None) -> None:
    """combine (moe.rs:802-822): routed [top_k, H] in slot order."""
    if tuple(routed.shape) != (selection.dims.top_k, out.shape[-1]):
        raise ValueError("combine: routed must be [top_k, hidden]")
    N.call("fpb_moe_combine", routed.data_ptr(), _dt(routed), routed.shape[0], routed.shape[1],
           _identity_inverse(selection).data_ptr(), selection.weights.data_ptr(), 1, selection.dims.width(),
           selection.dims.top_k, out.data_ptr(), _dt(out), _stream(routed, stream))


def combine_add_norm_view(out, normed, routed, selection: ExpertSelection, residual, gamma, eps: float,
                          stream=None) -> None:
    """combine_add_norm_view (moe.rs:824-842)."""
    N.call("fpb_moe_combine_add_norm", routed.data_ptr(), _dt(routed), routed.shape[0], routed.shape[1],
           _identity_inverse(selection).data_ptr(), selection.weights.data_ptr(), 1, selection.dims.width(),
           selection.dims.top_k, residual.data_ptr(), gamma.data_ptr(), C.c_float(eps), out.data_ptr(),
           normed.data_ptr(), _stream(routed, stream))


def combine_add_norm_prefill(out, normed, routed, plan: PrefillPlan, residual, gamma, eps: float,
                             stream=None) -> None:
    """combine_add_norm_prefill (moe.rs:844-859)."""
    N.call("fpb_moe_combine_add_norm", routed.data_ptr(), _dt(routed), routed.shape[0], routed.shape[1],
           plan.inverse.data_ptr(),
           plan.weights.data_ptr(), plan.tokens, plan.dims.width(), plan.dims.top_k, residual.data_ptr(),
           gamma.data_ptr(), C.c_float(eps), out.data_ptr(), normed.data_ptr(), _stream(routed, stream))
