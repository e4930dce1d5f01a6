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
