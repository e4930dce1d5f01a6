"""NVFP4 weight matrices (crates/firepit-kernels/src/weights/nvfp4.rs).

``HostNvfp4Matrix`` keeps the reference's host-side constructor, ``stack`` and
``upload``; ``Nvfp4Matrix`` is the device handle the kernels consume.  Device
memory, streams and tensors come from torch (plumbing only); every
computation runs in the CUDA library through the C ABI.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _native as N

NVFP4_GROUP = 16  # weights/nvfp4.rs:8
Q8_BLOCK = 32     # weights/q8_format.rs:3


class FormatError(ValueError):
    """The reference's ``Err(&'static str)`` from the weight constructors."""


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def current_stream_handle(device=None) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream


@dataclass
class HostNvfp4Matrix:
    """weights/nvfp4.rs:34-40: packed e2m1 pairs, e4m3 scales, per-row globals."""

    packed: np.ndarray      # uint8 [rows * cols / 2], even column in the low nibble
    scales: np.ndarray      # uint8 [rows * cols / 16] e4m3 bits
    row_scales: np.ndarray  # float32 [rows]
    rows: int
    cols: int

    @classmethod
    def from_parts(cls, packed, scales, global_scale: float, rows: int, cols: int) -> "HostNvfp4Matrix":
        """weights/nvfp4.rs:47-72 (validation runs in the C library)."""
        packed = np.ascontiguousarray(packed, dtype=np.uint8).reshape(-1)
        scales = np.ascontiguousarray(scales, dtype=np.uint8).reshape(-1)
        rows_g = np.full(max(rows, 0), global_scale, dtype=np.float32)
        st = N.lib.fpb_nvfp4_validate(_ptr(packed), packed.size, _ptr(scales), scales.size,
                                      _ptr(rows_g) if rows_g.size else _ptr(np.zeros(1, np.float32)),
                                      rows, cols)
        if st != N.FPB_OK:
            raise FormatError(N.last_error())
        return cls(packed, scales, rows_g, rows, cols)

    @classmethod
    def zeros(cls, rows: int, cols: int) -> "HostNvfp4Matrix":
        """weights/nvfp4.rs:74-82."""
        return cls.from_parts(np.zeros(rows * cols // 2, np.uint8), np.zeros(rows * cols // NVFP4_GROUP, np.uint8),
                              0.0, rows, cols)

    @staticmethod
    def stack(parts: list["HostNvfp4Matrix"]) -> "HostNvfp4Matrix":
        """weights/nvfp4.rs:84-97: concatenate rows, keep each part's globals."""
        if not parts:
            raise FormatError("no NVFP4 matrices to stack")
        cols = parts[0].cols
        if any(p.cols != cols for p in parts):
            raise FormatError("stacked NVFP4 matrices differ in columns")
        return HostNvfp4Matrix(np.concatenate([p.packed for p in parts]),
                               np.concatenate([p.scales for p in parts]),
                               np.concatenate([p.row_scales for p in parts]).astype(np.float32),
                               sum(p.rows for p in parts), cols)

    def upload(self, stream=None) -> "Nvfp4Matrix":
        """weights/nvfp4.rs:99-120: copy to the device (synchronises the stream)."""
        h = C.c_void_p()
        s = current_stream_handle() if stream is None else stream
        N.call("fpb_nvfp4_matrix_create", _ptr(self.packed), _ptr(self.scales),
               _ptr(np.ascontiguousarray(self.row_scales, np.float32)), self.rows, self.cols, s, C.byref(h))
        return Nvfp4Matrix(h, self.rows, self.cols)


class Nvfp4Matrix:
    """Device NVFP4 matrix (weights/nvfp4.rs:11-32); owns its storage."""

    def __init__(self, handle: C.c_void_p, rows: int, cols: int):
        self._h = handle
        self.rows = rows
        self.cols = cols

    @property
    def handle(self) -> C.c_void_p:
        if self._h is None:
            raise ValueError("NVFP4 matrix was destroyed")
        return self._h

    def destroy(self) -> None:
        if getattr(self, "_h", None) is not None:
            N.lib.fpb_nvfp4_matrix_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass

    @classmethod
    def from_device(cls, packed, scales, row_globals, rows: int, cols: int, stream=None) -> "Nvfp4Matrix":
        """Copies device tensors in the upload layout into a new handle."""
        h = C.c_void_p()
        s = current_stream_handle() if stream is None else stream
        N.call("fpb_nvfp4_matrix_create_device", packed.data_ptr(), scales.data_ptr(),
               row_globals.data_ptr(), rows, cols, s, C.byref(h))
        return cls(h, rows, cols)

    @classmethod
    def quantize(cls, w, rows_per_global: int | None = None, stream=None) -> "Nvfp4Matrix":
        """Quantizes a device f32/bf16 [rows, cols] tensor (one global per
        ``rows_per_global`` rows; default: the whole matrix)."""
        packed, scales, globals_ = quantize_nvfp4(w, rows_per_global, stream)
        return cls.from_device(packed, scales, globals_, w.shape[0], w.shape[1], stream)

    def device_ptrs(self) -> tuple[int, int, int]:
        p, s, g = C.c_void_p(), C.c_void_p(), C.c_void_p()
        N.call("fpb_nvfp4_matrix_device_ptrs", self.handle, C.byref(p), C.byref(s), C.byref(g))
        return p.value, s.value, g.value

    def prepare_glu(self, inter: int, stream=None) -> None:
        """Builds the interleaved factor copy of the fused gate/up + SwiGLU
        GEMM for experts of 2 * inter rows (fpb_nvfp4_matrix_prepare_glu):
        allocates and synchronises, so call it at load time."""
        if getattr(self, "_glu_inter", None) == inter:
            return
        s = current_stream_handle() if stream is None else stream
        N.call("fpb_nvfp4_matrix_prepare_glu", self.handle, inter, s)
        self._glu_inter = inter

    def to_host(self, stream=None) -> HostNvfp4Matrix:
        """Copies the device storage back (synchronises the stream)."""
        packed = np.empty(self.rows * self.cols // 2, np.uint8)
        scales = np.empty(self.rows * self.cols // NVFP4_GROUP, np.uint8)
        globals_ = np.empty(self.rows, np.float32)
        s = current_stream_handle() if stream is None else stream
        N.call("fpb_nvfp4_matrix_download", self.handle, _ptr(packed), _ptr(scales), _ptr(globals_), s)
        return HostNvfp4Matrix(packed, scales, globals_, self.rows, self.cols)

    def dequantize(self, stream=None):
        """f32 [rows, cols] in ModelOpt order (firepit checkpoint.rs:401-420)."""
        import torch
        out = torch.empty(self.rows, self.cols, dtype=torch.float32, device="cuda")
        s = current_stream_handle() if stream is None else stream
        N.call("fpb_nvfp4_dequantize", self.handle, out.data_ptr(), s)
        return out


def quantize_nvfp4(w, rows_per_global: int | None = None, stream=None):
    """Device quantize: returns (packed u8 [rows, cols/2], scales u8 [rows, cols/16],
    row_globals f32 [rows]) as torch tensors."""
    import torch
    if w.dim() != 2 or not w.is_cuda or not w.is_contiguous():
        raise ValueError("quantize_nvfp4 expects a contiguous 2-D CUDA tensor")
    rows, cols = w.shape
    rpg = rows if rows_per_global is None else rows_per_global
    dtype = {torch.float32: N.FPB_F32, torch.bfloat16: N.FPB_BF16}[w.dtype]
    packed = torch.empty(rows, cols // 2, dtype=torch.uint8, device=w.device)
    scales = torch.empty(rows, cols // NVFP4_GROUP, dtype=torch.uint8, device=w.device)
    globals_ = torch.empty(rows, dtype=torch.float32, device=w.device)
    scratch = torch.empty(max(1, rows // max(rpg, 1)), dtype=torch.float32, device=w.device)
    s = current_stream_handle(w.device) if stream is None else stream
    N.call("fpb_nvfp4_quantize", w.data_ptr(), dtype, rows, cols, rpg, packed.data_ptr(),
           scales.data_ptr(), globals_.data_ptr(), scratch.data_ptr(), s)
    return packed, scales, globals_
