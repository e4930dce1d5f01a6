"""Seeded synthetic tensors generated on the device (csrc/synth.cu)."""
from __future__ import annotations

from . import _native as N
from .weights import current_stream_handle


def synth_normal(shape, seed: int, stream_id: int, mean: float = 0.0, std: float = 1.0, dtype=None,
                 offset: int = 0, device="cuda", out=None):
    """mean + std * N(0,1), element i of (seed, stream_id) fixed for all time."""
    import torch
    dtype = dtype or torch.float32
    if out is None:
        out = torch.empty(shape, dtype=dtype, device=device)
    code = {torch.float32: N.FPB_F32, torch.bfloat16: N.FPB_BF16}[out.dtype]
    N.call("fpb_synth_normal", seed, stream_id, offset, out.numel(), mean, std, code, out.data_ptr(),
           current_stream_handle(out.device))
    return out
