"""ctypes binding of the firepit_b200 C ABI (include/firepit_b200.h).

The library is the in-tree ``firepit_b200/libfirepit_b200.so`` built by
``python firepit_b200/build.py``.  There is no fallback: if the library is
missing or fails to load, importing this module raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfirepit_b200.so"

FPB_OK = 0
FPB_ERR_INVALID_ARGUMENT = 1
FPB_ERR_SHAPE = 2
FPB_ERR_FORMAT = 3
FPB_ERR_CUDA = 4
FPB_ERR_UNSUPPORTED = 5
FPB_ERR_SELECTION = 6
FPB_ERR_WORKSPACE = 7
FPB_ERR_NO_DEVICE = 8
FPB_ERR_IO = 9
FPB_ERR_COMM = 10

FPB_F32 = 0
FPB_BF16 = 1
FPB_QUANT_AMAX_GIVEN = 1
FPB_QUANT_SKIP_PADDING = 2
FPB_COMM_U32, FPB_COMM_I32, FPB_COMM_BYTES = 2, 3, 4
FPB_COMM_SUM, FPB_COMM_MAX = 0, 1


class FpbError(RuntimeError):
    """A non-zero status from the C ABI; ``.status`` holds the code."""

    def __init__(self, status: int, func: str, message: str):
        super().__init__(f"{func}: status {status} ({_status_name(status)}): {message}")
        self.status = status


def _status_name(status: int) -> str:
    try:
        return lib.fpb_status_string(status).decode()
    except Exception:  # pragma: no cover - only while the library is loading
        return str(status)


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python firepit_b200/build.py` "
            "(the CUDA path has no fallback)")
    return C.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_LOCAL)


lib = _load()

vp = C.c_void_p
sz = C.c_size_t
i32 = C.c_int
u8p = C.POINTER(C.c_uint8)
f32p = C.POINTER(C.c_float)

class GemvSegment(C.Structure):
    """fpb_gemv_segment (include/firepit_b200.h)."""
    _fields_ = [("w", C.c_void_p), ("row_begin", C.c_size_t), ("row_end", C.c_size_t), ("x", C.c_void_p),
                ("y", C.c_void_p)]


FPB_COMM_ID_BYTES = 128
FPB_IPC_HANDLE_BYTES = 64
sizep = C.POINTER(C.c_size_t)

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "fpb_safetensors_open": (i32, [C.c_char_p, C.POINTER(vp)]),
    "fpb_safetensors_close": (None, [vp]),
    "fpb_safetensors_count": (sz, [vp]),
    "fpb_safetensors_name": (C.c_char_p, [vp, sz]),
    "fpb_safetensors_has": (i32, [vp, C.c_char_p]),
    "fpb_safetensors_metadata": (C.c_char_p, [vp, C.c_char_p]),
    "fpb_safetensors_dtype_name": (C.c_char_p, [i32]),
    "fpb_safetensors_info": (i32, [vp, C.c_char_p, C.POINTER(i32), C.POINTER(C.c_int64), i32, C.POINTER(i32),
                                   C.POINTER(sz)]),
    "fpb_safetensors_read": (i32, [vp, C.c_char_p, i32, sz, vp, sz]),
    "fpb_version": (C.c_char_p, []),
    "fpb_status_string": (C.c_char_p, [i32]),
    "fpb_last_error": (C.c_char_p, []),
    "fpb_launch_count": (C.c_uint64, []),
    "fpb_e2m1_to_f32": (C.c_float, [C.c_uint8]),
    "fpb_e4m3_to_f32": (C.c_float, [C.c_uint8]),
    "fpb_f32_to_e2m1": (C.c_uint8, [C.c_float]),
    "fpb_f32_to_e4m3": (C.c_uint8, [C.c_float]),
    "fpb_synth_normal": (i32, [C.c_uint64, C.c_uint32, C.c_uint64, sz, C.c_float, C.c_float, i32, vp, vp]),
    "fpb_nvfp4_validate": (i32, [vp, sz, vp, sz, vp, sz, sz]),
    "fpb_nvfp4_matrix_create": (i32, [vp, vp, vp, sz, sz, vp, C.POINTER(vp)]),
    "fpb_nvfp4_matrix_create_device": (i32, [vp, vp, vp, sz, sz, vp, C.POINTER(vp)]),
    "fpb_nvfp4_matrix_destroy": (i32, [vp]),
    "fpb_nvfp4_matrix_shape": (i32, [vp, C.POINTER(sz), C.POINTER(sz)]),
    "fpb_nvfp4_matrix_device_ptrs": (i32, [vp, C.POINTER(vp), C.POINTER(vp), C.POINTER(vp)]),
    "fpb_nvfp4_matrix_download": (i32, [vp, vp, vp, vp, vp]),
    "fpb_nvfp4_quantize": (i32, [vp, i32, sz, sz, sz, vp, vp, vp, vp, vp]),
    "fpb_nvfp4_quantize_noalloc": (i32, [vp, i32, sz, sz, sz, vp, vp, vp, vp]),
    "fpb_nvfp4_dequantize": (i32, [vp, vp, vp]),
    "fpb_nvfp4_gemv": (i32, [vp, sz, sz, vp, i32, vp, i32, i32, vp]),
    "fpb_nvfp4_gemv_batched": (i32, [C.POINTER(GemvSegment), i32, i32, i32, i32, vp]),
    "fpb_nvfp4_expert_gemv": (i32, [vp, vp, i32, vp, i32, sz, i32, vp, i32, vp]),
    "fpb_fp8_gemv": (i32, [vp, sz, sz, vp, i32, vp, i32, i32, vp]),
    "fpb_fp8_expert_gemv": (i32, [vp, vp, i32, vp, i32, sz, i32, vp, i32, vp]),
    "fpb_nvfp4_act_sf_bytes": (sz, [sz, sz]),
    "fpb_nvfp4_gemm_workspace_bytes": (sz, [sz, sz]),
    "fpb_nvfp4_quantize_act": (i32, [vp, i32, sz, sz, vp, vp, vp, vp, vp]),
    "fpb_nvfp4_matrix_prepare_gemm": (i32, [vp, vp]),
    "fpb_nvfp4_matrix_prepare_glu": (i32, [vp, sz, vp]),
    "fpb_nvfp4_gemm_q": (i32, [vp, sz, sz, vp, vp, vp, sz, vp, i32, vp]),
    "fpb_nvfp4_gemm": (i32, [vp, sz, sz, vp, i32, sz, vp, i32, vp, sz, vp]),
    "fpb_nvfp4_gemm_hilo_workspace_bytes": (sz, [sz, sz, sz, i32]),
    "fpb_nvfp4_gemm_hilo": (i32, [vp, sz, sz, vp, i32, sz, vp, i32, vp, sz, vp]),
    "fpb_fp8_gemm_hilo_workspace_bytes": (sz, [sz, sz, sz, i32, i32]),
    "fpb_fp8_gemm_hilo": (i32, [vp, sz, sz, vp, i32, sz, vp, i32, vp, sz, vp]),
    "fpb_nvfp4_grouped_gemm_q": (i32, [vp, vp, vp, vp, sz, vp, vp, sz, vp, i32, vp]),
    "fpb_device_error": (i32, [C.POINTER(i32), i32]),
    "fpb_fp8_validate": (i32, [sz, vp, sz, sz, sz, sz, sz]),
    "fpb_fp8_matrix_create": (i32, [vp, vp, sz, sz, sz, sz, vp, C.POINTER(vp)]),
    "fpb_fp8_matrix_create_device": (i32, [vp, vp, sz, sz, sz, sz, vp, C.POINTER(vp)]),
    "fpb_fp8_matrix_destroy": (i32, [vp]),
    "fpb_fp8_matrix_shape": (i32, [vp, C.POINTER(sz), C.POINTER(sz), C.POINTER(sz), C.POINTER(sz)]),
    "fpb_fp8_matrix_download": (i32, [vp, vp, vp, vp]),
    "fpb_fp8_quantize": (i32, [vp, i32, sz, sz, sz, sz, vp, vp, vp]),
    "fpb_fp8_gemm_workspace_bytes": (sz, [sz, sz]),
    "fpb_fp8_gemm_q": (i32, [vp, sz, sz, vp, vp, sz, vp, i32, vp]),
    "fpb_fp8_gemm_q_split": (i32, [vp, sz, sz, vp, vp, sz, vp, i32, vp, sz, vp]),
    "fpb_fp8_gemm_split_bytes": (sz, [sz, sz, sz]),
    "fpb_fp8_gemm": (i32, [vp, sz, sz, vp, i32, sz, vp, i32, vp, sz, vp]),
    "fpb_fp8_grouped_gemm_q": (i32, [vp, vp, vp, sz, vp, sz, vp, i32, vp]),
    "fpb_moe_topk": (i32, [vp, sz, vp, sz, sz, sz, sz, vp, vp, vp]),
    "fpb_moe_layout": (i32, [vp, sz, sz, sz, sz, sz, sz, vp, vp, vp, vp, vp, vp, sz, vp]),
    "fpb_moe_layout_scratch_bytes": (sz, [sz, sz, sz]),
    "fpb_moe_layout_masked": (i32, [vp, sz, sz, sz, sz, sz, sz, vp, vp, vp, vp, vp, vp, sz, vp]),
    "fpb_moe_gather_codes": (i32, [vp, sz, vp, sz, sz, sz, vp, sz, vp, i32, vp, vp, vp]),
    "fpb_ep_record_bytes": (sz, [sz, sz]),
    "fpb_nvfp4_gemm_batch_create": (i32, [C.POINTER(GemvSegment), i32, i32, i32, i32, vp, C.POINTER(vp)]),
    "fpb_nvfp4_gemv_batch_create_peers": (i32, [C.POINTER(GemvSegment), i32, i32, i32, i32, C.POINTER(vp), i32, vp,
                                                C.POINTER(vp)]),
    "fpb_ep_dispatch": (i32, [vp, i32, sz, sz, vp, vp, sz, sz, sz, sz, vp, vp, vp, vp, vp]),
    "fpb_ep_unpack": (i32, [vp, sz, sz, sz, vp, vp, vp]),
    "fpb_ep_dispatch_chunks": (i32, [vp, i32, sz, sz, vp, vp, sz, sz, sz, sz, vp, vp, i32, vp, vp, vp]),
    "fpb_moe_combine_chunks": (i32, [vp, i32, sz, sz, vp, vp, sz, sz, sz, vp, sz, i32, vp]),
    "fpb_ipc_alloc": (i32, [sz, C.POINTER(vp)]),
    "fpb_ipc_free": (i32, [vp]),
    "fpb_ipc_get_handle": (i32, [vp, vp]),
    "fpb_ipc_open": (i32, [vp, C.POINTER(vp)]),
    "fpb_ipc_close": (i32, [vp]),
    "fpb_peer_barrier": (i32, [vp, vp, vp, i32, i32, i32, vp]),
    "fpb_peer_all_reduce_max": (i32, [vp, vp, vp, i32, i32, vp, i32, vp]),
    "fpb_moe_gather": (i32, [vp, i32, sz, sz, vp, sz, vp, i32, vp]),
    "fpb_moe_gather_quantize": (i32, [vp, i32, sz, sz, vp, sz, vp, vp, vp, vp, vp, i32, vp, sz, vp]),
    "fpb_moe_gather_quantize_workspace_bytes": (sz, [sz, sz]),
    "fpb_swiglu": (i32, [vp, i32, sz, sz, vp, i32, vp]),
    "fpb_swiglu_quantize": (i32, [vp, i32, sz, vp, sz, vp, vp, vp, vp, i32, vp]),
    "fpb_nvfp4_grouped_gemm_swiglu_q": (i32, [vp, vp, vp, vp, sz, vp, vp, sz, vp, i32, vp, vp]),
    "fpb_rows_quantize": (i32, [vp, i32, sz, vp, vp, sz, vp, vp, vp, vp, i32, vp]),
    "fpb_act_amax": (i32, [vp, i32, sz, vp, i32, vp]),
    "fpb_swiglu_amax": (i32, [vp, i32, sz, vp, sz, vp, i32, vp]),
    "fpb_moe_combine": (i32, [vp, i32, sz, sz, vp, vp, sz, sz, sz, vp, i32, vp]),
    "fpb_moe_combine_add_norm": (i32, [vp, i32, sz, sz, vp, vp, sz, sz, sz, vp, vp, C.c_float, vp, vp, vp]),
    "fpb_moe_route_dest": (i32, [vp, sz, sz, sz, sz, vp, vp]),
    "fpb_moe_route_meta": (i32, [vp, vp, sz, sz, sz, sz, sz, vp, vp]),
    "fpb_embedding": (i32, [vp, sz, sz, vp, sz, vp, vp]),
    "fpb_rms_norm": (i32, [vp, i32, sz, vp, vp, sz, sz, vp, C.c_float, vp, i32, sz, vp]),
    "fpb_attn_prepare": (i32, [vp, sz, vp, sz, vp, sz, vp, vp, vp, sz, sz, sz, sz, sz, C.c_float, C.c_float, sz,
                               vp, vp, vp, vp]),
    "fpb_attn_decode_workspace_bytes": (sz, [sz, sz, sz, sz, sz]),
    "fpb_attn_decode": (i32, [vp, vp, vp, vp, vp, sz, sz, sz, sz, sz, sz, sz, C.c_float, vp, sz, vp, i32, vp]),
    "fpb_gdn_conv": (i32, [vp, sz, vp, vp, sz, sz, sz, vp, vp]),
    "fpb_gdn_delta": (i32, [vp, vp, vp, sz, vp, vp, vp, sz, sz, sz, sz, sz, C.c_float, vp, vp]),
    "fpb_gdn_gated_norm": (i32, [vp, vp, sz, vp, sz, sz, sz, C.c_float, vp, i32, vp]),
    "fpb_decode_combine_add_norm": (i32, [vp, vp, sz, sz, vp, vp, sz, sz, C.c_float, vp, vp, i32, vp]),
    "fpb_argmax_advance": (i32, [vp, sz, sz, vp, vp, vp, sz, vp, vp]),
    "fpb_nvfp4_expert_gemv_tokens": (i32, [vp, vp, i32, vp, i32, i32, sz, vp, i32, vp]),
    "fpb_moe_decode_plan": (i32, [vp, sz, sz, sz, sz, vp, vp, sz, vp, vp]),
    "fpb_nvfp4_gemv_planes_workspace_bytes": (sz, [sz, sz]),
    "fpb_nvfp4_gemv_planes": (i32, [vp, sz, sz, vp, i32, i32, vp, i32, vp, sz, vp]),
    "fpb_nvfp4_moe_gemv_planes": (i32, [vp, sz, vp, vp, i32, vp, i32, sz, i32, vp, i32, vp, sz, vp]),
    "fpb_nvfp4_moe_gemv_planes_glu": (i32, [vp, sz, vp, vp, i32, vp, sz, i32, vp, i32, vp, sz, vp]),
    "fpb_nvfp4_gemv_batch_create": (i32, [vp, i32, i32, i32, i32, vp, C.POINTER(vp)]),
    "fpb_nvfp4_gemv_batch_run": (i32, [vp, vp]),
    "fpb_nvfp4_gemv_batch_destroy": (i32, [vp]),
    "fpb_gdn_step": (i32, [vp, sz, vp, vp, sz, vp, vp, sz, vp, vp, vp, vp, sz, vp, sz, sz, sz, sz, sz, C.c_float, vp,
                           i32, vp]),
    "fpb_moe_decode_route": (i32, [vp, sz, C.c_longlong, sz, sz, sz, sz, vp, vp, vp, vp, sz, vp, vp]),
    "fpb_nvfp4_moe_gemv": (i32, [vp, sz, vp, vp, i32, vp, i32, sz, i32, vp, i32, vp]),
    "fpb_moe_decode_combine_add_norm": (i32, [vp, vp, vp, sz, sz, vp, vp, sz, sz, C.c_float, vp, vp, i32, vp]),
    "fpb_comm_available": (i32, []),
    "fpb_comm_version": (i32, [C.POINTER(i32)]),
    "fpb_comm_unique_id": (i32, [vp]),
    "fpb_comm_init": (i32, [vp, i32, i32, i32, C.POINTER(vp)]),
    "fpb_comm_destroy": (i32, [vp]),
    "fpb_comm_abort": (i32, [vp]),
    "fpb_comm_status": (i32, [vp]),
    "fpb_comm_size": (i32, [vp, C.POINTER(i32), C.POINTER(i32)]),
    "fpb_comm_all_gather": (i32, [vp, vp, vp, sz, i32, vp]),
    "fpb_comm_all_reduce": (i32, [vp, vp, vp, sz, i32, i32, vp]),
    "fpb_comm_all_to_all": (i32, [vp, vp, sizep, sizep, vp, sizep, sizep, i32, vp]),
    "fpb_moe_dims_validate": (i32, [sz, sz, sz, sz, sz]),
    "fpb_expert_selection_validate": (i32, [vp, vp, sz, sz, sz]),
    "fpb_prefill_layout_max_padded_rows": (i32, [sz, sz, sz, sz, C.POINTER(sz)]),
    "fpb_prefill_layout_host": (i32, [vp, vp, sz, sz, sz, sz, vp, sz, C.POINTER(sz), vp, sz,
                                      C.POINTER(sz), vp, vp]),
}

for _name, (_res, _args) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


def last_error() -> str:
    return lib.fpb_last_error().decode(errors="replace")


def check(status: int, func: str) -> None:
    if status != FPB_OK:
        raise FpbError(status, func, last_error())


def call(name: str, *args) -> None:
    """Calls an int-returning entry point and raises FpbError on failure."""
    check(getattr(lib, name)(*args), name)


def launch_count() -> int:
    return int(lib.fpb_launch_count())
