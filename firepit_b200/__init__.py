"""firepit_b200 — B200-native (sm_100a) quantized-matmul hot path of firepit.

The CUDA kernels live in ``libfirepit_b200.so`` behind a C ABI
(``include/firepit_b200.h``); this package is the host-side mirror of
firepit-kernels' entry points.  Importing it loads the library and fails if
the library is missing: there is no CPU fallback.
"""
from . import _native
from ._native import FpbError, launch_count
from .gemv import (DEFAULT_GEMV_TILE, BatchedGemv, ExpertGemvView, Gemv, GemvTile, PlanesGemvBatch, ShapeError,
                   expert_gemv_weight_view, fp8_tile, gemv, gemv_batch_planes, gemv_batched, row_scaled_tile)
from .moe import (ExpertSelection, ExpertSelectionError, MoeDimensionError, MoeDims, PrefillLayout, PrefillPlan,
                  layout_scratch,
                  combine, combine_add_norm_prefill, combine_add_norm_view, combine_prefill, gather_prefill_view,
                  gather_quantize, swiglu, swiglu_quantize, topk_device)
from .sink import Async, Dry, Eager, Graph, Traced
from .synth import synth_normal
from .weights import (NVFP4_GROUP, Q8_BLOCK, FormatError, HostNvfp4Matrix, Nvfp4Matrix, current_stream_handle,
                      quantize_nvfp4)

from .gemm import (DEFAULT_GEMM_TILE, DEFAULT_GROUPED_GEMM_TILE, GemmTile, Nvfp4Gemm, Nvfp4GemmBatch,
                   Nvfp4GroupedGemmView, device_error, nvfp4_gemm, nvfp4_gemm_batch, nvfp4_gemm_view,
                   nvfp4_grouped_gemm_q, nvfp4_grouped_gemm_swiglu_q, nvfp4_grouped_gemm_view, quantize_act,
                   rows_quantize)
from .fp8 import (Fp8Gemm, Fp8GroupedGemmView, Fp8Matrix, Fp8Scaling, HostFp8Matrix, fp8_gemm, fp8_gemm_view,
                  fp8_grouped_gemm_q, fp8_grouped_gemm_view, quantize_fp8)
from .checkpoint import (Checkpoint, CheckpointError, Fp8Config, HostBf16Weight, ModelOptConfig, Quantization,
                         SafetensorsFile, WeightFormat, check_companions, load_experts, load_weight, stack_weights,
                         verify_formats)

__version__ = _native.lib.fpb_version().decode()
