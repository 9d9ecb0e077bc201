"""B200 (sm_100a) implementation of the comfyui-turing-utils kernel package.

Import-compatible with the reference package ``comfyui_turing_utils_kernel``
(kernel/comfyui_turing_utils_kernel/__init__.py): the same ``turing_*``
functions and ``turing_utils::*`` custom ops, backed by hand-written sm_100a
kernels in libturing_b200.so (C ABI: include/turing_b200.h).
"""
from .ops import (
    turing_bf16_gelu_int4_convrot_quantize,
    turing_bf16_gelu_int8_convrot_quantize,
    turing_bf16_int4_convrot_quantize,
    turing_bf16_int8_convrot_quantize,
    turing_codebook_w4a8_linear,
    turing_dequantize_int8_bf16,
    turing_gelu_int4_convrot_quantize,
    turing_gelu_int8_convrot_quantize,
    turing_int4_linear,
    turing_layer_norm_adaln,
    turing_int8_gemm_s32,
    turing_int8_linear,
    turing_swiglu_int4_convrot_quantize,
    turing_segmented_rms_adaln,
    turing_swiglu_int8_convrot_quantize,
    turing_w4a8_linear,
)
from . import checkpoint, turing_sage

__version__ = "0.29.1"

__all__ = [
    "turing_bf16_int8_convrot_quantize",
    "turing_bf16_int4_convrot_quantize",
    "turing_bf16_gelu_int8_convrot_quantize",
    "turing_bf16_gelu_int4_convrot_quantize",
    "turing_codebook_w4a8_linear",
    "turing_dequantize_int8_bf16",
    "turing_gelu_int8_convrot_quantize",
    "turing_gelu_int4_convrot_quantize",
    "turing_int4_linear",
    "turing_int8_gemm_s32",
    "turing_int8_linear",
    "turing_swiglu_int8_convrot_quantize",
    "turing_swiglu_int4_convrot_quantize",
    "turing_w4a8_linear",
    "turing_segmented_rms_adaln",
    "turing_layer_norm_adaln",
    "turing_sage",
]
