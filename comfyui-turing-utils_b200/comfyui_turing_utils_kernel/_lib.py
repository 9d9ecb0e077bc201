"""ctypes binding of libturing_b200.so (the C ABI declared in include/turing_b200.h).

The library is loaded from this package directory.  There is no fallback: if
the shared object is missing or cannot be loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libturing_b200.so"

TB_OK = 0
TB_ERR_INVALID = 1
TB_ERR_CUDA = 2
TB_ERR_UNSUPPORTED = 3
TB_ERR_INTERNAL = 4

TB_DTYPE_BF16 = 0
TB_DTYPE_F16 = 1
TB_DTYPE_F32 = 2
TB_LAYOUT_NHD = 0
TB_LAYOUT_HND = 1

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int

# name -> argtypes (all entry points return int).
SIGNATURES: dict[str, list] = {
    "tb_abi_version": [],
    "tb_device_error": [_p],
    "tb_bf16_int8_convrot_quantize": [_p, _i64, _i64, _int, _int, _p, _p, _p],
    "tb_bf16_int4_convrot_quantize": [_p, _i64, _i64, _int, _p, _p, _p],
    "tb_bf16_gelu_int8_convrot_quantize": [_p, _i64, _i64, _p, _p, _p],
    "tb_bf16_gelu_int4_convrot_quantize": [_p, _i64, _i64, _p, _p, _p],
    "tb_swiglu_int8_convrot_quantize": [_p, _int, _i64, _i64, _p, _p, _p, _p, _p],
    "tb_swiglu_int4_convrot_quantize": [_p, _int, _i64, _i64, _p, _p, _p, _p, _p],
    "tb_gelu_int8_convrot_quantize": [_p, _int, _i64, _i64, _p, _p, _p, _p, _p],
    "tb_gelu_int4_convrot_quantize": [_p, _int, _i64, _i64, _p, _p, _p, _p, _p],
    "tb_swiglu_int8_convrot_quantize_noalloc": [_p, _int, _i64, _i64, _p, _p, _p],
    "tb_int8_linear": [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _int, _p],
    "tb_quant_qk_rms_rope_int8": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64,
                                  _i64, _i64, _i64, _p, _p, _i64, _i64, _i64, _int, _int, _int,
                                  ctypes.c_float, _p],
    "tb_row_sum_squares": [_p, _p, _i64, _i64, _i64, _i64, _p, _int, _p],
    "tb_segmented_rms_adaln": [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _int,
                               ctypes.c_float, _p],
    "tb_layer_norm_adaln": [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _int, ctypes.c_float, _p],
    "tb_w4a8_linear": [_p, _p, _p, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _int, _p],
    "tb_int4_linear": [_p, _p, _p, _p, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _p],
    "tb_codebook_w4a8_linear": [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64,
                                _int, _int, _p],
    "tb_int8_gemm_s32": [_p, _p, _p, _i64, _i64, _i64, _i64, _p],
    "tb_dequantize_int8_bf16": [_p, _i64, _p, _p, _i64, _p, _i64, _i64, _p],
    "tb_gated_residual_add": [_p, _i64, _p, _i64, _p, _i64, _i64, _p],
    "tb_quant_per_block_int8": [_p, _int, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _int,
                                _int, _p, _p],
    "tb_quant_per_warp_int8": [_p, _int, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _int,
                               _int, _int, _p],
    "tb_token_mean": [_p, _int, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _int, _p],
    "tb_qk_int8_sv_f16_accum_f32_attn": [_p, _p, _p, _int, _p, _int, _p, _p, _p, _i64, _i64,
                                         _i64, _i64, _i64, _i64, _p, _int, _int, _int,
                                         ctypes.c_float, _p],
    "tb_quant_qk_int8_rotated": [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64,
                                 _i64, _p, _int, _int, _int, _p],
    "tb_qk_rms_rope_apply": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64,
                             _i64, _p, _p, _i64, _i64, _i64, _int, _int, _int, ctypes.c_float,
                             _p],
    "tb_qk_anchor_processed": [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _p, _i64, _i64,
                               _i64, _int, _int, _int, ctypes.c_float, _p],
    "tb_quantize_v_int8": [_p, _int, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p],
    "tb_w8a8_attn": [_p, _p, _p, _p, _p, _int, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p,
                     _int, ctypes.c_float, _p],
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the native library (raises if it is missing — there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise ImportError(
                f"libturing_b200.so not found at {LIB_PATH}; build it with "
                "`make -C comfyui-turing-utils_b200/csrc` (sm_100a)")
        lib = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_LOCAL if hasattr(os, "RTLD_LOCAL") else 0)
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int
        lib.tb_last_error.argtypes = []
        lib.tb_last_error.restype = ctypes.c_char_p
        _lib = lib
    return _lib


def last_error() -> str:
    return (load().tb_last_error() or b"").decode("utf-8", "replace")


def call(name: str, *args) -> None:
    """Invoke a C entry point; a non-zero status raises RuntimeError with the
    library's message (the reference's TORCH_CHECK failures surface as
    RuntimeError too)."""
    status = getattr(load(), name)(*args)
    if status != TB_OK:
        msg = last_error()
        if status == TB_ERR_UNSUPPORTED:
            raise RuntimeError(msg or f"{name}: unsupported device")
        raise RuntimeError(msg or f"{name} failed with status {status}")


def device_error() -> int:
    """Read and clear the device watchdog word of the current device (0 = ok)."""
    code = ctypes.c_int(0)
    call("tb_device_error", ctypes.byref(code))
    return int(code.value)


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def float_dtype_code(t: torch.Tensor) -> int:
    """dtype code of a float16 / bfloat16 / float32 tensor (norm + AdaLN ops)."""
    if t.dtype == torch.float32:
        return TB_DTYPE_F32
    return dtype_code(t)


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return TB_DTYPE_BF16
    if t.dtype == torch.float16:
        return TB_DTYPE_F16
    raise TypeError("input must be float16 or bfloat16")
