"""Drop-in for the reference's ``_sage_qattn_sm75`` extension (dense Sage part).

``qk_int8_sv_f16_accum_f32_attn`` keeps the reference's name, argument order
and checks (kernel/csrc/turing/sage/qk_int_sv_f16_cuda_sm75.cu:984-1123) and
runs the tcgen05 attention kernel of libturing_b200.so.  The output tensor is
caller-allocated and written in place; the return value is the base-2 LSE
(or an empty tensor), as in the reference.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import call, dtype_code, ptr, stream_of


def _check(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _bhl(t: torch.Tensor, layout: int):
    if layout == 0:  # NHD
        return t.stride(0), t.stride(2), t.stride(1)
    return t.stride(0), t.stride(1), t.stride(2)


def qk_int8_sv_f16_accum_f32_attn(query, key, value, output, query_scale, key_scale,
                                  tensor_layout, is_causal, qk_quant_gran, sm_scale, return_lse):
    for name, t in (("query", query), ("key", key), ("value", value), ("output", output),
                    ("query_scale", query_scale), ("key_scale", key_scale)):
        _check(t.is_cuda, f"{name} must be a CUDA tensor")
    _check(query.is_contiguous() and key.is_contiguous(), "query and key must be contiguous")
    _check(value.stride(-1) == 1 and output.stride(-1) == 1,
           "value and output last dim must be contiguous")
    _check(query_scale.is_contiguous() and key_scale.is_contiguous(), "scales must be contiguous")
    _check(query.dtype == torch.int8 and key.dtype == torch.int8, "query and key must be int8")
    _check(value.dtype in (torch.float16, torch.bfloat16), "value must be float16 or bfloat16")
    _check(query_scale.dtype == torch.float32 and key_scale.dtype == torch.float32,
           "scales must be float32")
    _check(query.dim() == 4 and key.dim() == 4 and value.dim() == 4 and output.dim() == 4,
           "query, key, value and output must be 4D")
    _check(query_scale.dim() == 3 and key_scale.dim() == 3, "scales must be 3D")
    _check(qk_quant_gran == 2, "production Turing Sage requires per-warp Q/K quantization")
    layout = int(tensor_layout)
    _check(layout in (0, 1), "tensor_layout must be 0 or 1")
    B, D = query.size(0), query.size(3)
    if layout == 0:
        Lq, Hq, Lk, Hk = query.size(1), query.size(2), key.size(1), key.size(2)
        _check(tuple(key.shape) == (B, Lk, Hk, D) and tuple(value.shape) == (B, Lk, Hk, D),
               "key/value shape mismatch")
    else:
        Hq, Lq, Hk, Lk = query.size(1), query.size(2), key.size(1), key.size(2)
        _check(tuple(key.shape) == (B, Hk, Lk, D) and tuple(value.shape) == (B, Hk, Lk, D),
               "key/value shape mismatch")
    _check(Hq % Hk == 0, f"num_qo_heads ({Hq}) must be divisible by num_kv_heads ({Hk})")
    _check(tuple(query_scale.shape) == (B, Hq, (Lq + 63) // 64 * 4), "query_scale shape mismatch")
    _check(tuple(key_scale.shape) == (B, Hk, (Lk + 63) // 64), "key_scale shape mismatch")
    _check(output.dtype == value.dtype and tuple(output.shape) == tuple(query.shape),
           "output must match query's shape and value's dtype")
    lse = torch.empty(0, dtype=torch.float32)
    if return_lse:
        lse = torch.empty((B, Hq, Lq), dtype=torch.float32, device=query.device)
    strides = (ctypes.c_int64 * 12)(*_bhl(query, layout), *_bhl(key, layout),
                                    *_bhl(value, layout), *_bhl(output, layout))
    with torch.cuda.device(query.device):
        call("tb_qk_int8_sv_f16_accum_f32_attn", ptr(query), ptr(key), ptr(value),
             dtype_code(value), ptr(output), dtype_code(output), ptr(query_scale), ptr(key_scale),
             ptr(lse) if return_lse else None, B, Hq, Hk, Lq, Lk, D, strides, layout,
             int(is_causal), int(qk_quant_gran), float(sm_scale), stream_of(query))
    return lse
