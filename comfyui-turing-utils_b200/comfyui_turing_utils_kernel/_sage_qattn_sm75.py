"""Drop-in for the reference's ``_sage_qattn_sm75`` extension (dense Sage and
dense W8A8-PV parts).

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


def _v_geometry(value):
    _check(value.is_cuda, "value must be a CUDA tensor")
    _check(value.dim() == 4, "Turing W8A8 V must be four-dimensional")
    _check(value.dtype in (torch.float16, torch.bfloat16), "Turing W8A8 V must be FP16 or BF16")
    _check(value.stride(3) == 1, "Turing W8A8 V head dimension must be contiguous")
    B, H, L, D = value.shape
    _check(D > 0 and D % 8 == 0, "Turing W8A8 V head dimension must be divisible by 8")
    _check(D in (64, 128), "the sm_100a V quantizer takes head_dim 64 or 128 (pad first)")
    return B, H, L, D


def quantize_v_int8_sm75(value, quantized, scale):
    """Channel-wise INT8 V (quant_v_int8_cuda_sm75.cu:166-246): fills the
    caller's int8 ``quantized`` [B, H, D, ceil(N/64)*64] (channel-major,
    padding 0, without the sm75 16-token fragment permutation) and fp32
    ``scale`` [B, H, D]."""
    B, H, L, D = _v_geometry(value)
    _check(quantized.is_cuda and scale.is_cuda, "V outputs must be CUDA tensors")
    _check(quantized.dtype == torch.int8 and quantized.is_contiguous(),
           "quantized V must be a contiguous int8 tensor")
    _check(scale.dtype == torch.float32 and scale.is_contiguous(),
           "V scale must be a contiguous float32 tensor")
    lpad = (L + 63) // 64 * 64
    _check(tuple(quantized.shape) == (B, H, D, lpad),
           "Turing W8A8 quantized V must be [B,H,D,ceil(N/64)*64]")
    _check(tuple(scale.shape) == (B, H, D), "Turing W8A8 V scale must be [B,H,D]")
    _check(value.device == quantized.device and value.device == scale.device,
           "Turing W8A8 V tensors must share a CUDA device")
    strides = (ctypes.c_int64 * 3)(value.stride(0), value.stride(1), value.stride(2))
    with torch.cuda.device(value.device):
        call("tb_quantize_v_int8", ptr(value), dtype_code(value), None, ptr(quantized), ptr(scale),
             B, H, L, D, lpad, strides, stream_of(value))


def quantize_v_codes(value, codes, scale):
    """The same channel-wise INT8 V written as exact fp16 integers in V's own
    [B, H, N, D] layout (``codes`` contiguous fp16): the PV operand of
    :func:`w8a8_attn`."""
    B, H, L, D = _v_geometry(value)
    _check(codes.is_cuda and codes.dtype == torch.float16 and codes.is_contiguous()
           and tuple(codes.shape) == (B, H, L, D), "V codes must be contiguous fp16 [B,H,N,D]")
    _check(scale.is_cuda and scale.dtype == torch.float32 and scale.is_contiguous()
           and tuple(scale.shape) == (B, H, D), "Turing W8A8 V scale must be [B,H,D]")
    strides = (ctypes.c_int64 * 3)(value.stride(0), value.stride(1), value.stride(2))
    with torch.cuda.device(value.device):
        call("tb_quantize_v_int8", ptr(value), dtype_code(value), ptr(codes), None, ptr(scale),
             B, H, L, D, 0, strides, stream_of(value))


def w8a8_attn(query_int8, key_int8, value_codes, value_scale, output, query_scale, key_scale,
              softmax_scale, is_causal):
    """Dense W8A8-PV attention on HND INT8 Q/K (D = 128), fp16 V codes
    [B, Hk, N, D] and fp32 V scales [B, Hk, D]; writes ``output``."""
    for name, t in (("query", query_int8), ("key", key_int8), ("value", value_codes),
                    ("value_scale", value_scale), ("output", output),
                    ("query_scale", query_scale), ("key_scale", key_scale)):
        _check(t.is_cuda, f"{name} must be a CUDA tensor")
    _check(query_int8.dtype == torch.int8 and key_int8.dtype == torch.int8,
           "prequantized Sol W8A8 Q/K must be int8")
    _check(query_int8.dim() == 4 and key_int8.dim() == 4 and output.dim() == 4,
           "prequantized Sol W8A8 Q/K/O must be four-dimensional")
    _check(query_int8.stride(-1) == 1 and key_int8.stride(-1) == 1 and output.stride(-1) == 1,
           "Q/K/O last dim must be contiguous")
    B, Hq, Lq, D = query_int8.shape
    Hk, Lk = key_int8.size(1), key_int8.size(2)
    _check(D == 128 and key_int8.size(3) == D,
           "the sm_100a W8A8 kernel takes head_dim 128 (pad 64-channel codes with zeros)")
    _check(tuple(output.shape) == tuple(query_int8.shape), "prequantized Sol W8A8 output must match Q")
    _check(output.dtype in (torch.float16, torch.bfloat16), "output must be float16 or bfloat16")
    _check(Hk > 0 and Hq % Hk == 0, "prequantized Sol W8A8 Q heads must be divisible by KV heads")
    _check(value_codes.dtype == torch.float16 and tuple(value_codes.shape) == (B, Hk, Lk, D)
           and value_codes.stride(-1) == 1, "prequantized Sol W8A8 V shape is incompatible")
    _check(value_scale.dtype == torch.float32 and value_scale.is_contiguous()
           and tuple(value_scale.shape) == (B, Hk, D), "prequantized Sol W8A8 V scale is incompatible")
    _check(query_scale.dtype == torch.float32 and key_scale.dtype == torch.float32
           and query_scale.is_contiguous() and key_scale.is_contiguous()
           and tuple(query_scale.shape) == (B, Hq, (Lq + 63) // 64 * 4)
           and tuple(key_scale.shape) == (B, Hk, (Lk + 63) // 64),
           "prequantized Sol W8A8 Q/K scale shapes are incompatible")
    strides = (ctypes.c_int64 * 12)(*_bhl(query_int8, 1), *_bhl(key_int8, 1),
                                    *_bhl(value_codes, 1), *_bhl(output, 1))
    with torch.cuda.device(query_int8.device):
        call("tb_w8a8_attn", ptr(query_int8), ptr(key_int8), ptr(value_codes), ptr(value_scale),
             ptr(output), dtype_code(output), ptr(query_scale), ptr(key_scale), B, Hq, Hk, Lq, Lk,
             D, strides, int(bool(is_causal)), float(softmax_scale), stream_of(query_int8))


def sol_sparse_online_w8a8_prequantized_attn(query_int8, key_int8, value_int8, value_scale, output,
                                             query_scale, key_scale, key_summary,
                                             key_score_summary, value_mean, key_summary_mean,
                                             key_summary_variance, sparse_query_blocks,
                                             exact_kv_blocks, threshold_sigma, residual_subblocks,
                                             softmax_scale, return_stats, force_dense,
                                             key_tile_tokens, is_causal, route_original_basis):
    """The dense (force_dense=1) path of sol_sparse_cuda_sm75.cu:2767-2932.
    ``value_int8`` is either the fp16 codes of :func:`quantize_v_codes`
    ([B, Hk, N, D]) or the reference's int8 [B, Hk, D, ceil(N/64)*64]
    (transposed to the fp16 operand layout first).  Returns the selected-block
    counter (a zero int64 [1] with return_stats, else empty), as the reference."""
    _check(force_dense in (0, 1), "force_dense must be 0 or 1")
    _check(is_causal in (0, 1), "is_causal must be 0 or 1")
    _check(int(key_tile_tokens) in (64, 128), "key_tile_tokens must be 64 or 128")
    _check(int(force_dense) == 1,
           "Sol sparse routing is not part of the sm_100a build; call with force_dense=1")
    Lk = key_int8.size(2)
    if value_int8.dtype == torch.int8:
        _check(value_int8.dim() == 4 and value_int8.size(3) == (Lk + 63) // 64 * 64,
               "prequantized Sol W8A8 V shape is incompatible")
        value_int8 = value_int8[..., :Lk].transpose(2, 3).to(torch.float16).contiguous()
    w8a8_attn(query_int8, key_int8, value_int8, value_scale, output, query_scale, key_scale,
              softmax_scale, is_causal)
    if return_stats:
        return torch.zeros(1, dtype=torch.int64, device=output.device)
    return torch.empty(0, dtype=torch.int64, device=output.device)
