"""Sage INT8 attention facades (kernel/comfyui_turing_utils_kernel/turing_sage/
core.py:367-653): split prequantize / execute, head-dim padding, output
slicing, the same dataclass and validation messages.

The fused RMSNorm + RoPE Q/K prologue (core.py:222-285, 477-517) feeds the
same attention: prequantize_rms_rope_qk -> PrequantizedQK ->
prequantize_sageattn_from_qk -> sageattn_from_prequantized.

The dense W8A8-PV attention (core.py:656-708, 714-914, 916-990) follows the
reference's split: prequantize_sol_sageattn (rotated Q/K, channel-wise INT8
V) -> PrequantizedSolAttention -> sol_sparse_sageattn_from_prequantized, and
w8a8attn runs both.  Only the route-free dense specialization is built
(use_w8a8=True, force_dense=True); the Sol/SLA sparse routes are not.

Differences from the reference, by design:
  * no short-sequence SDPA fallback: the sm_100a kernel masks any length;
  * smooth_k=True is accepted (K mean smoothing, softmax-invariant); the
    reference rejects it in production (core.py:421-422);
  * head_dim <= 128 is padded to 128 (the kernel's one tile width).
"""
from __future__ import annotations

from dataclasses import dataclass
from functools import wraps
from typing import Any, Optional

import torch

from .. import _sage_qattn_sm75 as _qattn
from .quant import per_warp_int8, per_warp_int8_hadamard


@dataclass(frozen=True, slots=True)
class PrequantizedSageAttention:
    query_int8: torch.Tensor
    query_scale: torch.Tensor
    key_int8: torch.Tensor
    key_scale: torch.Tensor
    value: torch.Tensor
    tensor_layout: str
    original_head_dim: int
    is_causal: bool
    sm_scale: float


@dataclass(frozen=True, slots=True)
class PrequantizedQK:
    query_int8: torch.Tensor
    query_scale: torch.Tensor
    key_int8: torch.Tensor
    key_scale: torch.Tensor
    tensor_layout: str
    input_dtype: torch.dtype
    original_head_dim: int
    route_original_basis: bool = False


def _on_input_device(function):
    @wraps(function)
    def wrapped(q: torch.Tensor, *args, **kwargs):
        with torch.cuda.device(q.device):
            return function(q, *args, **kwargs)

    return wrapped


def _validate_fixed_qkv(q, k, v, tensor_layout: str) -> None:
    """core.py:323-340."""
    if tensor_layout not in {"HND", "NHD"}:
        raise ValueError(f"Unsupported tensor_layout: {tensor_layout}")
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("fixed-length Q/K/V must be four-dimensional")
    head_dim = q.size(-1)
    if k.size(-1) != head_dim or v.size(-1) != head_dim:
        raise ValueError("Q/K/V head dimensions must match")
    head_axis = 1 if tensor_layout == "HND" else 2
    seq_axis = 2 if tensor_layout == "HND" else 1
    if q.size(0) != k.size(0) or q.size(0) != v.size(0):
        raise ValueError("Q/K/V batch sizes must match")
    if k.size(head_axis) != v.size(head_axis) or k.size(seq_axis) != v.size(seq_axis):
        raise ValueError("K/V head counts and sequence lengths must match")
    if k.size(head_axis) == 0 or q.size(head_axis) % k.size(head_axis) != 0:
        raise ValueError("the Q head count must be divisible by the KV head count")
    if q.size(seq_axis) == 0 or k.size(seq_axis) == 0:
        raise ValueError("empty Q/K sequences are not supported")


@_on_input_device
def prequantize_sageattn(q, k, v, tensor_layout: str = "HND", is_causal: bool = False,
                         sm_scale: Optional[float] = None, smooth_k: bool = False,
                         **kwargs: Any) -> PrequantizedSageAttention:
    """Quantize Q (per 16-row warp tile) and K (per 64-key block) to INT8."""
    if not q.is_cuda:
        raise ValueError("Input tensors must be on CUDA")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("Turing Sage Q/K/V must be float16 or bfloat16")
    if q.device != k.device or q.device != v.device:
        raise ValueError("Q/K/V must be on the same device")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise TypeError("Q/K/V must have matching dtypes")
    _validate_fixed_qkv(q, k, v, tensor_layout)
    head_dim = q.size(-1)
    if head_dim > 128:
        raise ValueError(f"Unsupported head_dim: {head_dim}")
    padding = 128 - head_dim
    if padding:
        q = torch.nn.functional.pad(q, (0, padding))
        k = torch.nn.functional.pad(k, (0, padding))
        v = torch.nn.functional.pad(v, (0, padding))
    if q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1:
        raise ValueError("the last Q/K/V dimension must be contiguous")
    scale = float(sm_scale) if sm_scale is not None else head_dim ** -0.5
    q_int8, q_scale, k_int8, k_scale = per_warp_int8(q, k, tensor_layout=tensor_layout,
                                                     smooth_k=smooth_k)
    return PrequantizedSageAttention(q_int8, q_scale, k_int8, k_scale, v.contiguous(),
                                     tensor_layout, head_dim, bool(is_causal), scale)


@_on_input_device
def sageattn_prequantized(q_int8, q_scale, k_int8, k_scale, v, *, tensor_layout: str = "NHD",
                          is_causal: bool = False, sm_scale: Optional[float] = None,
                          return_lse: bool = False, output: Optional[torch.Tensor] = None):
    """core.py:573-653 checks, then the tcgen05 kernel."""
    if tensor_layout not in {"HND", "NHD"}:
        raise ValueError(f"Unsupported tensor_layout: {tensor_layout}")
    if q_int8.dtype != torch.int8 or k_int8.dtype != torch.int8:
        raise TypeError("prequantized Sage Q/K must be int8")
    if v.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("prequantized Sage V must be float16 or bfloat16")
    if q_int8.ndim != 4 or k_int8.ndim != 4 or v.ndim != 4:
        raise ValueError("prequantized Sage Q/K/V must be four-dimensional")
    head_axis = 1 if tensor_layout == "HND" else 2
    seq_axis = 2 if tensor_layout == "HND" else 1
    if (q_int8.size(0) != k_int8.size(0) or k_int8.size(head_axis) != v.size(head_axis)
            or k_int8.size(seq_axis) != v.size(seq_axis) or q_int8.size(-1) != k_int8.size(-1)
            or q_int8.size(-1) != v.size(-1)):
        raise ValueError("prequantized Sage Q/K/V shapes are incompatible")
    if q_int8.size(-1) != 128:
        raise ValueError("prequantized Sage on sm_100a requires head_dim 128 (pad smaller heads)")
    scale = float(sm_scale) if sm_scale is not None else q_int8.size(-1) ** -0.5
    if output is None:
        output = torch.empty(q_int8.shape, dtype=v.dtype, device=v.device)
    layout_id = 0 if tensor_layout == "NHD" else 1
    lse = _qattn.qk_int8_sv_f16_accum_f32_attn(
        q_int8.contiguous(), k_int8.contiguous(), v, output, q_scale.contiguous(),
        k_scale.contiguous(), layout_id, int(is_causal), 2, scale, int(return_lse))
    return (output, lse / 1.44269504) if return_lse else output


def sageattn_from_prequantized(quantized: PrequantizedSageAttention, *, return_lse: bool = False):
    with torch.cuda.device(quantized.query_int8.device):
        result = sageattn_prequantized(
            quantized.query_int8, quantized.query_scale, quantized.key_int8,
            quantized.key_scale, quantized.value, tensor_layout=quantized.tensor_layout,
            is_causal=quantized.is_causal, sm_scale=quantized.sm_scale, return_lse=return_lse)
    if return_lse:
        output, lse = result
        return output[..., :quantized.original_head_dim], lse
    return result[..., :quantized.original_head_dim]


@_on_input_device
def sageattn(q, k, v, tensor_layout: str = "HND", is_causal: bool = False,
             sm_scale: Optional[float] = None, return_lse: bool = False, smooth_k: bool = False,
             **kwargs: Any):
    """Sage INT8 attention: per-warp INT8 Q, per-block INT8 K (optionally mean
    smoothed), 16-bit PV with fp32 accumulation (core.py:543-570)."""
    quantized = prequantize_sageattn.__wrapped__(q, k, v, tensor_layout=tensor_layout,
                                                 is_causal=is_causal, sm_scale=sm_scale,
                                                 smooth_k=smooth_k)
    return sageattn_from_prequantized(quantized, return_lse=return_lse)


@_on_input_device
def prequantize_rms_rope_qk(q, k, q_norm, k_norm, freqs, *, epsilon: float, rot_dim: int,
                            tensor_layout: str = "HND", norm_scope: str = "head",
                            split_half: bool = False, rotate_qk: bool = False,
                            stabilize_k: bool = False) -> PrequantizedQK:
    """Normalize, rotate (RoPE) and quantize Q/K (core.py:222-285).  Without
    rotate_qk the 16-bit intermediates are never materialized; the
    Hadamard-rotated form (rotate_qk, optionally stabilize_k) that feeds the
    W8A8 attention writes them once and codes them in a second pass."""
    if not q.is_cuda or not k.is_cuda:
        raise ValueError("Q/K inputs must be on CUDA")
    if q.device != k.device:
        raise ValueError("Q/K inputs must share one CUDA device")
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype:
        raise TypeError("fused Q/K preprocessing requires matching FP16 or BF16 inputs")
    if q.ndim != 4 or k.ndim != 4 or q.shape[0] != k.shape[0] or q.shape[-1] != k.shape[-1]:
        raise ValueError("fused Q/K preprocessing requires compatible four-dimensional tensors")
    if q.stride(-1) != 1 or k.stride(-1) != 1:
        raise ValueError("the last Q/K dimension must be contiguous")
    head_dim = int(q.shape[-1])
    if head_dim not in (64, 128):
        raise ValueError("fused Q/K preprocessing requires head_dim 64 or 128")
    q_norm = q_norm.to(device=q.device, dtype=q.dtype).contiguous()
    k_norm = k_norm.to(device=q.device, dtype=q.dtype).contiguous()
    if freqs is None:
        freqs = torch.empty(0, device=q.device, dtype=q.dtype)
    else:
        freqs = freqs.to(device=q.device, dtype=q.dtype)
    from .custom_ops import qk_rms_rope_int8

    q_int8, q_scale, k_int8, k_scale = qk_rms_rope_int8(
        q, k, q_norm, k_norm, freqs, epsilon=float(epsilon), rot_dim=int(rot_dim),
        tensor_layout=tensor_layout, norm_scope=norm_scope, split_half=bool(split_half),
        rotate_qk=bool(rotate_qk), stabilize_k=bool(stabilize_k))
    return PrequantizedQK(q_int8, q_scale, k_int8, k_scale, tensor_layout, q.dtype, head_dim,
                          bool(rotate_qk))


def prequantize_sageattn_from_qk(qk: PrequantizedQK, value: torch.Tensor, *,
                                 is_causal: bool = False,
                                 sm_scale: Optional[float] = None) -> PrequantizedSageAttention:
    """Attach V to a fused Q/K result without rereading Q/K (core.py:477-517).
    Head dims below 128 are zero-padded: zero INT8 codes add nothing to QK^T."""
    if qk.tensor_layout not in {"HND", "NHD"}:
        raise ValueError(f"Unsupported tensor_layout: {qk.tensor_layout}")
    if value.dtype != qk.input_dtype:
        raise TypeError("preprocessed Q/K and V must have matching logical dtypes")
    if value.device != qk.query_int8.device:
        raise ValueError("preprocessed Q/K and V must share one CUDA device")
    if value.ndim != 4 or value.stride(-1) != 1:
        raise ValueError("preprocessed Sage V must be four-dimensional with contiguous channels")
    head_axis = 1 if qk.tensor_layout == "HND" else 2
    seq_axis = 2 if qk.tensor_layout == "HND" else 1
    if (value.size(0) != qk.key_int8.size(0)
            or value.size(head_axis) != qk.key_int8.size(head_axis)
            or value.size(seq_axis) != qk.key_int8.size(seq_axis)
            or value.size(-1) != qk.key_int8.size(-1)):
        raise ValueError("preprocessed Q/K and V shapes are incompatible")
    scale = float(sm_scale) if sm_scale is not None else qk.original_head_dim ** -0.5
    q_int8, k_int8 = qk.query_int8, qk.key_int8
    padding = 128 - value.size(-1)
    if padding:
        q_int8 = torch.nn.functional.pad(q_int8, (0, padding))
        k_int8 = torch.nn.functional.pad(k_int8, (0, padding))
        value = torch.nn.functional.pad(value, (0, padding))
    return PrequantizedSageAttention(q_int8, qk.query_scale, k_int8, qk.key_scale,
                                     value.contiguous(), qk.tensor_layout,
                                     qk.original_head_dim, bool(is_causal), scale)



# --------------------------------------------------------- dense W8A8-PV ----

@dataclass(frozen=True, slots=True)
class PrequantizedSolAttention:
    """core.py:50-72.  ``value_int8`` holds V's INT8 codes as exact fp16 values
    in V's [B, Hk, N, D] layout (the sm_100a PV operand); the summaries and
    routing blocks of the sparse variants stay empty."""
    query_int8: torch.Tensor
    query_scale: torch.Tensor
    key_int8: torch.Tensor
    key_scale: torch.Tensor
    value: Optional[torch.Tensor]
    value_int8: torch.Tensor
    value_scale: torch.Tensor
    summaries: tuple
    sparse_query_blocks: torch.Tensor
    exact_kv_blocks: torch.Tensor
    output_dtype: torch.dtype
    sm_scale: float
    threshold_sigma: float
    residual_subblocks: int
    possible_blocks: int
    use_w8a8: bool
    force_dense: bool
    original_head_dim: int
    key_tile_tokens: int
    is_causal: bool
    route_original_basis: bool


def _pad_codes(t: torch.Tensor, width: int) -> torch.Tensor:
    return t if t.size(-1) == width else torch.nn.functional.pad(t, (0, width - t.size(-1)))


def prequantize_sol_sageattn_from_qk(qk: PrequantizedQK, value: torch.Tensor, *,
                                     sm_scale: Optional[float] = None, dense_query_ranges=(),
                                     exact_kv_ranges=(), threshold_sigma: float = 1.0,
                                     residual_subblocks: int = 1, use_w8a8: bool = False,
                                     force_dense: bool = False, key_tile_tokens: int = 0,
                                     is_causal: bool = False) -> PrequantizedSolAttention:
    """Attach V to an already quantized Q/K pair (core.py:714-839), dense W8A8 only."""
    if qk.tensor_layout != "HND":
        raise ValueError("prequantized Sol/W8A8 attention requires HND layout")
    if value.dtype != qk.input_dtype:
        raise TypeError("preprocessed Q/K and V must have matching logical dtypes")
    if value.device != qk.query_int8.device:
        raise ValueError("preprocessed Q/K and V must share one CUDA device")
    if value.ndim != 4 or value.stride(-1) != 1:
        raise ValueError("preprocessed Sol V must be four-dimensional with contiguous channels")
    if (value.size(0) != qk.key_int8.size(0) or value.size(1) != qk.key_int8.size(1)
            or value.size(2) != qk.key_int8.size(2) or value.size(3) != qk.key_int8.size(3)):
        raise ValueError("preprocessed Q/K and V shapes are incompatible")
    key_tile_tokens = int(key_tile_tokens)
    if key_tile_tokens not in (0, 64, 128):
        raise ValueError("key_tile_tokens must be 0 (auto), 64, or 128")
    if key_tile_tokens == 0:
        key_tile_tokens = 128 if qk.key_int8.size(2) > 1024 else 64
    residual_subblocks = int(residual_subblocks)
    if residual_subblocks not in (1, 2):
        raise ValueError("residual_subblocks must be 1 or 2")
    if is_causal and (not use_w8a8 or not force_dense):
        raise ValueError("causal masking is supported only by dense W8A8")
    if not use_w8a8 or not force_dense or dense_query_ranges or exact_kv_ranges:
        raise ValueError("only the dense W8A8 attention (use_w8a8=True, force_dense=True) is "
                         "built; the Sol sparse routes are not part of this package")
    B, Hk, L, D = value.shape
    value_codes = torch.empty((B, Hk, L, D), dtype=torch.float16, device=value.device)
    value_scale = torch.empty((B, Hk, D), dtype=torch.float32, device=value.device)
    _qattn.quantize_v_codes(value, value_codes, value_scale)
    scale = float(sm_scale) if sm_scale is not None else qk.original_head_dim ** -0.5
    # The tcgen05 kernel's tile is 128 channels: 64-channel codes and V codes
    # are zero-padded (zero codes add nothing to either contraction).
    q_int8 = _pad_codes(qk.query_int8, 128)
    k_int8 = _pad_codes(qk.key_int8, 128)
    value_codes = _pad_codes(value_codes, 128)
    value_scale = _pad_codes(value_scale, 128).contiguous()
    query_blocks = (qk.query_int8.size(2) + 63) // 64
    key_blocks = (qk.key_int8.size(2) + 63) // 64
    empty_u8 = torch.empty(0, dtype=torch.uint8, device=value.device)
    return PrequantizedSolAttention(
        query_int8=q_int8, query_scale=qk.query_scale, key_int8=k_int8, key_scale=qk.key_scale,
        value=None, value_int8=value_codes, value_scale=value_scale, summaries=(),
        sparse_query_blocks=torch.zeros(query_blocks, dtype=torch.uint8, device=value.device),
        exact_kv_blocks=torch.zeros(key_blocks, dtype=torch.uint8, device=value.device)
        if key_blocks else empty_u8,
        output_dtype=value.dtype, sm_scale=scale, threshold_sigma=float(threshold_sigma),
        residual_subblocks=residual_subblocks, possible_blocks=0, use_w8a8=True,
        force_dense=True, original_head_dim=qk.original_head_dim,
        key_tile_tokens=key_tile_tokens, is_causal=bool(is_causal),
        route_original_basis=bool(qk.route_original_basis))


@_on_input_device
def prequantize_sol_sageattn(q, k, v, *, tensor_layout: str = "HND",
                             sm_scale: Optional[float] = None, dense_query_ranges=(),
                             exact_kv_ranges=(), threshold_sigma: float = 1.0,
                             residual_subblocks: int = 1, use_w8a8: bool = False,
                             force_dense: bool = False, key_tile_tokens: int = 0,
                             rotate_qk: bool = True, stabilize_k: bool = True,
                             is_causal: bool = False) -> PrequantizedSolAttention:
    """Prepare W8A8 Q/K/V before output allocation (core.py:842-914)."""
    if not q.is_cuda:
        raise ValueError("Input tensors must be on CUDA")
    if tensor_layout != "HND":
        raise ValueError("Sol sparse attention currently requires HND layout")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("Sol sparse Q/K/V must be float16 or bfloat16")
    if q.device != k.device or q.device != v.device:
        raise ValueError("Q/K/V must be on the same device")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise TypeError("Q/K/V must have matching dtypes")
    _validate_fixed_qkv(q, k, v, tensor_layout)
    head_dim = q.size(-1)
    if not 0 < head_dim <= 128:
        raise ValueError("Sol sparse attention requires head_dim in [1, 128]")
    if q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1:
        raise ValueError("the last Q/K/V dimension must be contiguous")
    kernel_head_dim = 64 if head_dim <= 64 else 128
    if head_dim < kernel_head_dim:
        padding = kernel_head_dim - head_dim
        q = torch.nn.functional.pad(q, (0, padding))
        k = torch.nn.functional.pad(k, (0, padding))
        v = torch.nn.functional.pad(v, (0, padding))
    if rotate_qk:
        q_int8, q_scale, k_int8, k_scale = per_warp_int8_hadamard(
            q, k, tensor_layout="HND", stabilize_k=bool(stabilize_k))
    else:
        q_int8, q_scale, k_int8, k_scale = per_warp_int8(q, k, tensor_layout="HND", fuse_qk=True)
    qk = PrequantizedQK(q_int8, q_scale, k_int8, k_scale, "HND", v.dtype, head_dim,
                        bool(rotate_qk))
    return prequantize_sol_sageattn_from_qk(
        qk, v, sm_scale=sm_scale, dense_query_ranges=dense_query_ranges,
        exact_kv_ranges=exact_kv_ranges, threshold_sigma=threshold_sigma,
        residual_subblocks=residual_subblocks, use_w8a8=use_w8a8, force_dense=force_dense,
        key_tile_tokens=key_tile_tokens, is_causal=is_causal)


def sol_sparse_sageattn_from_prequantized(quantized: PrequantizedSolAttention, *,
                                          return_stats: bool = False):
    """core.py:916-990, dense W8A8 only."""
    with torch.cuda.device(quantized.query_int8.device):
        output = torch.empty(quantized.query_int8.shape, dtype=quantized.output_dtype,
                             device=quantized.query_int8.device)
        selected = _qattn.sol_sparse_online_w8a8_prequantized_attn(
            quantized.query_int8, quantized.key_int8, quantized.value_int8,
            quantized.value_scale, output, quantized.query_scale, quantized.key_scale,
            None, None, None, None, None, quantized.sparse_query_blocks,
            quantized.exact_kv_blocks, quantized.threshold_sigma, quantized.residual_subblocks,
            quantized.sm_scale, int(return_stats), int(quantized.force_dense),
            quantized.key_tile_tokens, int(quantized.is_causal),
            int(quantized.route_original_basis))
    output = output[..., :quantized.original_head_dim]
    return (output, selected, quantized.possible_blocks) if return_stats else output


@_on_input_device
def w8a8attn(q, k, v, *, tensor_layout: str = "HND", is_causal: bool = False,
             sm_scale: Optional[float] = None, key_tile_tokens: int = 0,
             rotate_qk: bool = True, stabilize_k: bool = True):
    """Dense INT8 QK / u8 x s8 PV attention (core.py:656-708): rotated INT8
    Q/K, channel-wise INT8 V, probabilities packed to u8 codes."""
    if tensor_layout not in {"HND", "NHD"}:
        raise ValueError(f"Unsupported tensor_layout: {tensor_layout}")
    if tensor_layout == "NHD":
        q_hnd = q.transpose(1, 2).contiguous()
        k_hnd = k.transpose(1, 2).contiguous()
        v_hnd = v.transpose(1, 2).contiguous()
    else:
        q_hnd, k_hnd, v_hnd = q, k, v
    _validate_fixed_qkv(q_hnd, k_hnd, v_hnd, "HND")
    if q_hnd.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("Turing W8A8 Q/K/V must be float16 or bfloat16")
    if q_hnd.dtype != k_hnd.dtype or q_hnd.dtype != v_hnd.dtype:
        raise TypeError("Turing W8A8 Q/K/V must have matching dtypes")
    head_dim = q_hnd.size(-1)
    if not 0 < head_dim <= 128:
        raise ValueError("Turing W8A8 requires head_dim in [1, 128]")
    quantized = prequantize_sol_sageattn.__wrapped__(
        q_hnd, k_hnd, v_hnd, tensor_layout="HND", sm_scale=sm_scale, threshold_sigma=0.0,
        residual_subblocks=1, use_w8a8=True, force_dense=True, key_tile_tokens=key_tile_tokens,
        rotate_qk=rotate_qk, stabilize_k=stabilize_k, is_causal=bool(is_causal))
    output = sol_sparse_sageattn_from_prequantized(quantized)
    return output.transpose(1, 2) if tensor_layout == "NHD" else output
