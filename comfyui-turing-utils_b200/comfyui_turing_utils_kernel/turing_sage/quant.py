"""Sage Q/K INT8 quantization helpers (kernel/comfyui_turing_utils_kernel/
turing_sage/quant.py:95-179): same functions, shapes and scale layouts."""
from __future__ import annotations

import torch

from .. import _sage_fused_sm75 as _fused


def _geometry(t: torch.Tensor, tensor_layout: str):
    if tensor_layout == "HND":
        batch, heads, tokens, _ = t.shape
    elif tensor_layout == "NHD":
        batch, tokens, heads, _ = t.shape
    else:
        raise ValueError(f"Unknown tensor layout: {tensor_layout}")
    return batch, heads, tokens


def quantize_query_per_warp(q: torch.Tensor, BLKQ: int = 64, WARPQ: int = 16,
                            tensor_layout: str = "HND"):
    q_int8 = torch.empty(q.shape, dtype=torch.int8, device=q.device)
    batch, heads, tokens = _geometry(q, tensor_layout)
    q_scale = torch.empty((batch, heads, ((tokens + BLKQ - 1) // BLKQ) * (BLKQ // WARPQ)),
                          device=q.device, dtype=torch.float32)
    layout_id = 0 if tensor_layout == "NHD" else 1
    _fused.quant_per_warp_int8_cuda(q, q_int8, q_scale, BLKQ, WARPQ, layout_id)
    return q_int8, q_scale


def quantize_key_per_block(k: torch.Tensor, BLKK: int = 64, tensor_layout: str = "HND",
                           smooth_k: bool = False):
    """Per-block INT8 K.  smooth_k=True subtracts the per-channel token mean
    first (softmax-invariant K smoothing); the reference ships this arithmetic
    (fused.cu:97-128) but leaves it unwired."""
    k_int8 = torch.empty(k.shape, dtype=torch.int8, device=k.device)
    batch, heads, tokens = _geometry(k, tensor_layout)
    k_scale = torch.empty((batch, heads, (tokens + BLKK - 1) // BLKK), device=k.device,
                          dtype=torch.float32)
    layout_id = 0 if tensor_layout == "NHD" else 1
    if smooth_k:
        mean = torch.empty((batch, heads, k.size(-1)), dtype=k.dtype, device=k.device)
        _fused.token_mean_cuda(k, mean, layout_id)
        _fused.quant_per_block_int8_smooth_cuda(k, k_int8, k_scale, mean, BLKK, layout_id)
    else:
        _fused.quant_per_block_int8_cuda(k, k_int8, k_scale, BLKK, layout_id)
    return k_int8, k_scale


def per_warp_int8(q: torch.Tensor, k: torch.Tensor, BLKQ: int = 64, WARPQ: int = 16,
                  BLKK: int = 64, tensor_layout: str = "HND", fuse_qk: bool = False,
                  smooth_k: bool = False):
    """Quantize Q per warp and K per block (quant.py:140-179)."""
    q_int8, q_scale = quantize_query_per_warp(q, BLKQ, WARPQ, tensor_layout)
    k_int8, k_scale = quantize_key_per_block(k, BLKK, tensor_layout, smooth_k=smooth_k)
    return q_int8, q_scale, k_int8, k_scale
