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


def rms_rope_per_warp_int8(q: torch.Tensor, k: torch.Tensor, q_norm: torch.Tensor,
                           k_norm: torch.Tensor, freqs: torch.Tensor | None, *, epsilon: float,
                           rot_dim: int, tensor_layout: str, norm_scope: str, split_half: bool,
                           rotate_qk: bool, stabilize_k: bool, query_rrms=None, key_rrms=None):
    """Fused Q/K RMSNorm + RoPE into the production INT8 contract (quant.py:6-92):
    Q per 16-token warp tile, K per 64-token block, same output shapes.
    query_rrms / key_rrms ([B, L] fp32, row scope only; not in the
    reference): per-token reciprocal RMS computed by the caller, e.g. over
    heads held by several tensor-parallel ranks."""
    if tensor_layout == "HND":
        batch, q_heads, q_tokens, head_dim = q.shape
        _, k_heads, k_tokens, _ = k.shape
        layout_id = 1
    elif tensor_layout == "NHD":
        batch, q_tokens, q_heads, head_dim = q.shape
        _, k_tokens, k_heads, _ = k.shape
        layout_id = 0
    else:
        raise ValueError(f"Unknown tensor layout: {tensor_layout}")
    if head_dim not in (64, 128):
        raise ValueError("fused RMSNorm+RoPE Q/K quantization requires head_dim 64 or 128")
    if norm_scope not in {"head", "row"}:
        raise ValueError("norm_scope must be head or row")
    q_int8 = torch.empty(q.shape, dtype=torch.int8, device=q.device)
    k_int8 = torch.empty(k.shape, dtype=torch.int8, device=k.device)
    q_scale = torch.empty((batch, q_heads, ((q_tokens + 63) // 64) * 4), dtype=torch.float32,
                          device=q.device)
    k_scale = torch.empty((batch, k_heads, (k_tokens + 63) // 64), dtype=torch.float32,
                          device=k.device)
    given = query_rrms is not None or key_rrms is not None
    if given and (norm_scope != "row" or query_rrms is None or key_rrms is None):
        raise ValueError("query_rrms and key_rrms are given together, with norm_scope='row'")
    if given:
        q_rrms, k_rrms = query_rrms.contiguous(), key_rrms.contiguous()
    elif norm_scope == "row":
        q_rrms = torch.empty((batch, q_tokens), dtype=torch.float32, device=q.device)
        k_rrms = torch.empty((batch, k_tokens), dtype=torch.float32, device=k.device)
    else:
        q_rrms = torch.empty(0, dtype=torch.float32, device=q.device)
        k_rrms = torch.empty(0, dtype=torch.float32, device=k.device)
    if stabilize_k and rotate_qk:
        anchor_indices = torch.empty((batch, k_heads), dtype=torch.int32, device=k.device)
        anchor_values = torch.empty((batch, k_heads, head_dim), dtype=torch.float32,
                                    device=k.device)
    else:
        anchor_indices = torch.empty(0, dtype=torch.int32, device=k.device)
        anchor_values = torch.empty(0, dtype=torch.float32, device=k.device)
    if freqs is None:
        freqs = torch.empty(0, dtype=q.dtype, device=q.device)
    _fused.quant_qk_rms_rope_int8_cuda(
        q, k, q_int8, k_int8, q_scale, k_scale, q_norm, k_norm, freqs, q_rrms, k_rrms,
        anchor_indices, anchor_values, float(epsilon), int(rot_dim), 64, 16, 64, layout_id,
        (2 if given else 1) if norm_scope == "row" else 0, bool(split_half), bool(rotate_qk))
    return q_int8, q_scale, k_int8, k_scale


def row_sum_squares(x: torch.Tensor, tensor_layout: str = "HND") -> torch.Tensor:
    """[B, L] fp32 per-token sum of squares over all heads of x (the partial
    sums a tensor-parallel rank contributes to a row-scope RMSNorm)."""
    batch, _, tokens = _geometry(x, tensor_layout)
    sums = torch.empty((batch, tokens), dtype=torch.float32, device=x.device)
    _fused.row_sum_squares_cuda(x, sums, 0 if tensor_layout == "NHD" else 1)
    return sums



def per_warp_int8_hadamard(q: torch.Tensor, k: torch.Tensor, BLKQ: int = 64, WARPQ: int = 16,
                           BLKK: int = 64, tensor_layout: str = "HND", stabilize_k: bool = True):
    """Fuse the shared randomized Hadamard transform into Q/K quantization
    (quant.py:182-243): Q per 16-row warp tile, K per 64-key block, K first
    centred on its anchor row when stabilize_k and the anchor test passes."""
    batch, q_heads, q_tokens = _geometry(q, tensor_layout)
    _, kv_heads, kv_tokens = _geometry(k, tensor_layout)
    q_int8 = torch.empty(q.shape, dtype=torch.int8, device=q.device)
    k_int8 = torch.empty(k.shape, dtype=torch.int8, device=k.device)
    q_scale = torch.empty((batch, q_heads, ((q_tokens + BLKQ - 1) // BLKQ) * (BLKQ // WARPQ)),
                          device=q.device, dtype=torch.float32)
    k_scale = torch.empty((batch, kv_heads, (kv_tokens + BLKK - 1) // BLKK), device=q.device,
                          dtype=torch.float32)
    layout_id = 0 if tensor_layout == "NHD" else 1
    if stabilize_k:
        anchor_indices = torch.empty((batch, kv_heads), dtype=torch.int32, device=q.device)
        _fused.quant_qk_per_warp_int8_rotated_anchored_cuda(
            q, k, q_int8, k_int8, q_scale, k_scale, anchor_indices, BLKQ, WARPQ, BLKK, layout_id)
    else:
        _fused.quant_qk_per_warp_int8_rotated_cuda(q, k, q_int8, k_int8, q_scale, k_scale, BLKQ,
                                                   WARPQ, BLKK, layout_id)
    return q_int8, q_scale, k_int8, k_scale
