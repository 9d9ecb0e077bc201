"""``turing_utils::sage_attention`` (turing_sage/custom_ops.py:137-167),
``turing_utils::w8a8_attention`` (custom_ops.py:170-210) and
``turing_utils::qk_rms_rope_int8`` (custom_ops.py:63-130) custom ops: same
schemas and fake implementations, backed by the sm_100a kernels."""
from __future__ import annotations

import torch


@torch.library.custom_op("turing_utils::sage_attention", mutates_args=())
def sage_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                   tensor_layout: str, is_causal: bool, sm_scale: float) -> torch.Tensor:
    from .core import sageattn

    return sageattn(query, key, value, tensor_layout=tensor_layout, is_causal=is_causal,
                    sm_scale=sm_scale if sm_scale > 0.0 else None, smooth_k=False)


@sage_attention.register_fake
def _sage_attention_fake(query, key, value, tensor_layout, is_causal, sm_scale):
    return torch.empty_like(query)


@torch.library.custom_op("turing_utils::qk_rms_rope_int8", mutates_args=())
def qk_rms_rope_int8(query: torch.Tensor, key: torch.Tensor, query_norm: torch.Tensor,
                     key_norm: torch.Tensor, freqs: torch.Tensor, epsilon: float, rot_dim: int,
                     tensor_layout: str, norm_scope: str, split_half: bool, rotate_qk: bool,
                     stabilize_k: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor,
                                                 torch.Tensor]:
    from .quant import rms_rope_per_warp_int8

    return rms_rope_per_warp_int8(query, key, query_norm, key_norm,
                                  freqs if freqs.numel() else None, epsilon=epsilon,
                                  rot_dim=rot_dim, tensor_layout=tensor_layout,
                                  norm_scope=norm_scope, split_half=split_half,
                                  rotate_qk=rotate_qk, stabilize_k=stabilize_k)


@qk_rms_rope_int8.register_fake
def _qk_rms_rope_int8_fake(query, key, query_norm, key_norm, freqs, epsilon, rot_dim,
                           tensor_layout, norm_scope, split_half, rotate_qk, stabilize_k):
    if tensor_layout == "HND":
        batch, query_heads, query_tokens, _ = query.shape
        _, key_heads, key_tokens, _ = key.shape
    elif tensor_layout == "NHD":
        batch, query_tokens, query_heads, _ = query.shape
        _, key_tokens, key_heads, _ = key.shape
    else:
        raise ValueError(f"Unknown tensor layout: {tensor_layout}")
    query_scale = query.new_empty((batch, query_heads, ((query_tokens + 63) // 64) * 4),
                                  dtype=torch.float32)
    key_scale = key.new_empty((batch, key_heads, (key_tokens + 63) // 64), dtype=torch.float32)
    return (torch.empty_like(query, dtype=torch.int8), query_scale,
            torch.empty_like(key, dtype=torch.int8), key_scale)



@torch.library.custom_op("turing_utils::w8a8_attention", mutates_args=())
def w8a8_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                   tensor_layout: str, is_causal: bool, sm_scale: float, key_tile_tokens: int,
                   rotate_qk: bool, stabilize_k: bool) -> torch.Tensor:
    from .core import w8a8attn

    return w8a8attn(query, key, value, tensor_layout=tensor_layout, is_causal=is_causal,
                    sm_scale=sm_scale if sm_scale > 0.0 else None,
                    key_tile_tokens=key_tile_tokens, rotate_qk=rotate_qk,
                    stabilize_k=stabilize_k)


@w8a8_attention.register_fake
def _w8a8_attention_fake(query, key, value, tensor_layout, is_causal, sm_scale, key_tile_tokens,
                         rotate_qk, stabilize_k):
    return torch.empty_like(query)
