"""Sage INT8 attention facade (kernel/comfyui_turing_utils_kernel/turing_sage/
__init__.py:16-430): availability probes, the sageattn family, split
prequantize/execute, and the torch.compile-friendly custom-op wrapper."""
from __future__ import annotations

import importlib

import torch

from .quant import (per_warp_int8, per_warp_int8_hadamard, quantize_key_per_block,
                    quantize_query_per_warp, rms_rope_per_warp_int8)


def available() -> bool:
    try:
        importlib.import_module("comfyui_turing_utils_kernel._sage_qattn_sm75")
        importlib.import_module("comfyui_turing_utils_kernel._sage_fused_sm75")
        from .._lib import load

        load()
    except (ImportError, OSError):
        return False
    return True


def _not_built() -> bool:
    return False


def fused_qk_preprocessing_available() -> bool:
    """True when the fused RMSNorm + RoPE + INT8 Q/K prologue is present
    (turing_sage/__init__.py:97-107 of the reference)."""
    if not available():
        return False
    module = importlib.import_module("comfyui_turing_utils_kernel._sage_fused_sm75")
    return hasattr(module, "quant_qk_rms_rope_int8_cuda")


def w8a8_available() -> bool:
    """True when the dense W8A8-PV attention is present (turing_sage/__init__.py:52-62
    of the reference probes the extension for quantize_v_int8_sm75)."""
    if not available():
        return False
    module = importlib.import_module("comfyui_turing_utils_kernel._sage_qattn_sm75")
    return hasattr(module, "quantize_v_int8_sm75")


# The plugin probes these before choosing a backend (turing_sage/__init__.py:25-145 of the
# reference).  The sparse (Sol/SLA), varlen and VAE overlap kernels are not part of this
# package, so each of these probes answers False.
sparse_available = _not_built
sla_available = _not_built
w8a8_varlen_available = _not_built
split_prequantization_available = _not_built
overlap_blend_available = _not_built
overlap_accumulate_available = _not_built


def sageattn(*args, **kwargs):
    """Run the Sage INT8 attention (HND or NHD)."""
    from .core import sageattn as _impl

    return _impl(*args, **kwargs)


def sageattn_compiled(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, *,
                      tensor_layout: str = "HND", is_causal: bool = False,
                      sm_scale: float | None = None) -> torch.Tensor:
    """torch.compile leaf (turing_sage/__init__.py:166-184)."""
    from .custom_ops import sage_attention

    return sage_attention(query, key, value, tensor_layout, is_causal,
                          -1.0 if sm_scale is None else float(sm_scale))


def prequantize_sageattn(*args, **kwargs):
    from .core import prequantize_sageattn as _impl

    return _impl(*args, **kwargs)


def prequantize_rms_rope_qk(*args, **kwargs):
    from .core import prequantize_rms_rope_qk as _impl

    return _impl(*args, **kwargs)


def prequantize_sageattn_from_qk(*args, **kwargs):
    from .core import prequantize_sageattn_from_qk as _impl

    return _impl(*args, **kwargs)


def sageattn_from_prequantized(*args, **kwargs):
    from .core import sageattn_from_prequantized as _impl

    return _impl(*args, **kwargs)


def w8a8attn(*args, **kwargs):
    """Dense W8A8-PV attention (turing_sage/__init__.py:304-307)."""
    from .core import w8a8attn as _impl

    return _impl(*args, **kwargs)


def w8a8attn_compiled(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                      tensor_layout: str = "HND", is_causal: bool = False,
                      sm_scale: float | None = None, key_tile_tokens: int = 0,
                      rotate_qk: bool = True, stabilize_k: bool = True):
    """torch.compile leaf (turing_sage/__init__.py:310-334)."""
    from .custom_ops import w8a8_attention

    return w8a8_attention(q, k, v, tensor_layout, bool(is_causal),
                          float(sm_scale) if sm_scale is not None else -1.0,
                          int(key_tile_tokens), bool(rotate_qk), bool(stabilize_k))


def prequantize_sol_sageattn(*args, **kwargs):
    from .core import prequantize_sol_sageattn as _impl

    return _impl(*args, **kwargs)


def prequantize_sol_sageattn_from_qk(*args, **kwargs):
    from .core import prequantize_sol_sageattn_from_qk as _impl

    return _impl(*args, **kwargs)


def sol_sparse_sageattn_from_prequantized(*args, **kwargs):
    from .core import sol_sparse_sageattn_from_prequantized as _impl

    return _impl(*args, **kwargs)


from . import custom_ops  # noqa: E402,F401  (registers the turing_utils:: sage custom ops)

__all__ = ["available", "fused_qk_preprocessing_available", "overlap_accumulate_available",
           "overlap_blend_available", "per_warp_int8", "per_warp_int8_hadamard",
           "prequantize_rms_rope_qk", "prequantize_sageattn", "prequantize_sageattn_from_qk",
           "prequantize_sol_sageattn", "prequantize_sol_sageattn_from_qk",
           "quantize_key_per_block", "rms_rope_per_warp_int8", "quantize_query_per_warp",
           "sageattn", "sageattn_compiled", "sageattn_from_prequantized", "sla_available",
           "sol_sparse_sageattn_from_prequantized", "sparse_available",
           "split_prequantization_available", "w8a8_available", "w8a8_varlen_available",
           "w8a8attn", "w8a8attn_compiled"]
