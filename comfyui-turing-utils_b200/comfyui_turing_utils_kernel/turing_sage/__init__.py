"""Sage INT8 attention facade (kernel/comfyui_turing_utils_kernel/turing_sage/
__init__.py:16-430): availability probes, the sageattn family, split
prequantize/execute, and the torch.compile-friendly custom-op wrapper."""
from __future__ import annotations

import importlib

import torch

from .quant import (per_warp_int8, quantize_key_per_block, quantize_query_per_warp,
                    rms_rope_per_warp_int8)


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


# The plugin probes these before choosing a backend (turing_sage/__init__.py:25-145 of the
# reference).  The sparse (Sol/SLA), W8A8-PV, varlen and VAE overlap kernels are not part of
# this package, so each probe answers False and the plugin keeps the plain Sage INT8 backend.
sparse_available = _not_built
sla_available = _not_built
w8a8_available = _not_built
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


from . import custom_ops  # noqa: E402,F401  (registers the turing_utils:: sage custom ops)

__all__ = ["available", "fused_qk_preprocessing_available", "overlap_accumulate_available",
           "overlap_blend_available", "per_warp_int8", "prequantize_rms_rope_qk", "prequantize_sageattn",
           "prequantize_sageattn_from_qk", "quantize_key_per_block", "rms_rope_per_warp_int8",
           "quantize_query_per_warp", "sageattn", "sageattn_compiled",
           "sageattn_from_prequantized", "sla_available", "sparse_available",
           "split_prequantization_available", "w8a8_available", "w8a8_varlen_available"]
