"""Sage INT8 attention facade (kernel/comfyui_turing_utils_kernel/turing_sage/
__init__.py): quantizers and, once the attention kernel is loaded, the
sageattn family."""
from __future__ import annotations

import importlib

import torch

from .quant import per_warp_int8, quantize_key_per_block, quantize_query_per_warp


def available() -> bool:
    try:
        importlib.import_module("comfyui_turing_utils_kernel._sage_fused_sm75")
        from .._lib import load

        load()
    except (ImportError, OSError):
        return False
    return True


__all__ = ["available", "per_warp_int8", "quantize_key_per_block", "quantize_query_per_warp"]
