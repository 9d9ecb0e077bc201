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


def split_prequantization_available() -> bool:
    """True when the split prequantize / execute path is present
    (turing_sage/__init__.py:82-95 of the reference): the plugin then installs
    its dense container function (attention/patches.py:494-497), which calls
    prequantize_sageattn / prequantize_sol_sageattn(use_w8a8, force_dense) and
    the *_from_prequantized executors, all built here.  The Sol summary entry
    the reference's probe also looks for serves only the sparse routes, whose
    own probes answer False."""
    if not w8a8_available():
        return False
    module = importlib.import_module("comfyui_turing_utils_kernel._sage_qattn_sm75")
    return hasattr(module, "sol_sparse_online_w8a8_prequantized_attn")


# The plugin probes these before choosing a backend (turing_sage/__init__.py:25-145 of the
# reference).  The sparse (Sol/SLA), varlen and VAE overlap kernels are not part of this
# package, so each of these probes answers False.
sparse_available = _not_built
sla_available = _not_built
w8a8_varlen_available = _not_built
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


def _structured_qkv(heads, lengths, head_dim, dtype, divisor, device):
    """Deterministic self-test inputs (turing_sage/__init__.py:620-627 form)."""
    q_values = torch.arange(heads[0] * lengths[0] * head_dim, device=device, dtype=torch.float32)
    kv_values = torch.arange(heads[1] * lengths[1] * head_dim, device=device, dtype=torch.float32)
    q = (((q_values % 29) - 14) / divisor).reshape(1, heads[0], lengths[0], head_dim).to(dtype)
    k = ((((kv_values * 3) % 31) - 15) / divisor).reshape(1, heads[1], lengths[1],
                                                           head_dim).to(dtype)
    v = ((((kv_values * 5) % 37) - 18) / divisor).reshape_as(k).to(dtype)
    return q, k, v


def _sm100_device(device: torch.device, what: str) -> None:
    if device.type != "cuda" or not torch.cuda.is_available():
        raise RuntimeError(f"{what} requires CUDA, got {device}")
    if torch.cuda.get_device_capability(device) != (10, 0):
        raise RuntimeError(f"{what} requires sm100 (B200), got {device}")


def preflight(device: torch.device) -> None:
    """Self-test the Sage kernels on `device` before the plugin routes
    attention to them (turing_sage/__init__.py:612-663, called by the plugin's
    preflight_bundled, attention/stable.py:521-528): fp16 / bf16 at head dims
    64, 96 and 128 against fp32 SDPA.  The varlen half of the reference's test
    is absent with the varlen kernel."""
    _sm100_device(device, "Turing Sage")
    if not available():
        raise RuntimeError("the bundled Turing Sage extensions are not built")
    with torch.inference_mode(), torch.cuda.device(device):
        for dtype in (torch.float16, torch.bfloat16):
            for head_dim in (64, 96, 128):
                q, k, v = _structured_qkv((4, 2), (65, 73), head_dim, dtype, 32, device)
                output = sageattn(q, k, v, tensor_layout="HND", smooth_k=False)
                reference = torch.nn.functional.scaled_dot_product_attention(
                    q.float(), k.float(), v.float(), enable_gqa=True)
                if (output.dtype != dtype or output.shape != q.shape
                        or not torch.isfinite(output).all()
                        or not torch.allclose(output.float(), reference, rtol=0.08, atol=0.05)):
                    raise RuntimeError(f"Turing Sage {dtype} D={head_dim} self-test failed")
        torch.cuda.synchronize(device)


def preflight_w8a8(device: torch.device) -> None:
    """Self-test of the dense W8A8-PV attention (turing_sage/__init__.py:573-610,
    called by preflight_bundled_w8a8, attention/stable.py:551-558)."""
    _sm100_device(device, "W8A8 attention")
    if not w8a8_available():
        raise RuntimeError("the W8A8 attention extension is not built")
    with torch.inference_mode(), torch.cuda.device(device):
        for head_dim in (64, 128):
            q, k, v = _structured_qkv((4, 2), (129, 151), head_dim, torch.bfloat16, 16, device)
            output = w8a8attn(q, k, v)
            reference = torch.nn.functional.scaled_dot_product_attention(
                q.float(), k.float(), v.float(), enable_gqa=True)
            if (output.dtype != torch.bfloat16 or output.shape != q.shape
                    or not torch.isfinite(output).all()
                    or not torch.allclose(output.float(), reference, rtol=0.12, atol=0.09)):
                raise RuntimeError(f"Turing W8A8 attention BF16 D={head_dim} self-test failed")
        torch.cuda.synchronize(device)


def preflight_sparse(device: torch.device) -> None:
    """The Sol sparse kernels are not part of this package
    (turing_sage/__init__.py:432-468 raises the same way when unbuilt)."""
    raise RuntimeError("the Sol sparse attention extension is not built")


def preflight_sla(device: torch.device) -> None:
    """The SLA sparse kernels are not part of this package (:471-510)."""
    raise RuntimeError("the SLA sparse attention extension is not built")


def _unbuilt(name: str, what: str):
    def entry(*args, **kwargs):
        raise RuntimeError(f"the {what} extension is not built")

    entry.__name__ = name
    entry.__doc__ = (f"{name} of the reference's turing_sage: the {what} kernels are not part "
                     "of this package (their availability probe answers False).")
    return entry


# Entry points of the reference's sparse (Sol / SLA), varlen and VAE-overlap
# backends (turing_sage/__init__.py:122-369): named here so callers that reach
# them past a False probe get the reference's "not built" error.
sol_sparse_sageattn = _unbuilt("sol_sparse_sageattn", "Sol sparse attention")
sol_sparse_sageattn_compiled = _unbuilt("sol_sparse_sageattn_compiled", "Sol sparse attention")
sla_sparse_sageattn = _unbuilt("sla_sparse_sageattn", "SLA sparse attention")
sla_sparse_sageattn_compiled = _unbuilt("sla_sparse_sageattn_compiled", "SLA sparse attention")
sla_sparse_sageattn_from_prequantized = _unbuilt("sla_sparse_sageattn_from_prequantized",
                                                 "SLA sparse attention")
prequantize_sla_sageattn = _unbuilt("prequantize_sla_sageattn", "SLA sparse attention")
prequantize_sla_sageattn_from_qk = _unbuilt("prequantize_sla_sageattn_from_qk",
                                            "SLA sparse attention")
sageattn_varlen = _unbuilt("sageattn_varlen", "Turing Sage varlen")
sageattn_varlen_compiled = _unbuilt("sageattn_varlen_compiled", "Turing Sage varlen")
w8a8attn_varlen = _unbuilt("w8a8attn_varlen", "W8A8 varlen attention")
w8a8attn_varlen_compiled = _unbuilt("w8a8attn_varlen_compiled", "W8A8 varlen attention")
overlap_blend_compiled = _unbuilt("overlap_blend_compiled", "VAE overlap blend")
overlap_accumulate_compiled = _unbuilt("overlap_accumulate_compiled", "VAE overlap accumulate")
run_attention_correctness_gate = _unbuilt("run_attention_correctness_gate", "Sol sparse attention")


from . import custom_ops  # noqa: E402,F401  (registers the turing_utils:: sage custom ops)

__all__ = ["available", "fused_qk_preprocessing_available", "overlap_accumulate_available",
           "overlap_blend_available", "per_warp_int8", "per_warp_int8_hadamard", "preflight",
           "preflight_sla", "preflight_sparse", "preflight_w8a8",
           "prequantize_rms_rope_qk", "prequantize_sageattn", "prequantize_sageattn_from_qk",
           "prequantize_sol_sageattn", "prequantize_sol_sageattn_from_qk",
           "quantize_key_per_block", "rms_rope_per_warp_int8", "quantize_query_per_warp",
           "sageattn", "sageattn_compiled", "sageattn_from_prequantized", "sla_available",
           "sol_sparse_sageattn_from_prequantized", "sparse_available",
           "split_prequantization_available", "w8a8_available", "w8a8_varlen_available",
           "w8a8attn", "w8a8attn_compiled"]
