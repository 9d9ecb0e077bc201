"""``turing_utils::*`` custom ops of the linear path.

Same op names, schemas, Python-side checks and fake (meta) implementations as
the reference (kernel/comfyui_turing_utils_kernel/ops.py:8-352), so
``torch.compile(fullgraph=True)`` treats them as leaves and the plugin's
dispatcher calls them unchanged.  The CUDA implementations run the sm_100a
kernels of libturing_b200.so through ``_C``.
"""
from __future__ import annotations

import torch

from . import _C


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise RuntimeError(f"{what} requires CUDA tensors")
    if torch.cuda.get_device_capability(t.device)[0] != 10:
        raise RuntimeError(f"{what} requires an sm_100 (B200) device for this build")


@torch.library.custom_op("turing_utils::w4a8_linear", mutates_args=())
def turing_w4a8_linear(
    activation: torch.Tensor,
    weight: torch.Tensor,
    activation_scale: torch.Tensor,
    weight_scale: torch.Tensor,
    bias: torch.Tensor | None = None,
) -> torch.Tensor:
    """Signed-nibble W4A8 linear (ops.py:8-26)."""
    _require_cuda(activation, "Turing W4A8")
    return _C.turing_w4a8_linear(
        activation.contiguous(), weight.contiguous(), activation_scale.contiguous(),
        weight_scale.contiguous(), None if bias is None else bias.contiguous())


@turing_w4a8_linear.register_fake
def _w4a8_fake(activation, weight, activation_scale, weight_scale, bias=None):
    return torch.empty((activation.size(0), weight.size(0)), dtype=torch.bfloat16,
                       device=activation.device)


@torch.library.custom_op("turing_utils::int4_linear", mutates_args=())
def turing_int4_linear(
    activation: torch.Tensor,
    weight: torch.Tensor,
    activation_scale: torch.Tensor,
    weight_scale: torch.Tensor,
    bias: torch.Tensor | None = None,
) -> torch.Tensor:
    """W4A4 linear on packed INT4 ConvRot activations (no counterpart in the
    reference package: the plugin calls comfy-kitchen's int4_linear there,
    comfyui_turing_utils/quantization/dispatch.py:791-804)."""
    _require_cuda(activation, "Turing W4A4")
    return _C.turing_int4_linear(
        activation.contiguous(), weight.contiguous(), activation_scale.contiguous(),
        weight_scale.contiguous(), None if bias is None else bias.contiguous())


@turing_int4_linear.register_fake
def _int4_fake(activation, weight, activation_scale, weight_scale, bias=None):
    return torch.empty((activation.size(0), weight.size(0)), dtype=torch.bfloat16,
                       device=activation.device)


@torch.library.custom_op("turing_utils::codebook_w4a8_linear", mutates_args=())
def turing_codebook_w4a8_linear(
    activation: torch.Tensor,
    weight: torch.Tensor,
    activation_scale: torch.Tensor,
    group_scale: torch.Tensor,
    channel_scale: torch.Tensor,
    codebook: torch.Tensor,
    bias: torch.Tensor | None = None,
    group_size: int = 16,
    chunk_rows: int = 0,
) -> torch.Tensor:
    """Grouped-codebook W4A8 (ops.py:38-74).  ``chunk_rows`` bounds the staged
    decode workspace (0 = production policy)."""
    _require_cuda(activation, "Turing codebook W4A8")
    if group_scale.dtype == torch.float8_e4m3fn:
        group_scale = group_scale.view(torch.uint8)
    if group_scale.dtype != torch.uint8:
        raise TypeError("group_scale must be float8_e4m3fn or its raw uint8 view")
    return _C.turing_codebook_w4a8_linear(
        activation.contiguous(), weight.contiguous(), activation_scale.contiguous(),
        group_scale.contiguous(), channel_scale.contiguous(), codebook.contiguous(),
        None if bias is None else bias.contiguous(), group_size, chunk_rows)


@turing_codebook_w4a8_linear.register_fake
def _codebook_fake(activation, weight, activation_scale, group_scale, channel_scale, codebook,
                   bias=None, group_size=16, chunk_rows=0):
    return torch.empty((activation.size(0), weight.size(0)), dtype=torch.bfloat16,
                       device=activation.device)


@torch.library.custom_op("turing_utils::int8_linear", mutates_args=())
def turing_int8_linear(
    activation: torch.Tensor,
    weight: torch.Tensor,
    activation_scale: torch.Tensor,
    weight_scale: torch.Tensor,
    bias: torch.Tensor | None = None,
) -> torch.Tensor:
    """W8A8 contraction with the fused dequant/bias/bf16 epilogue (ops.py:96-126)."""
    _require_cuda(activation, "Turing INT8 linear")
    return _C.turing_int8_linear(activation.contiguous(), weight.contiguous(),
                                 activation_scale.contiguous(), weight_scale.contiguous(),
                                 None if bias is None else bias.contiguous())


@turing_int8_linear.register_fake
def _int8_linear_fake(activation, weight, activation_scale, weight_scale, bias=None):
    return torch.empty((activation.size(0), weight.size(0)), dtype=torch.bfloat16,
                       device=activation.device)


@torch.library.custom_op("turing_utils::int8_gemm_s32", mutates_args=())
def turing_int8_gemm_s32(activation: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Exact INT32 accumulators (feeds turing_dequantize_int8_bf16)."""
    _require_cuda(activation, "Turing INT8 GEMM")
    return _C.turing_int8_gemm_s32(activation.contiguous(), weight.contiguous())


@turing_int8_gemm_s32.register_fake
def _int8_gemm_s32_fake(activation, weight):
    return torch.empty((activation.size(0), weight.size(0)), dtype=torch.int32,
                       device=activation.device)


@torch.library.custom_op("turing_utils::dequantize_int8_bf16", mutates_args=())
def turing_dequantize_int8_bf16(
    accumulator: torch.Tensor,
    activation_scale: torch.Tensor,
    weight_scale: torch.Tensor,
    output_columns: int = -1,
) -> torch.Tensor:
    """Dequantize an INT32 GEMM workspace directly into packed BF16 stores."""
    _require_cuda(accumulator, "Turing BF16 epilogue")
    if accumulator.dtype != torch.int32 or accumulator.ndim != 2:
        raise TypeError("accumulator must be a 2D int32 tensor")
    return _C.turing_dequantize_int8_bf16(accumulator.contiguous(), activation_scale.contiguous(),
                                          weight_scale.contiguous(), output_columns)


@turing_dequantize_int8_bf16.register_fake
def _dequant_fake(accumulator, activation_scale, weight_scale, output_columns=-1):
    columns = accumulator.size(1) if output_columns < 0 else output_columns
    return torch.empty((accumulator.size(0), columns), dtype=torch.bfloat16,
                       device=accumulator.device)


def _staged_op(name, doc, width_div, int4):
    @torch.library.custom_op(f"turing_utils::{name}", mutates_args=())
    def op(x: torch.Tensor, group_size: int = 256) -> tuple[torch.Tensor, torch.Tensor]:
        _require_cuda(x, doc)
        if x.dtype not in (torch.float16, torch.bfloat16):
            raise TypeError(f"{doc} input must be float16 or bfloat16")
        if x.ndim != 2:
            raise ValueError(f"{doc} input must be 2D")
        return getattr(_C, f"turing_{name}")(x.contiguous(), group_size)

    @op.register_fake
    def _fake(x, group_size=256):
        hidden = x.size(1) // width_div
        return (torch.empty((x.size(0), hidden // 2 if int4 else hidden), dtype=torch.int8,
                            device=x.device),
                torch.empty((x.size(0), 1), dtype=torch.float32, device=x.device))

    return op


turing_swiglu_int8_convrot_quantize = _staged_op(
    "swiglu_int8_convrot_quantize", "Turing SwiGLU ConvRot", 2, False)
turing_swiglu_int4_convrot_quantize = _staged_op(
    "swiglu_int4_convrot_quantize", "Turing SwiGLU INT4 ConvRot", 2, True)
turing_gelu_int8_convrot_quantize = _staged_op(
    "gelu_int8_convrot_quantize", "Turing GELU ConvRot", 1, False)
turing_gelu_int4_convrot_quantize = _staged_op(
    "gelu_int4_convrot_quantize", "Turing GELU INT4 ConvRot", 1, True)


@torch.library.custom_op("turing_utils::bf16_int8_convrot_quantize", mutates_args=())
def turing_bf16_int8_convrot_quantize(
    x: torch.Tensor,
    group_size: int = 256,
    *,
    swiglu: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Whole-row BF16 ConvRot INT8 quantization (ops.py:257-273)."""
    _require_cuda(x, "BF16 row-buffer ConvRot")
    if x.dtype != torch.bfloat16:
        raise TypeError("BF16 row-buffer ConvRot input must be bfloat16")
    if x.ndim != 2:
        raise ValueError("BF16 row-buffer ConvRot input must be 2D")
    return _C.turing_bf16_int8_convrot_quantize(x.contiguous(), group_size, swiglu)


@turing_bf16_int8_convrot_quantize.register_fake
def _bf16_int8_fake(x, group_size=256, *, swiglu=False):
    hidden = x.size(1) // 2 if swiglu else x.size(1)
    return (torch.empty((x.size(0), hidden), dtype=torch.int8, device=x.device),
            torch.empty((x.size(0), 1), dtype=torch.float32, device=x.device))


@torch.library.custom_op("turing_utils::bf16_int4_convrot_quantize", mutates_args=())
def turing_bf16_int4_convrot_quantize(
    x: torch.Tensor,
    group_size: int = 256,
    *,
    swiglu: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Whole-row BF16 ConvRot INT4 quantization (ops.py:285-301)."""
    _require_cuda(x, "BF16 row-buffer INT4 ConvRot")
    if x.dtype != torch.bfloat16:
        raise TypeError("BF16 row-buffer INT4 ConvRot input must be bfloat16")
    if x.ndim != 2:
        raise ValueError("BF16 row-buffer INT4 ConvRot input must be 2D")
    return _C.turing_bf16_int4_convrot_quantize(x.contiguous(), group_size, swiglu)


@turing_bf16_int4_convrot_quantize.register_fake
def _bf16_int4_fake(x, group_size=256, *, swiglu=False):
    hidden = x.size(1) // 2 if swiglu else x.size(1)
    return (torch.empty((x.size(0), hidden // 2), dtype=torch.int8, device=x.device),
            torch.empty((x.size(0), 1), dtype=torch.float32, device=x.device))


@torch.library.custom_op("turing_utils::bf16_gelu_int8_convrot_quantize", mutates_args=())
def turing_bf16_gelu_int8_convrot_quantize(
    x: torch.Tensor,
    group_size: int = 256,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Whole-row BF16 tanh-GELU + ConvRot INT8 quantization."""
    _require_cuda(x, "BF16 GELU ConvRot")
    if x.dtype != torch.bfloat16 or x.ndim != 2:
        raise TypeError("BF16 GELU ConvRot input must be a 2D bfloat16 tensor")
    return _C.turing_bf16_gelu_int8_convrot_quantize(x.contiguous(), group_size)


@turing_bf16_gelu_int8_convrot_quantize.register_fake
def _bf16_gelu_int8_fake(x, group_size=256):
    return (torch.empty(x.shape, dtype=torch.int8, device=x.device),
            torch.empty((x.size(0), 1), dtype=torch.float32, device=x.device))


@torch.library.custom_op("turing_utils::bf16_gelu_int4_convrot_quantize", mutates_args=())
def turing_bf16_gelu_int4_convrot_quantize(
    x: torch.Tensor,
    group_size: int = 256,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Whole-row BF16 tanh-GELU + ConvRot INT4 quantization."""
    _require_cuda(x, "BF16 GELU INT4 ConvRot")
    if x.dtype != torch.bfloat16 or x.ndim != 2:
        raise TypeError("BF16 GELU INT4 ConvRot input must be a 2D bfloat16 tensor")
    return _C.turing_bf16_gelu_int4_convrot_quantize(x.contiguous(), group_size)


@turing_bf16_gelu_int4_convrot_quantize.register_fake
def _bf16_gelu_int4_fake(x, group_size=256):
    return (torch.empty((x.size(0), x.size(1) // 2), dtype=torch.int8, device=x.device),
            torch.empty((x.size(0), 1), dtype=torch.float32, device=x.device))


@torch.library.custom_op("turing_utils::segmented_rms_adaln", mutates_args=())
def turing_segmented_rms_adaln(
    x: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
    shift: torch.Tensor,
    segments: torch.Tensor,
    epsilon: float = 1.0e-5,
) -> torch.Tensor:
    """Fused affine RMSNorm and segmented AdaLN modulation (ops.py:355-396)."""
    if x.device.type != "cuda":
        raise RuntimeError("Segmented RMSNorm+AdaLN requires CUDA tensors")
    _require_cuda(x, "Segmented RMSNorm+AdaLN")
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError("segmented RMSNorm+AdaLN input must be float16, bfloat16, or float32")
    if x.ndim != 2:
        raise ValueError("segmented RMSNorm+AdaLN input must be 2D [M, K]")
    if weight.device != x.device or scale.device != x.device or shift.device != x.device:
        raise ValueError("weight, scale, and shift must be on the input device")
    weight = weight.to(dtype=x.dtype).contiguous()
    scale = scale.to(dtype=x.dtype)
    shift = shift.to(dtype=x.dtype)
    if scale.stride(-1) != 1:
        scale = scale.contiguous()
    if shift.stride(-1) != 1:
        shift = shift.contiguous()
    if segments.device != x.device or segments.dtype != torch.int32:
        raise ValueError("segments must be an int32 tensor on the input device")
    return _C.turing_segmented_rms_adaln(x.contiguous(), weight, scale, shift,
                                         segments.contiguous(), epsilon)


@turing_segmented_rms_adaln.register_fake
def _segmented_rms_adaln_fake(x, weight, scale, shift, segments, epsilon=1.0e-5):
    return torch.empty_like(x)


@torch.library.custom_op("turing_utils::layer_norm_adaln", mutates_args=())
def turing_layer_norm_adaln(
    x: torch.Tensor,
    scale: torch.Tensor,
    shift: torch.Tensor,
    epsilon: float = 1.0e-5,
) -> torch.Tensor:
    """Fused FP32-statistics LayerNorm and Wan AdaLN modulation (ops.py:399-418)."""
    if x.device.type != "cuda":
        raise RuntimeError("LayerNorm+AdaLN requires a CUDA tensor")
    _require_cuda(x, "LayerNorm+AdaLN")
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32) or x.ndim != 3:
        raise TypeError("LayerNorm+AdaLN input must be 3D float16, bfloat16, or float32")
    scale = scale.to(device=x.device, dtype=x.dtype).contiguous()
    shift = shift.to(device=x.device, dtype=x.dtype).contiguous()
    return _C.turing_layer_norm_adaln(x.contiguous(), scale, shift, epsilon)


@turing_layer_norm_adaln.register_fake
def _layer_norm_adaln_fake(x, scale, shift, epsilon=1.0e-5):
    return torch.empty_like(x)
