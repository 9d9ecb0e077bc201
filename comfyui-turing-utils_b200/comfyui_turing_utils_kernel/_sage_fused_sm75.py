"""Drop-in for the reference's ``_sage_fused_sm75`` extension (quantizer part).

Same entry-point names and argument order as
kernel/csrc/turing/sage/pybind_fused.cpp:23-33 (fused.h); the work runs in the
sm_100a quantizer kernels of libturing_b200.so.  Outputs are caller-allocated
and written in place, as in the reference.
"""
from __future__ import annotations

import torch

from ._lib import TB_LAYOUT_HND, TB_LAYOUT_NHD, call, dtype_code, ptr, stream_of


def _check(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _geometry(input: torch.Tensor, tensor_layout: int):
    _check(input.is_cuda, "input must be a CUDA tensor")
    _check(input.dim() == 4, "input must be a 4D tensor")
    _check(input.stride(-1) == 1, "input last dim must be contiguous")
    B, D = input.size(0), input.size(3)
    if tensor_layout == TB_LAYOUT_NHD:
        L, H = input.size(1), input.size(2)
        sb, sl, sh = input.stride(0), input.stride(1), input.stride(2)
    elif tensor_layout == TB_LAYOUT_HND:
        H, L = input.size(1), input.size(2)
        sb, sh, sl = input.stride(0), input.stride(1), input.stride(2)
    else:
        raise RuntimeError("tensor_layout must be 0 or 1")
    return B, H, L, D, sb, sh, sl


def _check_outputs(input, output, scale, B, H, expected_tiles):
    _check(output.is_cuda and scale.is_cuda, "output and scale must be CUDA tensors")
    _check(output.dtype == torch.int8, "output must be int8")
    _check(scale.dtype == torch.float32, "scale must be float32")
    _check(output.is_contiguous() and scale.is_contiguous(),
           "output and scale must be contiguous")
    _check(tuple(output.shape) == tuple(input.shape), "output shape must match input")
    _check(tuple(scale.shape) == (B, H, expected_tiles), "scale shape mismatch")


def quant_per_block_int8_cuda(input, output, scale, *args):
    """quant_per_block_int8_cuda(input, output, scale, block_size, tensor_layout)
    (fused.cu:983-1067).  The 6-argument sm_scale overload of the reference is
    not used by the production path and is rejected."""
    if len(args) != 2:
        raise RuntimeError("quant_per_block_int8_cuda(input, output, scale, block_size, tensor_layout)")
    block_size, tensor_layout = int(args[0]), int(args[1])
    B, H, L, D, sb, sh, sl = _geometry(input, tensor_layout)
    _check_outputs(input, output, scale, B, H, (L + block_size - 1) // block_size)
    with torch.cuda.device(input.device):
        call("tb_quant_per_block_int8", ptr(input), dtype_code(input), ptr(output), ptr(scale),
             B, H, L, D, sb, sh, sl, block_size, tensor_layout, None, stream_of(input))


def quant_per_block_int8_smooth_cuda(input, output, scale, mean, block_size, tensor_layout):
    """Per-block INT8 with K mean-smoothing: the sub_mean form of the reference's
    QuantInt8Kernel (fused.cu:97-128).  mean: [B, H, D] of the input dtype."""
    B, H, L, D, sb, sh, sl = _geometry(input, int(tensor_layout))
    _check_outputs(input, output, scale, B, H, (L + block_size - 1) // block_size)
    _check(mean.is_cuda and mean.dtype == input.dtype and mean.is_contiguous()
           and tuple(mean.shape) == (B, H, D), "mean must be a contiguous [B, H, D] tensor")
    with torch.cuda.device(input.device):
        call("tb_quant_per_block_int8", ptr(input), dtype_code(input), ptr(output), ptr(scale),
             B, H, L, D, sb, sh, sl, int(block_size), int(tensor_layout), ptr(mean),
             stream_of(input))


def quant_per_warp_int8_cuda(input, output, scale, block_size, warp_block_size, tensor_layout):
    """fused.cu:1070-1150."""
    B, H, L, D, sb, sh, sl = _geometry(input, int(tensor_layout))
    tiles = (L + block_size - 1) // block_size * (block_size // warp_block_size)
    _check_outputs(input, output, scale, B, H, tiles)
    with torch.cuda.device(input.device):
        call("tb_quant_per_warp_int8", ptr(input), dtype_code(input), ptr(output), ptr(scale),
             B, H, L, D, sb, sh, sl, int(block_size), int(warp_block_size), int(tensor_layout),
             stream_of(input))


def quant_qk_per_warp_int8_cuda(query, key, query_output, key_output, query_scale, key_scale,
                                query_block_size, query_warp_block_size, key_block_size,
                                tensor_layout):
    """Q per warp + K per block in one call (fused.h:43-53); two launches here."""
    quant_per_warp_int8_cuda(query, query_output, query_scale, query_block_size,
                             query_warp_block_size, tensor_layout)
    quant_per_block_int8_cuda(key, key_output, key_scale, key_block_size, tensor_layout)


def token_mean_cuda(input, mean, tensor_layout):
    """Per-(batch, head, channel) token mean in the input dtype (fp64 sum)."""
    B, H, L, D, sb, sh, sl = _geometry(input, int(tensor_layout))
    _check(mean.is_cuda and mean.dtype == input.dtype and mean.is_contiguous()
           and tuple(mean.shape) == (B, H, D), "mean must be a contiguous [B, H, D] tensor")
    with torch.cuda.device(input.device):
        call("tb_token_mean", ptr(input), dtype_code(input), ptr(mean), B, H, L, D, sb, sh, sl,
             int(tensor_layout), stream_of(input))
