"""Fake-tensor and call contracts of the custom ops, ported from the
reference's tests/test_kernel_custom_ops.py:194-277 and
tests/test_turing_sage_quant.py:144-175."""
from __future__ import annotations

from unittest import mock

import torch

import comfyui_turing_utils_kernel as kernel
from comfyui_turing_utils_kernel.turing_sage import quant


def test_convrot_fake_contracts():
    x = torch.empty((3, 512), dtype=torch.bfloat16, device="meta")
    expectations = {
        "turing_swiglu_int8_convrot_quantize": (3, 256),
        "turing_swiglu_int4_convrot_quantize": (3, 128),
        "turing_gelu_int8_convrot_quantize": (3, 512),
        "turing_gelu_int4_convrot_quantize": (3, 256),
        "turing_bf16_gelu_int8_convrot_quantize": (3, 512),
        "turing_bf16_gelu_int4_convrot_quantize": (3, 256),
    }
    for name, shape in expectations.items():
        q, s = getattr(kernel, name)(x)
        assert q.shape == shape and q.dtype == torch.int8
        assert s.shape == (3, 1) and s.dtype == torch.float32 and s.device.type == "meta"
    for bits, shape in ((8, (3, 256)), (4, (3, 128))):
        q, s = getattr(kernel, f"turing_bf16_int{bits}_convrot_quantize")(x, swiglu=True)
        assert q.shape == shape and s.shape == (3, 1)


def test_linear_and_epilogue_fake_contracts():
    activation = torch.empty((7, 128), dtype=torch.int8, device="meta")
    weight = torch.empty((64, 64), dtype=torch.int8, device="meta")
    row_scale = torch.empty((7,), dtype=torch.float32, device="meta")
    column_scale = torch.empty((64,), dtype=torch.float32, device="meta")
    cb = kernel.turing_codebook_w4a8_linear(
        activation, weight, row_scale, torch.empty((64, 8), dtype=torch.uint8, device="meta"),
        column_scale, torch.empty((16,), dtype=torch.float32, device="meta"))
    assert cb.shape == (7, 64) and cb.dtype == torch.bfloat16
    long_cb = kernel.turing_codebook_w4a8_linear(
        torch.empty((9000, 128), dtype=torch.int8, device="meta"), weight,
        torch.empty((9000,), dtype=torch.float32, device="meta"),
        torch.empty((64, 8), dtype=torch.uint8, device="meta"), column_scale,
        torch.empty((16,), dtype=torch.float32, device="meta"), chunk_rows=-1)
    assert long_cb.shape == (9000, 64)
    lin = kernel.turing_int8_linear(activation,
                                    torch.empty((64, 128), dtype=torch.int8, device="meta"),
                                    row_scale, column_scale)
    assert lin.shape == (7, 64) and lin.dtype == torch.bfloat16
    acc = kernel.turing_int8_gemm_s32(activation,
                                      torch.empty((64, 128), dtype=torch.int8, device="meta"))
    assert acc.shape == (7, 64) and acc.dtype == torch.int32
    epi = kernel.turing_dequantize_int8_bf16(torch.empty((7, 80), dtype=torch.int32, device="meta"),
                                            row_scale, column_scale, 64)
    assert epi.shape == (7, 64) and epi.dtype == torch.bfloat16


def test_int8_linear_is_a_fullgraph_leaf():
    a = torch.empty((7, 128), dtype=torch.int8, device="meta")
    w = torch.empty((64, 128), dtype=torch.int8, device="meta")
    s1 = torch.empty((7,), device="meta")
    s2 = torch.empty((64,), device="meta")
    f = torch.compile(lambda *t: kernel.turing_int8_linear(*t), backend="eager", fullgraph=True)
    assert f(a, w, s1, s2).shape == (7, 64)


def test_split_quantizers_preserve_production_scale_contract():
    q = torch.empty((2, 4, 129, 128), dtype=torch.bfloat16)
    k = torch.empty((2, 2, 151, 128), dtype=torch.bfloat16)
    with (mock.patch.object(quant._fused, "quant_per_warp_int8_cuda") as quant_q,
          mock.patch.object(quant._fused, "quant_per_block_int8_cuda") as quant_k):
        q_int8, q_scale = quant.quantize_query_per_warp(q)
        k_int8, k_scale = quant.quantize_key_per_block(k)
    assert q_int8.shape == q.shape and k_int8.shape == k.shape
    assert q_scale.shape == (2, 4, 12) and k_scale.shape == (2, 2, 3)
    quant_q.assert_called_once_with(q, q_int8, q_scale, 64, 16, 1)
    quant_k.assert_called_once_with(k, k_int8, k_scale, 64, 1)


def test_production_per_warp_scale_shapes():
    q = torch.empty((2, 4, 65, 64), dtype=torch.float16)
    k = torch.empty((2, 2, 73, 64), dtype=torch.float16)
    with (mock.patch.object(quant._fused, "quant_per_warp_int8_cuda"),
          mock.patch.object(quant._fused, "quant_per_block_int8_cuda")):
        q_int8, q_scale, k_int8, k_scale = quant.per_warp_int8(q, k)
    assert q_scale.shape == (2, 4, 8) and k_scale.shape == (2, 2, 2)
