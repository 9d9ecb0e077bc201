"""Fake-tensor and call contracts of the custom ops, ported from the
reference's tests/test_kernel_custom_ops.py:194-277 and
tests/test_turing_sage_quant.py:144-175."""
from __future__ import annotations

from unittest import mock

import pytest
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


def test_fused_qk_preprocessor_has_fake_tensor_contract():
    """turing_utils::qk_rms_rope_int8 on meta tensors (reference
    tests/test_turing_sage_quant.py:22-50): production Q per-warp and K
    per-block scale shapes."""
    from comfyui_turing_utils_kernel.turing_sage.custom_ops import qk_rms_rope_int8

    q = torch.empty((2, 4, 129, 128), dtype=torch.bfloat16, device="meta")
    k = torch.empty((2, 2, 129, 128), dtype=torch.bfloat16, device="meta")
    qn = torch.empty((128,), dtype=torch.bfloat16, device="meta")
    kn = torch.empty((128,), dtype=torch.bfloat16, device="meta")
    f = torch.empty((1, 129, 1, 64, 2, 2), dtype=torch.bfloat16, device="meta")
    q8, qs, k8, ks = qk_rms_rope_int8(q, k, qn, kn, f, 1e-6, 128, "HND", "head", True, True, True)
    assert q8.shape == q.shape and q8.dtype == torch.int8
    assert qs.shape == (2, 4, 12) and qs.dtype == torch.float32
    assert k8.shape == k.shape and k8.dtype == torch.int8
    assert ks.shape == (2, 2, 3) and ks.dtype == torch.float32
    nq = torch.empty((2, 129, 4, 128), dtype=torch.bfloat16, device="meta")
    nk = torch.empty((2, 70, 2, 128), dtype=torch.bfloat16, device="meta")
    _, nqs, _, nks = qk_rms_rope_int8(nq, nk, qn, kn, f, 1e-6, 0, "NHD", "row", False, False, False)
    assert nqs.shape == (2, 4, 12) and nks.shape == (2, 2, 2)


def test_fused_qk_preprocessor_is_a_fullgraph_leaf():
    from comfyui_turing_utils_kernel.turing_sage.custom_ops import qk_rms_rope_int8

    q = torch.empty((1, 4, 129, 64), dtype=torch.float16, device="meta")
    k = torch.empty((1, 2, 129, 64), dtype=torch.float16, device="meta")
    w = torch.empty((64,), dtype=torch.float16, device="meta")
    f = torch.empty((0,), dtype=torch.float16, device="meta")
    compiled = torch.compile(
        lambda a, b, c, d, e: qk_rms_rope_int8(a, b, c, d, e, 1e-6, 0, "HND", "head", False,
                                               False, False),
        backend="eager", fullgraph=True)
    q8, qs, k8, ks = compiled(q, k, w, w, f)
    assert q8.shape == q.shape and qs.shape == (1, 4, 12) and ks.shape == (1, 2, 3)


def test_fused_qk_wrapper_passes_the_production_contract():
    """The wrapper calls the native entry with the 64/16/64 tile contract,
    the layout id and the norm scope id (2 when the caller gives the RRMS)."""
    q = torch.empty((2, 129, 4, 128), dtype=torch.bfloat16)
    k = torch.empty((2, 129, 2, 128), dtype=torch.bfloat16)
    w = torch.empty((4 * 128,), dtype=torch.bfloat16)
    kw = torch.empty((2 * 128,), dtype=torch.bfloat16)
    with mock.patch.object(quant._fused, "quant_qk_rms_rope_int8_cuda") as native:
        q8, qs, k8, ks = quant.rms_rope_per_warp_int8(
            q, k, w, kw, None, epsilon=1e-6, rot_dim=0, tensor_layout="NHD", norm_scope="row",
            split_half=True, rotate_qk=False, stabilize_k=False)
    args = native.call_args.args
    assert args[0] is q and args[2] is q8 and args[4] is qs and args[5] is ks
    assert args[9].shape == (2, 129) and args[10].shape == (2, 129)   # row RRMS scratch
    assert args[13:] == (1e-6, 0, 64, 16, 64, 0, 1, True, False)
    rq, rk = torch.ones((2, 129)), torch.ones((2, 129))
    with mock.patch.object(quant._fused, "quant_qk_rms_rope_int8_cuda") as native:
        quant.rms_rope_per_warp_int8(q, k, w, kw, None, epsilon=1e-6, rot_dim=0,
                                     tensor_layout="NHD", norm_scope="row", split_half=False,
                                     rotate_qk=False, stabilize_k=False, query_rrms=rq,
                                     key_rrms=rk)
    assert native.call_args.args[19] == 2 and native.call_args.args[9] is rq


def test_preflight_contract_without_gpu():
    """preflight / preflight_w8a8 refuse a non-CUDA device with the reference's
    message form; the unbuilt sparse backends report themselves
    (turing_sage/__init__.py:432-663)."""
    from comfyui_turing_utils_kernel import turing_sage

    for fn, what in ((turing_sage.preflight, "Turing Sage"),
                     (turing_sage.preflight_w8a8, "W8A8 attention")):
        with pytest.raises(RuntimeError, match=f"{what} requires CUDA"):
            fn(torch.device("cpu"))
    for fn in (turing_sage.preflight_sparse, turing_sage.preflight_sla):
        with pytest.raises(RuntimeError, match="not built"):
            fn(torch.device("cpu"))
    assert {"preflight", "preflight_w8a8", "w8a8attn", "w8a8attn_compiled",
            "prequantize_sol_sageattn"} <= set(turing_sage.__all__)


def test_w8a8_attention_op_fake():
    """turing_utils::w8a8_attention has the reference's schema and fake
    (custom_ops.py:170-210)."""
    from comfyui_turing_utils_kernel.turing_sage.custom_ops import w8a8_attention

    q = torch.empty((1, 2, 50, 128), dtype=torch.bfloat16, device="meta")
    out = w8a8_attention(q, q, q, "HND", False, -1.0, 0, True, True)
    assert out.shape == q.shape and out.dtype == q.dtype and out.device.type == "meta"


def test_backend_probes():
    """The probes the plugin reads (turing_sage/__init__.py:16-107 of the
    reference): dense Sage, W8A8, split prequantization and the fused Q/K
    prologue are built; the sparse and varlen backends are not."""
    from comfyui_turing_utils_kernel import turing_sage

    assert turing_sage.available() and turing_sage.w8a8_available()
    assert turing_sage.split_prequantization_available()
    assert turing_sage.fused_qk_preprocessing_available()
    for probe in (turing_sage.sparse_available, turing_sage.sla_available,
                  turing_sage.w8a8_varlen_available, turing_sage.overlap_blend_available,
                  turing_sage.overlap_accumulate_available):
        assert probe() is False


def test_unbuilt_backends_raise():
    """Entry points of the sparse / varlen / overlap backends exist and raise the
    reference's "not built" error."""
    from comfyui_turing_utils_kernel import turing_sage

    for name in ("sol_sparse_sageattn", "sla_sparse_sageattn", "sageattn_varlen",
                 "w8a8attn_varlen", "overlap_blend_compiled", "prequantize_sla_sageattn"):
        with pytest.raises(RuntimeError, match="not built"):
            getattr(turing_sage, name)(None, None, None)


def test_rotated_fused_qk_wrapper_contract():
    """rotate_qk with stabilize_k hands the native entry the reference's K
    anchor scratch (int32 [B, Hk], fp32 [B, Hk, D]) and rotate=True
    (turing_sage/quant.py:59-92); without stabilize_k the scratch is empty."""
    q = torch.empty((1, 3, 70, 64), dtype=torch.float16)
    k = torch.empty((1, 1, 90, 64), dtype=torch.float16)
    w = torch.empty((64,), dtype=torch.float16)
    with mock.patch.object(quant._fused, "quant_qk_rms_rope_int8_cuda") as native:
        quant.rms_rope_per_warp_int8(q, k, w, w, None, epsilon=1e-6, rot_dim=0,
                                     tensor_layout="HND", norm_scope="head", split_half=False,
                                     rotate_qk=True, stabilize_k=True)
    args = native.call_args.args
    assert args[11].dtype == torch.int32 and args[11].shape == (1, 1)
    assert args[12].dtype == torch.float32 and args[12].shape == (1, 1, 64)
    assert args[21] is True
    with mock.patch.object(quant._fused, "quant_qk_rms_rope_int8_cuda") as native:
        quant.rms_rope_per_warp_int8(q, k, w, w, None, epsilon=1e-6, rot_dim=0,
                                     tensor_layout="HND", norm_scope="head", split_half=False,
                                     rotate_qk=True, stabilize_k=False)
    assert native.call_args.args[11].numel() == 0 and native.call_args.args[12].numel() == 0


def test_w8a8_facade_rejections():
    """w8a8attn / prequantize_sol_sageattn / the prequantized entry raise the
    reference's errors before any device work (core.py:656-914,
    sol_sparse_cuda_sm75.cu:2824-2833)."""
    from comfyui_turing_utils_kernel import _sage_qattn_sm75 as qattn
    from comfyui_turing_utils_kernel.turing_sage import core

    q = torch.zeros((1, 2, 64, 128), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="Unsupported tensor_layout"):
        core.w8a8attn.__wrapped__(q, q, q, tensor_layout="BHLD")
    with pytest.raises(TypeError, match="float16 or bfloat16"):
        core.w8a8attn.__wrapped__(q.float(), q.float(), q.float())
    wide = torch.zeros((1, 2, 64, 160), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match=r"head_dim in \[1, 128\]"):
        core.w8a8attn.__wrapped__(wide, wide, wide)
    with pytest.raises(ValueError, match="must be on CUDA"):
        core.w8a8attn.__wrapped__(q, q, q)
    with pytest.raises(ValueError, match="must be on CUDA"):   # checked before the layout
        core.prequantize_sol_sageattn.__wrapped__(q, q, q, tensor_layout="NHD")
    qk = core.PrequantizedQK(q.to(torch.int8), torch.zeros((1, 2, 4)), q.to(torch.int8),
                             torch.zeros((1, 2, 1)), "HND", torch.bfloat16, 128, True)
    with pytest.raises(ValueError, match="dense W8A8"):
        core.prequantize_sol_sageattn_from_qk(qk, q, use_w8a8=False)
    with pytest.raises(ValueError, match="causal masking is supported only by dense W8A8"):
        core.prequantize_sol_sageattn_from_qk(qk, q, use_w8a8=True, is_causal=True)
    with pytest.raises(ValueError, match="key_tile_tokens"):
        core.prequantize_sol_sageattn_from_qk(qk, q, use_w8a8=True, force_dense=True,
                                              key_tile_tokens=32)
    with pytest.raises(RuntimeError, match="force_dense"):
        qattn.sol_sparse_online_w8a8_prequantized_attn(
            q, q, q, q, q, q, q, None, None, None, None, None, None, None, 1.0, 1, 0.1, 0, 0, 64,
            0, 1)
    with pytest.raises(RuntimeError, match="key_tile_tokens must be 64 or 128"):
        qattn.sol_sparse_online_w8a8_prequantized_attn(
            q, q, q, q, q, q, q, None, None, None, None, None, None, None, 1.0, 1, 0.1, 0, 1, 96,
            0, 1)


def test_w8a8_attention_is_a_fullgraph_leaf():
    from comfyui_turing_utils_kernel.turing_sage.custom_ops import w8a8_attention

    q = torch.empty((1, 8, 300, 128), dtype=torch.bfloat16, device="meta")
    k = torch.empty((1, 2, 300, 128), dtype=torch.bfloat16, device="meta")
    compiled = torch.compile(
        lambda a, b, c: w8a8_attention(a, b, c, "HND", True, -1.0, 0, True, True),
        backend="eager", fullgraph=True)
    out = compiled(q, k, k)
    assert out.shape == q.shape and out.dtype == q.dtype


def test_staged_w4_weight_chunks():
    """One decode + GEMM round for every configs shape; above the cap, equal
    chunks on the GEMM's 256-column tile that cover N."""
    from comfyui_turing_utils_kernel._C import _WEIGHT_CHUNK_BYTES, _weight_chunk_rows

    for n, k in ((5120, 5120), (13824, 5120), (5120, 13824), (8, 16)):
        assert _weight_chunk_rows(n, k) == n
    for n, k in ((65536, 5120), (40000, 8192), (1 << 20, 4096)):
        rows = _weight_chunk_rows(n, k)
        assert rows % 256 == 0 and rows * k <= _WEIGHT_CHUNK_BYTES + 256 * k
        assert -(-n // rows) == -(-(n * k) // _WEIGHT_CHUNK_BYTES)
