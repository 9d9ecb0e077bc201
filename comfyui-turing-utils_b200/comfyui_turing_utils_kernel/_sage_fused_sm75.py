"""Drop-in for the reference's ``_sage_fused_sm75`` extension (quantizer part).

Same entry-point names and argument order as
kernel/csrc/turing/sage/pybind_fused.cpp:23-33 (fused.h); the work runs in the
sm_100a quantizer kernels of libturing_b200.so.  Outputs are caller-allocated
and written in place, as in the reference.
"""
from __future__ import annotations

import ctypes

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


def quant_qk_rms_rope_int8_cuda(query, key, query_output, key_output, query_scale, key_scale,
                                query_norm, key_norm, freqs, query_rrms, key_rrms, anchor_indices,
                                anchor_values, epsilon, rot_dim, query_block_size,
                                query_warp_block_size, key_block_size, tensor_layout, norm_scope,
                                split_half, rotate):
    """Fused RMSNorm + RoPE + Q/K INT8 quantization (qk_preprocess.cu:566-753).
    rotate=True is the W8A8 form: the normalized + rotated values are written
    once in the input dtype (tb_qk_rms_rope_apply), K's anchor is chosen from
    nine processed samples when anchor_indices is non-empty
    (tb_qk_anchor_processed; as in the reference, anchors are ignored without
    rotate), and the randomized-Hadamard quantizer codes them
    (tb_quant_qk_int8_rotated, NaN -> -127 as in this prologue)."""
    for t, name in ((query, "query"), (key, "key"), (query_output, "query_output"),
                    (key_output, "key_output"), (query_scale, "query_scale"),
                    (key_scale, "key_scale"), (query_norm, "query_norm"), (key_norm, "key_norm")):
        _check(t.is_cuda, f"{name} must be a CUDA tensor")
    _check(query.dim() == 4 and key.dim() == 4, "Q/K must be 4D tensors")
    _check(query.stride(-1) == 1 and key.stride(-1) == 1, "Q/K last dim must be contiguous")
    _check(query_output.is_contiguous() and key_output.is_contiguous()
           and query_scale.is_contiguous() and key_scale.is_contiguous(),
           "outputs and scales must be contiguous")
    _check(query_output.dtype == torch.int8 and key_output.dtype == torch.int8,
           "Q/K outputs must be int8")
    _check(query_scale.dtype == torch.float32 and key_scale.dtype == torch.float32,
           "Q/K scales must be float32")
    _check(query.dtype == key.dtype, "Q/K dtypes must match")
    _check(query_norm.dtype == query.dtype and key_norm.dtype == query.dtype,
           "Q/K norm weights must match the input dtype")
    _check(query_block_size == 64 and query_warp_block_size == 16 and key_block_size == 64,
           "fused Q/K preprocessing requires the production 64/16/64 quantization contract")
    _check(norm_scope in (0, 1, 2),
           "norm_scope must be 0 (per head), 1 (whole row) or 2 (whole row, RRMS given)")
    head_dim = query.size(3)
    _check(head_dim in (64, 128), "fused Q/K preprocessing requires head_dim 64 or 128")
    _check(key.size(3) == head_dim and query.size(0) == key.size(0), "Q/K shapes are incompatible")
    B, qh, ql, _, qsb, qsh, qsl = _geometry(query, int(tensor_layout))
    _, kh, kl, _, ksb, ksh, ksl = _geometry(key, int(tensor_layout))
    _check(rot_dim >= 0 and rot_dim <= head_dim and rot_dim % 2 == 0,
           "rot_dim must be even and within head_dim")
    _check(query_norm.numel() == (head_dim if norm_scope == 0 else qh * head_dim)
           and key_norm.numel() == (head_dim if norm_scope == 0 else kh * head_dim),
           "Q/K norm weight shapes are incompatible")
    _check(query_output.shape == query.shape and key_output.shape == key.shape,
           "Q/K output shapes must match inputs")
    qsl_len, ksl_len = (ql + 63) // 64 * 4, (kl + 63) // 64
    _check(tuple(query_scale.shape) == (B, qh, qsl_len), "Q scale shape is incompatible")
    _check(tuple(key_scale.shape) == (B, kh, ksl_len), "K scale shape is incompatible")
    fstr, fb, fs = None, 1, 1
    if rot_dim > 0:
        _check(freqs.is_cuda and freqs.dim() == 6, "freqs must be a 6D CUDA tensor")
        _check(freqs.dtype == query.dtype, "RoPE frequencies must match Q/K dtype")
        _check(freqs.size(2) == 1 and freqs.size(3) == rot_dim // 2 and freqs.size(4) == 2
               and freqs.size(5) == 2, "RoPE frequency shape is incompatible")
        fb, fs = freqs.size(0), freqs.size(1)
        _check((fb == 1 or fb == B) and (fs == 1 or (fs == ql and ql == kl)),
               "RoPE batch/sequence broadcasting is incompatible")
        fstr = torch.tensor([freqs.stride(0), freqs.stride(1), freqs.stride(3), freqs.stride(4),
                             freqs.stride(5)], dtype=torch.int64)
    if norm_scope in (1, 2):
        _check(query_rrms.is_cuda and key_rrms.is_cuda and query_rrms.dtype == torch.float32
               and key_rrms.dtype == torch.float32, "row RRMS scratch must be float32 CUDA")
        _check(query_rrms.numel() == B * ql and key_rrms.numel() == B * kl,
               "row RRMS scratch shapes are incompatible")
    # The kernel reads the weights as 16-byte packs: give it an aligned copy of
    # a weight view that starts mid-allocation.
    if query_norm.data_ptr() % 16:
        query_norm = query_norm.clone()
    if key_norm.data_ptr() % 16:
        key_norm = key_norm.clone()
    qo = _geometry(query_output, int(tensor_layout))
    ko = _geometry(key_output, int(tensor_layout))
    if rotate:
        _rms_rope_rotated(query, key, query_output, key_output, query_scale, key_scale, query_norm,
                          key_norm, freqs, query_rrms, key_rrms, anchor_indices, anchor_values,
                          epsilon, rot_dim, tensor_layout, norm_scope, split_half, fstr, fb, fs)
        return
    strides = torch.tensor([qsb, qsh, qsl, ksb, ksh, ksl, qo[4], qo[5], qo[6], ko[4], ko[5], ko[6],
                            query_scale.stride(0), query_scale.stride(1), key_scale.stride(0),
                            key_scale.stride(1)], dtype=torch.int64)
    with torch.cuda.device(query.device):
        call("tb_quant_qk_rms_rope_int8", ptr(query), ptr(key), ptr(query_output),
             ptr(key_output), ptr(query_scale), ptr(key_scale), ptr(query_norm), ptr(key_norm),
             ptr(freqs) if rot_dim > 0 else None,
             ptr(query_rrms) if norm_scope else None,
             ptr(key_rrms) if norm_scope else None, B, qh, kh, ql, kl, head_dim,
             strides.data_ptr(), None if fstr is None else fstr.data_ptr(), fb, fs, int(rot_dim),
             int(norm_scope), int(bool(split_half)), dtype_code(query), float(epsilon),
             stream_of(query))


def _rms_rope_rotated(query, key, query_output, key_output, query_scale, key_scale, query_norm,
                      key_norm, freqs, query_rrms, key_rrms, anchor_indices, anchor_values,
                      epsilon, rot_dim, tensor_layout, norm_scope, split_half, fstr, fb, fs):
    layout = int(tensor_layout)
    B, qh, ql, D, qsb, qsh, qsl = _geometry(query, layout)
    _, kh, kl, _, ksb, ksh, ksl = _geometry(key, layout)
    stabilize = anchor_indices.numel() != 0
    if stabilize:
        _check(anchor_indices.is_cuda and anchor_values.is_cuda
               and anchor_indices.dtype == torch.int32 and anchor_values.dtype == torch.float32,
               "K anchor scratch must be int32 / float32 CUDA tensors")
        _check(tuple(anchor_indices.shape) == (B, kh), "anchor index shape is incompatible")
        _check(tuple(anchor_values.shape) == (B, kh, D) and anchor_values.is_contiguous()
               and anchor_indices.is_contiguous(), "anchor value shape is incompatible")
    # The normalized + rotated Q/K, once, in the input dtype and output layout.
    q_proc = torch.empty(query_output.shape, dtype=query.dtype, device=query.device)
    k_proc = torch.empty(key_output.shape, dtype=key.dtype, device=key.device)
    qp, kp = _geometry(q_proc, layout), _geometry(k_proc, layout)
    qo, ko = _geometry(query_output, layout), _geometry(key_output, layout)
    apply_strides = torch.tensor([qsb, qsh, qsl, ksb, ksh, ksl, qp[4], qp[5], qp[6], kp[4], kp[5],
                                  kp[6]], dtype=torch.int64)
    quant_strides = (ctypes.c_int64 * 12)(qp[4], qp[5], qp[6], kp[4], kp[5], kp[6], qo[4], qo[5],
                                          qo[6], ko[4], ko[5], ko[6])
    fptr = ptr(freqs) if rot_dim > 0 else None
    fsp = None if fstr is None else fstr.data_ptr()
    with torch.cuda.device(query.device):
        stream = stream_of(query)
        call("tb_qk_rms_rope_apply", ptr(query), ptr(key), ptr(q_proc), ptr(k_proc),
             ptr(query_norm), ptr(key_norm), fptr, ptr(query_rrms) if norm_scope else None,
             ptr(key_rrms) if norm_scope else None, B, qh, kh, ql, kl, D,
             apply_strides.data_ptr(), fsp, fb, fs, int(rot_dim), int(norm_scope),
             int(bool(split_half)), dtype_code(query), float(epsilon), stream)
        if stabilize:
            kst = (ctypes.c_int64 * 3)(ksb, ksh, ksl)
            call("tb_qk_anchor_processed", ptr(key), ptr(key_norm), fptr,
                 ptr(key_rrms) if norm_scope else None, ptr(anchor_indices), ptr(anchor_values),
                 B, kh, kl, D, kst, fsp, fb, fs, int(rot_dim), int(norm_scope),
                 int(bool(split_half)), dtype_code(query), float(epsilon), stream)
        call("tb_quant_qk_int8_rotated", ptr(q_proc), ptr(k_proc), ptr(query_output),
             ptr(key_output), ptr(query_scale), ptr(key_scale),
             ptr(anchor_indices) if stabilize else None, ptr(anchor_values) if stabilize else None,
             B, qh, kh, ql, kl, D, quant_strides, 2 if stabilize else 0, -127, dtype_code(query),
             stream)


def row_sum_squares_cuda(input, sums, tensor_layout):
    """Per-token sum of squares over all heads of a [B, H, L, D] / [B, L, H, D]
    tensor into sums [B, L] fp32 (tensor-parallel row RMS; norm_scope 2 of
    quant_qk_rms_rope_int8_cuda takes the resulting RRMS).  Not in the
    reference, whose fused prologue always owns every head."""
    B, H, L, D, sb, sh, sl = _geometry(input, int(tensor_layout))
    _check(D in (64, 128), "head_dim must be 64 or 128")
    _check(sums.is_cuda and sums.dtype == torch.float32 and sums.is_contiguous()
           and sums.numel() == B * L, "sums must be a contiguous float32 CUDA [B, L] tensor")
    st = torch.tensor([sb, sh, sl], dtype=torch.int64)
    with torch.cuda.device(input.device):
        call("tb_row_sum_squares", ptr(input), ptr(sums), B, H, L, D, st.data_ptr(),
             dtype_code(input), stream_of(input))



def _rotated(query, key, query_output, key_output, query_scale, key_scale, anchor_indices,
             query_block_size, query_warp_block_size, key_block_size, tensor_layout):
    for name, t in (("query", query), ("key", key), ("query_output", query_output),
                    ("key_output", key_output), ("query_scale", query_scale),
                    ("key_scale", key_scale)):
        _check(t.is_cuda, f"{name} must be a CUDA tensor")
    _check(query_output.dtype == torch.int8 and key_output.dtype == torch.int8,
           "Q/K outputs must be int8")
    _check(query_scale.dtype == torch.float32 and key_scale.dtype == torch.float32,
           "Q/K scales must be float32")
    _check(query_output.is_contiguous() and key_output.is_contiguous()
           and query_scale.is_contiguous() and key_scale.is_contiguous(),
           "Q/K outputs and scales must be contiguous")
    _check(query.dtype == key.dtype,
           "Query and key must have the same data type")
    _check(query.size(0) == key.size(0), "Query and key batch size must match")
    _check(query.size(3) == key.size(3), "Query and key head_dim must match")
    _check((int(query_block_size), int(query_warp_block_size), int(key_block_size)) == (64, 16, 64),
           "the sm_100a rotated quantizer takes the production 64/16/64 tiles")
    layout = int(tensor_layout)
    B, Hq, Lq, D, qb, qh, ql = _geometry(query, layout)
    _, Hk, Lk, _, kb, kh, kl = _geometry(key, layout)
    _check(tuple(query_output.shape) == tuple(query.shape)
           and tuple(key_output.shape) == tuple(key.shape), "Q/K output shapes must match inputs")
    _check(tuple(query_scale.shape) == (B, Hq, (Lq + 63) // 64 * 4), "query_scale shape mismatch")
    _check(tuple(key_scale.shape) == (B, Hk, (Lk + 63) // 64), "key_scale shape mismatch")
    if anchor_indices is not None:
        _check(anchor_indices.is_cuda and anchor_indices.dtype == torch.int32
               and anchor_indices.is_contiguous() and tuple(anchor_indices.shape) == (B, Hk),
               "K anchor scratch must be a contiguous int32 [B, Hk] CUDA tensor")
        _check(anchor_indices.device == key.device,
               "K anchor scratch must be on the same CUDA device as K")
    _, _, _, _, qob, qoh, qol = _geometry(query_output, layout)
    _, _, _, _, kob, koh, kol = _geometry(key_output, layout)
    strides = (ctypes.c_int64 * 12)(qb, qh, ql, kb, kh, kl, qob, qoh, qol, kob, koh, kol)
    values = None
    if anchor_indices is not None:
        values = torch.empty((B, Hk, D), dtype=torch.float32, device=key.device)
    with torch.cuda.device(query.device):
        call("tb_quant_qk_int8_rotated", ptr(query), ptr(key), ptr(query_output), ptr(key_output),
             ptr(query_scale), ptr(key_scale), ptr(anchor_indices), ptr(values), B, Hq, Hk, Lq,
             Lk, D, strides, 1 if anchor_indices is not None else 0, 0, dtype_code(query),
             stream_of(query))


def quant_qk_per_warp_int8_rotated_cuda(query, key, query_output, key_output, query_scale,
                                        key_scale, query_block_size, query_warp_block_size,
                                        key_block_size, tensor_layout):
    """Randomized-Hadamard Q/K INT8 without K anchoring (fused.cu:1252-1268)."""
    _rotated(query, key, query_output, key_output, query_scale, key_scale, None,
             query_block_size, query_warp_block_size, key_block_size, tensor_layout)


def quant_qk_per_warp_int8_rotated_anchored_cuda(query, key, query_output, key_output,
                                                 query_scale, key_scale, anchor_indices,
                                                 query_block_size, query_warp_block_size,
                                                 key_block_size, tensor_layout):
    """Randomized-Hadamard Q/K INT8 with the conditional K anchor
    (fused.cu:1270-1287); anchor_indices receives the chosen rows (or -1)."""
    _rotated(query, key, query_output, key_output, query_scale, key_scale, anchor_indices,
             query_block_size, query_warp_block_size, key_block_size, tensor_layout)
