"""CPU oracle for the quantized DiT path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the arithmetic of the reference plugin
``comfyui-turing-utils`` (kernel package 0.29.1) for the hot path this
repository accelerates.  It is the checker: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) import it.  The product library never calls it and
has no CPU fallback.

Integer/byte work (ConvRot codes and scales, INT32 accumulators, W4 and
codebook decode, Sage Q/K codes and scales) is restated in ``oracle.c`` and is
the bit-exact bar.  Floating-point outputs (bf16 GEMM outputs, attention) are
checked against the reference's own dequantize-then-matmul /
dequantize-then-attention fp32 torch path (kernel/scripts/validate_compatible.py:
110-114, 163-167, 540-546) within the north-star tolerances (cosine >= 0.9995,
relative L2 <= 1e-2).

Parity pinning: the reference publishes no stored fixtures; its checks are
seeded in-process on CUDA.  ``oracle/ref/`` builds the reference's own CUDA
sources (read from the reference checkout at build time) into ``oracle/_ref``;
``tests/golden/make_golden.py`` runs those on a B200 and commits the input /
output pairs under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks
this oracle against them on the CPU.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle.so"
_lib = None

_i64 = ctypes.c_int64
_int = ctypes.c_int
_ptr = ctypes.c_void_p


def build(force: bool = False) -> Path:
    """Compile oracle.c into liboracle.so (gcc, strict IEEE, no FMA contraction)."""
    src = _HERE / "oracle.c"
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.check_call(
            ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
             "-o", str(_LIB_PATH), str(src), "-lm"])
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(_LIB_PATH))
        L.orc_convrot_quantize.argtypes = [_ptr, _i64, _i64, _int, _int, _int, _int, _ptr, _ptr]
        L.orc_convrot_rotate_bf16.argtypes = [_ptr, _i64, _i64, _ptr, _ptr]
        L.orc_int8_gemm_rows.argtypes = [_ptr, _ptr, _i64, _i64, _ptr, _i64, _ptr]
        L.orc_dequant_bf16.argtypes = [_ptr, _i64, _i64, _i64, _ptr, _ptr, _int, _ptr, _ptr]
        L.orc_unpack_int4.argtypes = [_ptr, _i64, _i64, _ptr]
        L.orc_codebook_decode.argtypes = [_ptr, _ptr, _ptr, _i64, _i64, _i64, _ptr]
        L.orc_sage_quant.argtypes = [_ptr, _int, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _ptr,
                                     _i64, _ptr, _ptr]
        L.orc_token_mean.argtypes = [_ptr, _int, _i64, _i64, _i64, _i64, _i64, _ptr]
        L.orc_qk_rms_rope.argtypes = [_ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _i64, _i64,
                                      _i64, _i64, _int, _int, _int, _int, ctypes.c_float, _ptr,
                                      _ptr]
        L.orc_k_anchor.argtypes = [_ptr, _int, _i64, _i64, _i64, _i64, _i64, _ptr, _ptr]
        L.orc_rot_quant.argtypes = [_ptr, _int, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _ptr,
                                    _int, _ptr, _ptr]
        L.orc_qk_processed.argtypes = [_ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _i64, _i64,
                                       _int, _int, _int, _int, ctypes.c_float, _ptr]
        L.orc_qk_anchor_processed.argtypes = [_ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _i64,
                                              _i64, _int, _int, _int, _int, ctypes.c_float, _ptr,
                                              _ptr]
        L.orc_quant_v.argtypes = [_ptr, _int, _i64, _i64, _i64, _i64, _i64, _i64, _ptr, _ptr]
        L.orc_w8a8_attn.argtypes = [_ptr, _ptr, _ptr, _ptr, _ptr, _ptr, _i64, _i64, _i64, _i64,
                                    _i64, _i64, _i64, _i64, _i64, ctypes.c_float, _int, _ptr]
        L.orc_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.orc_e4m3_to_f32.restype = ctypes.c_float
        for name in ("orc_f32_to_bf16", "orc_bf16_to_f32", "orc_f32_to_f16", "orc_f16_to_f32"):
            getattr(L, name).argtypes = [_ptr, _i64, _ptr]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ------------------------------------------------------------------ dtypes --

def f32_to_bf16(x) -> np.ndarray:
    """fp32 -> bf16 bits (uint16), round to nearest even (convrot_quant.cu:293-305)."""
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_bf16(_p(x), x.size, _p(out))
    return out


def bf16_to_f32(h) -> np.ndarray:
    h = _c(h, np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().orc_bf16_to_f32(_p(h), h.size, _p(out))
    return out


def f32_to_f16(x) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_f16(_p(x), x.size, _p(out))
    return out


def f16_to_f32(h) -> np.ndarray:
    h = _c(h, np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().orc_f16_to_f32(_p(h), h.size, _p(out))
    return out


def e4m3_to_f32(b) -> np.ndarray:
    b = _c(b, np.uint8)
    table = np.array([lib().orc_e4m3_to_f32(i) for i in range(256)], np.float32)
    return table[b]


# ---------------------------------------------------------------- ConvRot ---

_ACT = {None: 0, "none": 0, "swiglu": 1, "gelu": 2}


def convrot_quantize(x_bits: np.ndarray, *, int4: bool = False, act=None, staged: bool = False,
                     fp16: bool = False):
    """ConvRot rotate + per-token quantize.

    x_bits: uint16 bf16 (or fp16 when fp16=True) bits, shape [rows, width]; width
    is 2*hidden for act="swiglu".  Returns (codes int8 [rows, hidden] or packed
    [rows, hidden/2], scales fp32 [rows, 1]).
    """
    x = _c(x_bits, np.uint16)
    rows, width = x.shape
    mode = _ACT[act]
    hidden = width // 2 if mode == 1 else width
    if hidden % 256:
        raise ValueError("hidden must be a multiple of 256")
    out = np.empty((rows, hidden // 2 if int4 else hidden), np.int8)
    scales = np.empty((rows, 1), np.float32)
    lib().orc_convrot_quantize(_p(x), rows, hidden, mode, int(int4), int(staged), int(fp16),
                               _p(out), _p(scales))
    return out, scales


def convrot_rotate_bf16(x_bits: np.ndarray):
    x = _c(x_bits, np.uint16)
    rows, k = x.shape
    out = np.empty((rows, k), np.uint16)
    gmax = np.empty((rows, k // 256), np.float32)
    lib().orc_convrot_rotate_bf16(_p(x), rows, k, _p(out), _p(gmax))
    return out, gmax


def hadamard256_matrix() -> np.ndarray:
    """The 256x256 orthogonal ConvRot rotation kron(M,M,M,M), M = 1/2[[1,1,1,-1],...]
    (convrot_quant.cu:104-116), in float64 — for property tests."""
    m = 0.5 * np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], np.float64)
    h = m
    for _ in range(3):
        h = np.kron(h, m)
    return h


# ------------------------------------------------------------------- GEMM ---

def int8_gemm_rows(a: np.ndarray, w: np.ndarray, rows=None) -> np.ndarray:
    """Exact INT32 accumulators acc[r, n] = sum_k a[rows[r], k] * w[n, k]."""
    a = _c(a, np.int8)
    w = _c(w, np.int8)
    m, k = a.shape
    n = w.shape[0]
    idx = np.arange(m, dtype=np.int64) if rows is None else _c(rows, np.int64)
    acc = np.empty((idx.size, n), np.int32)
    lib().orc_int8_gemm_rows(_p(a), _p(w), n, k, _p(idx), idx.size, _p(acc))
    return acc


def dequant_bf16(acc: np.ndarray, a_s, w_s, bias=None) -> np.ndarray:
    """bf16 bits of ((acc * a_s[m]) * w_s[n]) (+ bias[n])."""
    acc = _c(acc, np.int32)
    rows, cols = acc.shape
    a_s = _c(np.reshape(a_s, -1), np.float32)
    w_s = _c(np.reshape(w_s, -1), np.float32)
    out = np.empty((rows, cols), np.uint16)
    b = None if bias is None else _c(np.reshape(bias, -1), np.float32)
    lib().orc_dequant_bf16(_p(acc), rows, cols, cols, _p(a_s), _p(w_s), int(w_s.size == 1),
                           None if b is None else _p(b), _p(out))
    return out


def unpack_int4(packed: np.ndarray, k: int) -> np.ndarray:
    packed = _c(packed, np.int8)
    n = packed.shape[0]
    out = np.empty((n, k), np.int8)
    lib().orc_unpack_int4(_p(packed), n, k, _p(out))
    return out


def pack_int4(values: np.ndarray) -> np.ndarray:
    """Pack signed int4 values [-8, 7] two per byte, low nibble = even column
    (validate_compatible.py:28-31)."""
    v = values.astype(np.int32)
    return ((v[:, 0::2] & 0xF) | ((v[:, 1::2] & 0xF) << 4)).astype(np.uint8).view(np.int8)


def codebook_decode(packed: np.ndarray, group_scale_u8: np.ndarray, codebook: np.ndarray,
                    group_size: int) -> np.ndarray:
    packed = _c(packed, np.int8)
    gs = _c(group_scale_u8, np.uint8)
    cb = _c(np.reshape(codebook, -1), np.float32)
    n = packed.shape[0]
    k = packed.shape[1] * 2
    out = np.empty((n, k), np.int8)
    lib().orc_codebook_decode(_p(packed), _p(gs), _p(cb), n, k, group_size, _p(out))
    return out


# -------------------------------------------------------------- Sage quant --

def sage_quant(x_bits: np.ndarray, tile_tokens: int, *, layout: str = "HND", fp16: bool = False,
               mean_bits: np.ndarray | None = None, block: int | None = None):
    """Per-tile INT8 quantization of a [B, H, L, D] (HND) or [B, L, H, D] (NHD)
    tensor (fused.cu:66-200).  Returns (codes int8, same shape; scale fp32
    [B, H, tiles]) with tiles = ceil(L/T), or ceil(L/block) * (block/T) when
    block is given (per-warp Q layout).  mean_bits: optional [B, H, D] mean."""
    x = _c(x_bits, np.uint16)
    if layout == "HND":
        B, H, L, D = x.shape
        xs = x.reshape(B * H, L, D)
        s_outer, s_tok = L * D, D
        xv, outer = xs, B * H
        out = np.empty_like(x, dtype=np.int8)
        ov = out.reshape(B * H, L, D)
        tiles = (L + tile_tokens - 1) // tile_tokens
        if block is not None:
            tiles = (L + block - 1) // block * (block // tile_tokens)
        scale = np.empty((B, H, tiles), np.float32)
        m = None if mean_bits is None else _c(mean_bits, np.uint16).reshape(B * H, D)
        lib().orc_sage_quant(_p(xv), int(fp16), outer, L, D, s_outer, s_tok, tile_tokens, tiles,
                             None if m is None else _p(m), D, _p(ov), _p(scale))
        return out, scale
    if layout == "NHD":
        B, L, H, D = x.shape
        xt = np.ascontiguousarray(x.transpose(0, 2, 1, 3))
        mt = mean_bits
        q, s = sage_quant(xt, tile_tokens, layout="HND", fp16=fp16, mean_bits=mt, block=block)
        return np.ascontiguousarray(q.transpose(0, 2, 1, 3)), s
    raise ValueError(f"Unknown tensor layout: {layout}")


def token_mean(x_bits: np.ndarray, *, layout: str = "HND", fp16: bool = False) -> np.ndarray:
    """Per-(batch, head, channel) token mean rounded to the input dtype -> [B, H, D] bits."""
    x = _c(x_bits, np.uint16)
    if layout == "NHD":
        x = np.ascontiguousarray(x.transpose(0, 2, 1, 3))
    B, H, L, D = x.shape
    out = np.empty((B, H, D), np.uint16)
    lib().orc_token_mean(_p(x), int(fp16), B * H, L, D, L * D, D, _p(out))
    return out


def qk_rms_rope_int8(x_bits: np.ndarray, norm_bits: np.ndarray, freqs_bits, *, tile_tokens: int,
                     eps: float, rot_dim: int, layout: str = "HND", norm_scope: str = "head",
                     split_half: bool = False, fp16: bool = False):
    """Fused RMSNorm + RoPE + INT8 of one of Q (tile_tokens 16, per-warp
    layout) / K (64) (kernel/csrc/turing/sage/qk_preprocess.cu:151-201,
    :203-251, :417-563).  x_bits [B, H, L, D] (HND) or [B, L, H, D] (NHD);
    norm_bits [D] or [H*D]; freqs_bits [fb, fs, 1, rot_dim/2, 2, 2] or None.
    Returns (codes int8 in the input layout, scale fp32 [B, H, tiles])."""
    x = _c(x_bits, np.uint16)
    if layout == "NHD":
        x = np.ascontiguousarray(x.transpose(0, 2, 1, 3))
    elif layout != "HND":
        raise ValueError(f"Unknown tensor layout: {layout}")
    B, H, L, D = x.shape
    tiles = (L + 63) // 64 * (64 // tile_tokens)
    f = None
    fb = fs = 1
    if rot_dim > 0:
        f = _c(freqs_bits, np.uint16)
        fb, fs = f.shape[0], f.shape[1]
        f = np.ascontiguousarray(f.reshape(fb, fs, rot_dim // 2, 2, 2))
    n = _c(norm_bits, np.uint16).reshape(-1)
    out = np.empty(x.shape, np.int8)
    scale = np.empty((B, H, tiles), np.float32)
    lib().orc_qk_rms_rope(_p(x), _p(n), None if f is None else _p(f), B, H, L, D, tile_tokens,
                          tiles, fb, fs, int(rot_dim), int(bool(split_half)),
                          int(norm_scope == "row"), int(fp16), float(eps), _p(out), _p(scale))
    if layout == "NHD":
        out = np.ascontiguousarray(out.transpose(0, 2, 1, 3))
    return out, scale


def _hnd(x_bits, layout):
    x = _c(x_bits, np.uint16)
    if layout == "NHD":
        return np.ascontiguousarray(x.transpose(0, 2, 1, 3))
    if layout != "HND":
        raise ValueError(f"Unknown tensor layout: {layout}")
    return x


def k_anchor(k_bits: np.ndarray, *, layout: str = "HND", fp16: bool = False,
             with_values: bool = False):
    """K stabilization anchor row per (batch, kv head), or -1
    (DetectKAnchorKernel, sage/fused.cu:406-556).  Returns int32 [B, Hk]
    (and, with_values, the anchor rows as fp32 [B, Hk, D], zeros for -1)."""
    k = _hnd(k_bits, layout)
    B, H, L, D = k.shape
    out = np.empty((B, H), np.int32)
    vals = np.empty((B, H, D), np.float32)
    lib().orc_k_anchor(_p(k), int(fp16), B * H, L, D, L * D, D, _p(out), _p(vals))
    return (out, vals) if with_values else out


def rot_quant(x_bits: np.ndarray, tile_tokens: int, *, layout: str = "HND", fp16: bool = False,
              anchor_values: np.ndarray | None = None, block: int | None = None,
              nan_code: int = 0):
    """Randomized-Hadamard per-tile INT8 (quant_int8_tile, sage/fused.cu:260-398)
    of a [B, H, L, D] (HND) / [B, L, H, D] (NHD) tensor with D = 64 or 128.
    tile_tokens 16 (Q, per-warp layout: pass block=64) or 64 (K).
    anchor_values: optional fp32 [B, H, D] subtracted first (K; zeros = no
    anchor).  nan_code: code of a NaN (0 as fused.cu, -127 as the fused
    prologue).  Returns (codes int8 in the input layout, scale fp32
    [B, H, tiles])."""
    x = _hnd(x_bits, layout)
    B, H, L, D = x.shape
    if D not in (64, 128):
        raise ValueError("rot_quant takes the kernel head dim 64 or 128 (pad first)")
    tiles = (L + tile_tokens - 1) // tile_tokens
    if block is not None:
        tiles = (L + block - 1) // block * (block // tile_tokens)
    out = np.empty(x.shape, np.int8)
    scale = np.empty((B, H, tiles), np.float32)
    a = None if anchor_values is None else _c(anchor_values, np.float32).reshape(B * H, D)
    lib().orc_rot_quant(_p(x), int(fp16), B * H, L, D, L * D, D, tile_tokens, tiles,
                        None if a is None else _p(a), int(nan_code), _p(out), _p(scale))
    if layout == "NHD":
        out = np.ascontiguousarray(out.transpose(0, 2, 1, 3))
    return out, scale


def per_warp_int8_hadamard(q_bits, k_bits, *, layout: str = "HND", fp16: bool = False,
                           stabilize_k: bool = True):
    """Q per 16 rows and K per 64 rows, both rotated, K anchored when
    stabilize_k (turing_sage/quant.py:182-243).  Returns (q8, q_scale, k8,
    k_scale, anchors or None)."""
    anchors, values = (k_anchor(k_bits, layout=layout, fp16=fp16, with_values=True)
                       if stabilize_k else (None, None))
    q8, qs = rot_quant(q_bits, 16, layout=layout, fp16=fp16, block=64)
    k8, ks = rot_quant(k_bits, 64, layout=layout, fp16=fp16, anchor_values=values)
    return q8, qs, k8, ks, anchors


def _prologue_args(x_bits, norm_bits, freqs_bits, rot_dim, layout):
    x = _hnd(x_bits, layout)
    f = None
    fb = fs = 1
    if rot_dim > 0:
        f = _c(freqs_bits, np.uint16)
        fb, fs = f.shape[0], f.shape[1]
        f = np.ascontiguousarray(f.reshape(fb, fs, rot_dim // 2, 2, 2))
    return x, _c(norm_bits, np.uint16).reshape(-1), f, fb, fs


def qk_processed(x_bits, norm_bits, freqs_bits, *, eps: float, rot_dim: int,
                 layout: str = "HND", norm_scope: str = "head", split_half: bool = False,
                 fp16: bool = False) -> np.ndarray:
    """RMSNorm + RoPE of every token as the fused prologue computes it before
    quantizing (qk_preprocess.cu:151-201): bits of the input dtype, input layout."""
    x, n, f, fb, fs = _prologue_args(x_bits, norm_bits, freqs_bits, rot_dim, layout)
    B, H, L, D = x.shape
    out = np.empty(x.shape, np.uint16)
    lib().orc_qk_processed(_p(x), _p(n), None if f is None else _p(f), B, H, L, D, fb, fs,
                           int(rot_dim), int(bool(split_half)), int(norm_scope == "row"),
                           int(fp16), float(eps), _p(out))
    if layout == "NHD":
        out = np.ascontiguousarray(out.transpose(0, 2, 1, 3))
    return out


def qk_anchor_processed(k_bits, norm_bits, freqs_bits, *, eps: float, rot_dim: int,
                        layout: str = "HND", norm_scope: str = "head", split_half: bool = False,
                        fp16: bool = False):
    """The fused prologue's K anchor (detect_anchor_kernel, qk_preprocess.cu:252-415).
    Returns (int32 [B, H] row or -1, fp32 [B, H, D] anchor values)."""
    k, n, f, fb, fs = _prologue_args(k_bits, norm_bits, freqs_bits, rot_dim, layout)
    B, H, L, D = k.shape
    idx = np.empty((B, H), np.int32)
    vals = np.empty((B, H, D), np.float32)
    lib().orc_qk_anchor_processed(_p(k), _p(n), None if f is None else _p(f), B, H, L, D, fb, fs,
                                  int(rot_dim), int(bool(split_half)), int(norm_scope == "row"),
                                  int(fp16), float(eps), _p(idx), _p(vals))
    return idx, vals


def qk_rms_rope_rotated_int8(q_bits, k_bits, q_norm, k_norm, freqs_bits, *, eps: float,
                             rot_dim: int, layout: str = "HND", norm_scope: str = "head",
                             split_half: bool = False, fp16: bool = False,
                             stabilize_k: bool = True):
    """The fused prologue with rotate_qk (qk_preprocess.cu:417-753): processed
    Q/K, K minus its processed anchor, randomized Hadamard, per-tile INT8 with
    NaN -> -127.  Returns (q8, q_scale, k8, k_scale, anchors or None)."""
    kw = dict(eps=eps, rot_dim=rot_dim, layout=layout, norm_scope=norm_scope,
              split_half=split_half, fp16=fp16)
    qp = qk_processed(q_bits, q_norm, freqs_bits, **kw)
    kp = qk_processed(k_bits, k_norm, freqs_bits, **kw)
    anchors, values = (qk_anchor_processed(k_bits, k_norm, freqs_bits, **kw)
                       if stabilize_k else (None, None))
    q8, qs = rot_quant(qp, 16, layout=layout, fp16=fp16, block=64, nan_code=-127)
    k8, ks = rot_quant(kp, 64, layout=layout, fp16=fp16, anchor_values=values, nan_code=-127)
    return q8, qs, k8, ks, anchors


def quant_v(v_bits: np.ndarray, *, layout: str = "HND", fp16: bool = False):
    """Channel-wise INT8 V (quant_v_int8_cuda_sm75.cu:58-164).  Returns (codes
    int8 [B, H, D, ceil(L/64)*64] channel-major, un-permuted; scale fp32
    [B, H, D])."""
    v = _hnd(v_bits, layout)
    B, H, L, D = v.shape
    lpad = (L + 63) // 64 * 64
    codes = np.empty((B, H, D, lpad), np.int8)
    scale = np.empty((B, H, D), np.float32)
    lib().orc_quant_v(_p(v), int(fp16), B * H, L, D, L * D, D, lpad, _p(codes), _p(scale))
    return codes, scale


def w8a8_attn(q8, k8, v8, v_scale, q_scale, k_scale, *, sm_scale: float,
              is_causal: bool = False) -> np.ndarray:
    """Dense W8A8-PV attention (sol_sparse_cuda_sm75.cu:1197-1320) on HND INT8
    Q/K, channel-major INT8 V [B, Hk, D, Lpad] and their scales.  Returns the
    fp32 output [B, Hq, Lq, D] before the final rounding."""
    q8, k8, v8 = _c(q8, np.int8), _c(k8, np.int8), _c(v8, np.int8)
    B, Hq, Lq, D = q8.shape
    Hk, Lk = k8.shape[1], k8.shape[2]
    qs, ks, vs = _c(q_scale, np.float32), _c(k_scale, np.float32), _c(v_scale, np.float32)
    out = np.empty((B, Hq, Lq, D), np.float32)
    lib().orc_w8a8_attn(_p(q8), _p(k8), _p(v8), _p(vs), _p(qs), _p(ks), B, Hq, Hk, Lq, Lk, D,
                        v8.shape[3], qs.shape[2], ks.shape[2], float(sm_scale),
                        int(bool(is_causal)), _p(out))
    return out


def w8a8attn(q_bits, k_bits, v_bits, *, layout: str = "HND", fp16: bool = False,
             sm_scale: float | None = None, is_causal: bool = False, rotate_qk: bool = True,
             stabilize_k: bool = True) -> np.ndarray:
    """The whole dense W8A8 path (turing_sage/core.py:656-708 with
    prequantize_sol_sageattn :842-914): head dim padded to 64 / 128, rotated
    (anchored) or plain per-warp Q/K INT8, channel-wise INT8 V, W8A8-PV
    attention, output rounded to the input dtype.  Returns output bits
    (uint16) in the input layout with the original head dim."""
    q, k, v = (_hnd(t, layout) for t in (q_bits, k_bits, v_bits))
    D = q.shape[-1]
    kd = 64 if D <= 64 else 128
    if D < kd:
        q, k, v = (np.pad(t, ((0, 0), (0, 0), (0, 0), (0, kd - D))) for t in (q, k, v))
    if rotate_qk:
        q8, qs, k8, ks, _ = per_warp_int8_hadamard(q, k, fp16=fp16, stabilize_k=stabilize_k)
    else:
        q8, qs = sage_quant(q, 16, fp16=fp16, block=64)
        k8, ks = sage_quant(k, 64, fp16=fp16)
    v8, vs = quant_v(v, fp16=fp16)
    scale = float(sm_scale) if sm_scale is not None else D ** -0.5
    o = w8a8_attn(q8, k8, v8, vs, qs, ks, sm_scale=scale, is_causal=is_causal)
    bits = (f32_to_f16 if fp16 else f32_to_bf16)(o)[..., :D]
    if layout == "NHD":
        bits = bits.transpose(0, 2, 1, 3)
    return np.ascontiguousarray(bits)


def q_scale_shape(B, H, L, block=64, warp=16):
    """q_scale layout of the reference (quant.py:95-115, core.py:622-627)."""
    return (B, H, ((L + block - 1) // block) * (block // warp))


def k_scale_shape(B, H, L, block=64):
    return (B, H, (L + block - 1) // block)


# ----------------------------------------------- float references (torch) --

def dequant_matmul_reference(a_int8, w_int8, a_s, w_s, bias=None):
    """fp32 dequantize-then-matmul (validate_compatible.py:110-114): returns fp32."""
    import torch
    a = torch.as_tensor(np.asarray(a_int8)).float()
    w = torch.as_tensor(np.asarray(w_int8)).float()
    ref = (a @ w.t()) * torch.as_tensor(np.reshape(a_s, (-1, 1))).float() \
        * torch.as_tensor(np.reshape(w_s, (1, -1))).float()
    if bias is not None:
        ref = ref + torch.as_tensor(np.reshape(bias, (1, -1))).float()
    return ref


def dequant_attention_reference(q8, q_scale, k8, k_scale, v, *, sm_scale, is_causal=False,
                                q_tile=16, k_tile=64, layout="HND", q_rows=None):
    """fp32 dequantize-then-attention (validate_compatible.py:458-575 semantics, on
    the dequantized INT8 Q/K).  q8/k8 int8 torch tensors, scales fp32 torch
    tensors [B, H, tiles], v float torch tensor.  q_rows: optional index tensor
    of query rows to evaluate (sampling for large shapes).  Returns fp32 in HND."""
    import torch
    if layout == "NHD":
        q8, k8, v = (t.transpose(1, 2) for t in (q8, k8, v))
    B, Hq, Lq, D = q8.shape
    Hk, Lk = k8.shape[1], k8.shape[2]
    qs = q_scale.float().repeat_interleave(q_tile, dim=2)[:, :, :Lq]
    ks = k_scale.float().repeat_interleave(k_tile, dim=2)[:, :, :Lk]
    qf = q8.float() * qs[..., None]
    kf = k8.float() * ks[..., None]
    vf = v.float()
    if Hq != Hk:
        kf = kf.repeat_interleave(Hq // Hk, dim=1)
        vf = vf.repeat_interleave(Hq // Hk, dim=1)
    if q_rows is not None:
        qf = qf[:, :, q_rows]
    scores = torch.matmul(qf, kf.transpose(-1, -2)) * sm_scale
    if is_causal:
        qi = torch.arange(Lq)[:, None] if q_rows is None else torch.as_tensor(q_rows)[:, None]
        mask = torch.arange(Lk)[None, :] > qi
        scores = scores.masked_fill(mask, float("-inf"))
    return torch.softmax(scores, dim=-1) @ vf


def metrics(actual, expected) -> dict:
    """max_abs / relative L2 / cosine (turing_sage/correctness.py:30-143 semantics)."""
    import torch
    a = torch.as_tensor(actual).double().flatten()
    e = torch.as_tensor(expected).double().flatten()
    diff = a - e
    rel_l2 = (diff.norm() / e.norm().clamp_min(1e-30)).item()
    cos = (torch.dot(a, e) / (a.norm() * e.norm()).clamp_min(1e-30)).item()
    return {"max_abs": diff.abs().max().item() if diff.numel() else 0.0,
            "rel_l2": rel_l2, "cosine": cos}


NORTH_STAR_COSINE = 0.9995
NORTH_STAR_REL_L2 = 1.0e-2


__all__ = [name for name in dir() if not name.startswith("_")]


# ------------------------------------------------------------ norm + AdaLN --
# CPU restatement of kernel/csrc/turing/segmented_rms_adaln.cu with float64
# statistics (the kernels reduce in fp32 in their own orders, so results agree
# to the last-bit rounding of the output dtype, not bit for bit).

def _round_to(a64: np.ndarray, dtype) -> np.ndarray:
    """float64 -> dtype (torch float16 / bfloat16 / float32) -> float64."""
    import torch

    return torch.from_numpy(np.asarray(a64, np.float64)).to(dtype).double().numpy()


def segment_rows(segments: np.ndarray, rows: int, modulation_rows: int) -> np.ndarray:
    """Modulation row of every token row (segmented_rms_adaln.cu:115-132):
    the [start, stop, row] segment holding it (segments sorted by stop), 0 when
    none does or the named row is out of range."""
    seg = np.asarray(segments, np.int64).reshape(-1, 3)
    out = np.zeros(rows, np.int64)
    for r in range(rows):
        i = int(np.searchsorted(seg[:, 1], r, side="right"))
        m = -1
        if i < len(seg) and r >= seg[i, 0]:
            m = int(seg[i, 2])
        out[r] = m if 0 <= m < modulation_rows else 0
    return out


def rms_adaln(x, w, scale, shift, segments, eps, dtype):
    """out = T(x * rsqrt(mean(x^2) + eps) * w * (1 + scale[m]) + shift[m])
    (segmented_rms_adaln.cu:135-235); inputs as float arrays of T values."""
    x = np.asarray(x, np.float64)
    inv = 1.0 / np.sqrt(np.mean(x * x, axis=1, keepdims=True) + eps)
    m = segment_rows(segments, x.shape[0], np.asarray(scale).shape[0])
    sc, sh = np.asarray(scale, np.float64)[m], np.asarray(shift, np.float64)[m]
    return _round_to(x * inv * np.asarray(w, np.float64)[None] * (1.0 + sc) + sh, dtype)


def layer_norm_adaln(x, scale, shift, eps, dtype):
    """n = T((x - mean) * rsqrt(var + eps)), out = T(n * T(1 + scale) + shift) with
    token t of a batch on modulation step min(t / ceil(seq / steps), steps - 1)
    (segmented_rms_adaln.cu:237-306)."""
    x = np.asarray(x, np.float64)
    batch, seq, hid = x.shape
    steps = np.asarray(scale).shape[1]
    per = -(-seq // steps)
    tok = np.minimum(np.arange(seq) // max(per, 1), steps - 1) if steps > 1 else np.zeros(seq, int)
    mean = x.mean(axis=2, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=2, keepdims=True)
    n = _round_to((x - mean) / np.sqrt(var + eps), dtype)
    sc = np.asarray(scale, np.float64)[:, tok]
    sh = np.asarray(shift, np.float64)[:, tok]
    mult = _round_to(1.0 + sc, dtype)
    return _round_to(n * mult + sh, dtype)
