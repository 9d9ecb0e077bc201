"""Pins the CPU oracle to the reference itself: tests/golden/*.npz hold inputs
and the outputs of the reference's own CUDA kernels (compiled from its sources
and run on a B200 by tests/golden/make_golden.py).

Exactness bar per fixture:
  * ConvRot (plain rotation, all forms), W8A8/W4A8/codebook decode, dequant:
    bit-exact codes and scales (the reference's `_C` is built without
    fast-math, so its arithmetic is reproducible);
  * ConvRot with fused SwiGLU / GELU: the reference calls CUDA's expf/tanhf,
    the oracle the C library's; codes may differ by 1 in a few elements and
    scales by a few ulp;
  * bf16 GEMM outputs: the reference's CUTLASS epilogue may contract the bias
    add into an FMA, so outputs may differ by 1 bf16 ulp;
  * Sage quant: the reference's attention extension is built with
    --use_fast_math (approximate divides); codes may differ by 1 in a few
    elements, scales by a couple of ulp;
  * Sage attention: the reference output vs the oracle's fp32
    dequantize-then-attention on the reference's own INT8 Q/K, within the
    north-star bounds.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    path = GOLDEN / f"{name}.npz"
    if not path.exists():
        pytest.skip(f"golden fixture {name} not present")
    return dict(np.load(path))


def _ulp_diff(a, b):
    ai = a.view(np.int32).astype(np.int64)
    bi = b.view(np.int32).astype(np.int64)
    return np.abs(ai - bi)


def _bf16_ulp_diff(a_bits, b_bits):
    return np.abs(a_bits.astype(np.int32) - b_bits.astype(np.int32))


def _close_codes(got, want, max_frac):
    d = np.abs(got.astype(np.int16) - want.astype(np.int16))
    assert d.max() <= 1, d.max()
    assert (d > 0).mean() <= max_frac, (d > 0).mean()


@pytest.mark.parametrize("name", ["plain_5120", "plain_256", "edge_512"])
def test_convrot_plain_bit_exact(oracle, name):
    f = load(f"convrot_{name}")
    for int4 in (False, True):
        q, s = oracle.convrot_quantize(f["x"], int4=int4)
        tag = "4" if int4 else "8"
        assert np.array_equal(q, f[f"q{tag}"])
        assert np.array_equal(s.view(np.uint32), f[f"s{tag}"].view(np.uint32))


@pytest.mark.parametrize("name,act", [("swiglu_5376", "swiglu"), ("gelu_13824", "gelu")])
def test_convrot_fused_activation(oracle, name, act):
    f = load(f"convrot_{name}")
    x = f["x"]
    hidden = x.shape[1] // (2 if act == "swiglu" else 1)
    for int4 in (False, True):
        tag = "4" if int4 else "8"
        variants = [("", False, False), (f"_staged_{tag}", True, False),
                    (f"_staged16_{tag}", True, True)]
        for key, staged, fp16 in variants:
            qk = f"q{tag}" if key == "" else f"q{key}"
            sk = f"s{tag}" if key == "" else f"s{key}"
            xin = x
            if fp16:
                xin = oracle.f32_to_f16(oracle.bf16_to_f32(x))
            q, s = oracle.convrot_quantize(xin, int4=int4, act=act, staged=staged, fp16=fp16)
            if int4:
                _close_codes(oracle.unpack_int4(q, hidden), oracle.unpack_int4(f[qk], hidden), 1e-3)
            else:
                _close_codes(q, f[qk], 1e-3)
            assert _ulp_diff(s, f[sk]).max() <= 8


@pytest.mark.parametrize("name", ["int8_linear_33x128x128", "int8_linear_129x264x256"])
def test_int8_linear(oracle, name):
    f = load(name)
    acc = oracle.int8_gemm_rows(f["a"], f["w"])
    out = oracle.dequant_bf16(acc, f["a_s"], f["w_s"], f["bias"])
    assert _bf16_ulp_diff(out, f["out"]).max() <= 1


def test_w4a8_signed_nibble(oracle):
    f = load("w4a8_17x72x80")
    w = oracle.unpack_int4(f["w_packed"], f["a"].shape[1])
    acc = oracle.int8_gemm_rows(f["a"], w)
    out = oracle.dequant_bf16(acc, f["a_s"], f["w_s"])
    assert _bf16_ulp_diff(out, f["out"]).max() <= 1


@pytest.mark.parametrize("g", [16, 128])
def test_codebook(oracle, g):
    f = load(f"codebook_g{g}")
    w8 = oracle.codebook_decode(f["w_packed"], f["gs"], f["codebook"], g)
    assert np.array_equal(w8, f["w8"][: w8.shape[0]])
    acc = oracle.int8_gemm_rows(f["a"], w8)
    out = oracle.dequant_bf16(acc, f["a_s"], f["c_s"], f["bias"])
    assert _bf16_ulp_diff(out, f["out"]).max() <= 1


def test_dequant_epilogue_bit_exact(oracle):
    f = load("dequant_37x64")
    out = oracle.dequant_bf16(f["acc"], f["a_s"], f["w_s"])
    assert np.array_equal(out, f["out"])


@pytest.mark.parametrize("layout", ["HND", "NHD"])
def test_sage_quant_and_attention(oracle, layout):
    f = load(f"sage_{layout}")
    q8, qs = oracle.sage_quant(f["q"], 16, layout=layout, block=64)
    k8, ks = oracle.sage_quant(f["k"], 64, layout=layout)
    _close_codes(q8, f["q8"], 1e-3)
    _close_codes(k8, f["k8"], 1e-3)
    assert _ulp_diff(qs, f["qs"]).max() <= 2 and _ulp_diff(ks, f["ks"]).max() <= 2
    from conftest import from_bits

    v = from_bits(f["v"])
    ref = oracle.dequant_attention_reference(
        torch.from_numpy(f["q8"]), torch.from_numpy(f["qs"]), torch.from_numpy(f["k8"]),
        torch.from_numpy(f["ks"]), v, sm_scale=128 ** -0.5, layout=layout)
    got = from_bits(f["out"]).float()
    if layout == "NHD":
        got = got.transpose(1, 2)
    m = oracle.metrics(got, ref)
    assert m["cosine"] >= oracle.NORTH_STAR_COSINE and m["rel_l2"] <= oracle.NORTH_STAR_REL_L2, m
