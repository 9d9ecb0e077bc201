"""GPU parity: tcgen05 INT8 GEMM (through the C ABI) vs the CPU oracle.

Bar: INT32 accumulators bit-exact; the bf16 outputs bit-exact with the
oracle's epilogue (same operation order: (acc * a_s) * w_s, then + bias, one
bf16 rounding) and within the north-star bounds (cosine >= 0.9995, rel-L2 <=
1e-2) of the fp32 dequantize-then-matmul reference."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_bits, make_activation

pytestmark = pytest.mark.gpu

import comfyui_turing_utils_kernel as kernel  # noqa: E402

CASES = [(1, 8, 16), (17, 72, 80), (33, 128, 128), (129, 264, 256), (513, 520, 64),
         (8193, 8, 16), (300, 1000, 496), (256, 512, 4096)]


def _inputs(m, n, k, seed, bias=True):
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand((m,), generator=g) * 0.02 + 0.001
    w_s = torch.rand((n,), generator=g) * 4e-3 + 1e-3
    b = (torch.randn((n,), generator=g) * 0.02).to(torch.bfloat16) if bias else None
    return a, w, a_s, w_s, b


@pytest.mark.parametrize("index,case", list(enumerate(CASES)))
def test_accumulators_bit_exact(oracle, index, case):
    m, n, k = case
    a, w, *_ = _inputs(m, n, k, 4300 + index)
    acc = kernel.turing_int8_gemm_s32(a.cuda(), w.cuda()).cpu().numpy()
    want = oracle.int8_gemm_rows(a.numpy(), w.numpy())
    assert np.array_equal(acc, want)


@pytest.mark.parametrize("index,case", list(enumerate(CASES)))
def test_int8_linear_bit_exact_epilogue(oracle, index, case):
    m, n, k = case
    a, w, a_s, w_s, b = _inputs(m, n, k, 4400 + index, bias=index % 2 == 0)
    out = kernel.turing_int8_linear(a.cuda(), w.cuda(), a_s.cuda(), w_s.cuda(),
                                    None if b is None else b.cuda())
    acc = oracle.int8_gemm_rows(a.numpy(), w.numpy())
    want = oracle.dequant_bf16(acc, a_s.numpy(), w_s.numpy(),
                               None if b is None else b.float().numpy())
    assert np.array_equal(bf16_bits(out), want)


@pytest.mark.parametrize("index,case", list(enumerate(CASES)))
def test_single_cta_form_bit_exact(oracle, monkeypatch, index, case):
    """TB_GEMM_PAIR=0 selects the single-CTA kernel (the default runs CTA
    pairs); its accumulators and epilogue are the oracle's too."""
    monkeypatch.setenv("TB_GEMM_PAIR", "0")
    m, n, k = case
    a, w, a_s, w_s, b = _inputs(m, n, k, 4500 + index, bias=index % 2 == 1)
    acc = kernel.turing_int8_gemm_s32(a.cuda(), w.cuda()).cpu().numpy()
    want_acc = oracle.int8_gemm_rows(a.numpy(), w.numpy())
    assert np.array_equal(acc, want_acc)
    out = kernel.turing_int8_linear(a.cuda(), w.cuda(), a_s.cuda(), w_s.cuda(),
                                    None if b is None else b.cuda())
    want = oracle.dequant_bf16(want_acc, a_s.numpy(), w_s.numpy(),
                               None if b is None else b.float().numpy())
    assert np.array_equal(bf16_bits(out), want)


def test_dequantize_epilogue_bit_exact(oracle):
    g = torch.Generator().manual_seed(2)
    acc = torch.randint(-2 ** 24, 2 ** 24, (37, 80), generator=g, dtype=torch.int32)
    a_s = torch.rand((37,), generator=g) * 0.01
    for w_s in (torch.rand((64,), generator=g) * 0.02, torch.rand((1,), generator=g)):
        out = kernel.turing_dequantize_int8_bf16(acc.cuda(), a_s.cuda(), w_s.cuda(), 64)
        want = oracle.dequant_bf16(acc[:, :64].numpy(), a_s.numpy(), w_s.numpy())
        assert np.array_equal(bf16_bits(out), want)


def test_config1_linear(oracle):
    """BASELINE config 1 end to end: ConvRot INT8 of X [4096, 5120] (0.5% outlier
    channels x20), W8A8 GEMM against W [13824, 5120], per-channel scales, bias."""
    m, k, n = 4096, 5120, 13824
    x = make_activation(m, k, seed=0)
    g = torch.Generator().manual_seed(0)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    w_s = torch.rand((n,), generator=g) * 4e-3 + 1e-3
    bias = (torch.randn((n,), generator=g) * 0.02).to(torch.bfloat16)
    xq, xs = kernel.turing_bf16_int8_convrot_quantize(x.cuda())
    out = kernel.turing_int8_linear(xq, w.cuda(), xs, w_s.cuda(), bias.cuda())
    acc_full = kernel.turing_int8_gemm_s32(xq, w.cuda())
    torch.cuda.synchronize()
    want_q, want_s = oracle.convrot_quantize(bf16_bits(x))
    assert np.array_equal(xq.cpu().numpy(), want_q)
    assert np.array_equal(xs.cpu().numpy(), want_s)
    rows = torch.randperm(m, generator=torch.Generator().manual_seed(3))[:48].numpy()
    want_acc = oracle.int8_gemm_rows(want_q, w.numpy(), rows)
    assert np.array_equal(acc_full.cpu().numpy()[rows], want_acc)
    want_out = oracle.dequant_bf16(want_acc, want_s[rows], w_s.numpy(), bias.float().numpy())
    assert np.array_equal(bf16_bits(out)[rows], want_out)
    ref = oracle.dequant_matmul_reference(want_q[rows], w.numpy(), want_s[rows], w_s.numpy(),
                                          bias.float().numpy())
    met = oracle.metrics(out.cpu()[rows].float(), ref)
    assert met["cosine"] >= oracle.NORTH_STAR_COSINE
    assert met["rel_l2"] <= oracle.NORTH_STAR_REL_L2


@pytest.mark.parametrize("group_size", [16, 128])
def test_codebook_w4a8(oracle, group_size):
    """validate_compatible.py:123-173 contract: exact decode (output == INT8 GEMM
    of the oracle-decoded weight), and rtol 0.01 / atol 0.02 vs dequant-matmul."""
    g = torch.Generator().manual_seed(4388)
    m, n, k = 129, 264, 512
    a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
    codes = torch.randint(0, 16, (n, k), generator=g, dtype=torch.int32)
    packed = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).to(torch.uint8).view(torch.int8)
    codebook = torch.linspace(-1.0, 1.0, 16)
    gs = (torch.rand((n, k // group_size), generator=g) * 64.0 + 4.0).to(torch.float8_e4m3fn)
    a_s = torch.rand((m,), generator=g) * 0.01
    c_s = torch.rand((n,), generator=g) * 0.02
    bias = torch.randn((n,), generator=g).to(torch.bfloat16)
    for chunk in (0, 64):
        out = kernel.turing_codebook_w4a8_linear(a.cuda(), packed.cuda(), a_s.cuda(), gs.cuda(),
                                                 c_s.cuda(), codebook.cuda(), bias.cuda(),
                                                 group_size, chunk)
        w8 = oracle.codebook_decode(packed.numpy(), gs.view(torch.uint8).numpy(), codebook.numpy(),
                                    group_size)
        acc = oracle.int8_gemm_rows(a.numpy(), w8)
        want = oracle.dequant_bf16(acc, a_s.numpy(), c_s.numpy(), bias.float().numpy())
        assert np.array_equal(bf16_bits(out), want)
        ref = oracle.dequant_matmul_reference(a.numpy(), w8, a_s.numpy(), c_s.numpy(),
                                              bias.float().numpy())
        torch.testing.assert_close(out.cpu().float(), ref, rtol=0.01, atol=0.02)


def test_no_watchdog_errors():
    from comfyui_turing_utils_kernel import _lib

    assert _lib.device_error() == 0
