"""CPU checks of the GEMM / decode / Sage-quant oracle against the reference's
known answers and formulas (validate_compatible.py:78-173, fused.cu:66-200)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_bits

W4A8_CASES = [(7, 13, 64), (3, 16, 12), (1, 8, 16), (17, 72, 80), (33, 128, 128),
              (129, 264, 256), (513, 520, 508), (513, 520, 64)]


@pytest.mark.parametrize("index,case", list(enumerate(W4A8_CASES)))
def test_int8_acc_and_epilogue_match_dequant_matmul(oracle, index, case):
    """validate_compatible.py:78-121 cases: exact INT32 accumulators, epilogue
    within rtol/atol 0.01 of the fp32 dequantize-then-matmul reference."""
    m, n, k = case
    g = torch.Generator().manual_seed(4300 + index)
    a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand((m,), generator=g) * 0.02 + 0.001
    w_s = torch.rand((n,), generator=g) * 0.03 + 0.001
    bias = (torch.randn((n,), generator=g) * 0.1).to(torch.bfloat16) if index % 2 == 0 else None
    acc = oracle.int8_gemm_rows(a.numpy(), w.numpy())
    assert np.array_equal(acc, (a.long() @ w.long().t()).numpy())
    out = oracle.dequant_bf16(acc, a_s.numpy(), w_s.numpy(),
                              None if bias is None else bias.float().numpy())
    ref = oracle.dequant_matmul_reference(a.numpy(), w.numpy(), a_s.numpy(), w_s.numpy(),
                                          None if bias is None else bias.float().numpy())
    torch.testing.assert_close(torch.from_numpy(oracle.bf16_to_f32(out)), ref, rtol=0.01, atol=0.01)


def test_signed_nibble_pack_roundtrip(oracle):
    g = torch.Generator().manual_seed(3)
    w = torch.randint(-8, 8, (24, 64), generator=g, dtype=torch.int8).numpy()
    assert np.array_equal(oracle.unpack_int4(oracle.pack_int4(w), 64), w)


def test_e4m3_table_matches_torch(oracle):
    b = np.arange(256, dtype=np.uint8)
    ref = torch.from_numpy(b).view(torch.float8_e4m3fn).float().numpy()
    got = oracle.e4m3_to_f32(b)
    finite = np.isfinite(ref)
    assert np.array_equal(got[finite], ref[finite])
    assert np.all(np.isnan(got[~finite]))


def test_codebook_decode_known_answer(oracle):
    """validate_compatible.py:123-173 decode formula:
    (codebook[codes] * e4m3(group_scale)).round().clamp(-127, 127)."""
    g = torch.Generator().manual_seed(4388)
    n, k, group = 24, 256, 16
    codes = torch.randint(0, 16, (n, k), generator=g, dtype=torch.int32)
    packed = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).to(torch.uint8).view(torch.int8)
    codebook = torch.linspace(-1.0, 1.0, 16)
    gs = (torch.rand((n, k // group), generator=g) * 64.0 + 4.0).to(torch.float8_e4m3fn)
    want = (codebook[codes.long()] * gs.float().repeat_interleave(group, dim=1)).round().clamp(-127, 127)
    got = oracle.codebook_decode(packed.numpy(), gs.view(torch.uint8).numpy(), codebook.numpy(), group)
    assert np.array_equal(got, want.to(torch.int8).numpy())
    for gsz in (4, 8, 32, 128):
        gs2 = (torch.rand((n, k // gsz), generator=g) * 64.0 + 4.0).to(torch.float8_e4m3fn)
        want2 = (codebook[codes.long()] * gs2.float().repeat_interleave(gsz, dim=1)).round().clamp(-127, 127)
        got2 = oracle.codebook_decode(packed.numpy(), gs2.view(torch.uint8).numpy(), codebook.numpy(), gsz)
        assert np.array_equal(got2, want2.to(torch.int8).numpy())


@pytest.mark.parametrize("layout", ["HND", "NHD"])
def test_sage_quant_scale_layouts(oracle, layout):
    """Scale shapes of the production contract (tests/test_turing_sage_quant.py:
    144-175): q_scale (2,4,12) for L=129, k_scale (2,2,3) for L=151."""
    g = torch.Generator().manual_seed(0)
    q = torch.randn((2, 4, 129, 128), generator=g).to(torch.bfloat16)
    k = torch.randn((2, 2, 151, 128), generator=g).to(torch.bfloat16)
    if layout == "NHD":
        q, k = q.transpose(1, 2).contiguous(), k.transpose(1, 2).contiguous()
    q8, qs = oracle.sage_quant(bf16_bits(q), 16, layout=layout, block=64)
    k8, ks = oracle.sage_quant(bf16_bits(k), 64, layout=layout)
    assert qs.shape == (2, 4, 12) and ks.shape == (2, 2, 3)
    # Empty warp tiles of the padded last block carry the 1e-7 amax floor.
    assert np.all(qs[:, :, 9:] == np.float32(np.float32(1e-7) / np.float32(127.0)))
    assert q8.shape == q.shape and k8.shape == k.shape


def test_sage_quant_formula(oracle):
    g = torch.Generator().manual_seed(5)
    x = torch.randn((1, 2, 100, 64), generator=g).to(torch.bfloat16)
    q8, s = oracle.sage_quant(bf16_bits(x), 64)
    xf = x.float().numpy().reshape(2, 100, 64)
    for h in range(2):
        for t in range(2):
            tile = xf[h, t * 64:(t + 1) * 64]
            amax = np.float32(max(np.float32(1e-7), np.abs(tile).max()))
            assert s[0, h, t] == np.float32(amax / np.float32(127.0))
            inv = np.float32(np.float32(127.0) / amax)
            want = np.clip(np.rint((tile * inv).astype(np.float32)), -128, 127)
            assert np.array_equal(q8[0, h, t * 64:(t + 1) * 64], want.astype(np.int8))


def test_smoothing_is_softmax_invariant(oracle):
    """K mean-smoothing shifts every score of a query row by one constant, so
    the dequantize-then-attention output is unchanged up to quantization."""
    g = torch.Generator().manual_seed(11)
    q = torch.randn((1, 2, 128, 64), generator=g).to(torch.bfloat16)
    k = (torch.randn((1, 2, 192, 64), generator=g) + torch.randn((1, 2, 1, 64), generator=g) * 2.0
         ).to(torch.bfloat16)
    v = torch.randn((1, 2, 192, 64), generator=g).to(torch.bfloat16)
    mean = oracle.token_mean(bf16_bits(k))
    mref = k.double().mean(dim=2).float().to(torch.bfloat16)
    assert np.array_equal(mean, bf16_bits(mref))
    q8, qs = oracle.sage_quant(bf16_bits(q), 16, block=64)
    k8, ks = oracle.sage_quant(bf16_bits(k), 64)
    k8s, kss = oracle.sage_quant(bf16_bits(k), 64, mean_bits=mean)
    sm = 64 ** -0.5
    plain = oracle.dequant_attention_reference(torch.from_numpy(q8), torch.from_numpy(qs),
                                               torch.from_numpy(k8), torch.from_numpy(ks), v,
                                               sm_scale=sm)
    smooth = oracle.dequant_attention_reference(torch.from_numpy(q8), torch.from_numpy(qs),
                                                torch.from_numpy(k8s), torch.from_numpy(kss), v,
                                                sm_scale=sm)
    exact = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), scale=sm)
    for got in (plain, smooth):
        m = oracle.metrics(got, exact)
        assert m["cosine"] >= 0.999 and m["rel_l2"] <= 0.03
    assert kss.max() < ks.max()  # smoothing shrinks the K range
