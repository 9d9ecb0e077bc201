"""CPU checks of the dense W8A8-PV oracle (oracle/oracle.c: orc_k_anchor,
orc_rot_quant, orc_quant_v, orc_w8a8_attn).

Pinned against the reference's own kernels: tests/golden/w8a8_*.npz hold
inputs and outputs of quant_qk_per_warp_int8_rotated[_anchored]_cuda,
quantize_v_int8_sm75 and sol_sparse_online_w8a8_prequantized_attn
(force_dense) run on a B200 (tests/golden/make_golden.py --only w8a8).  The
reference extension is built with --use_fast_math, so its two divides per
tile are approximate: codes may differ by one in a handful of elements,
scales by an ulp; anchors and the attention output (through the oracle's own
quantization of the same inputs) are compared directly.  Property checks
(rotation orthogonality, anchor choice, V round trip, agreement with fp32
attention) need no fixture."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
FIXTURES = sorted(GOLDEN.glob("w8a8_*.npz"))


def _bf16(x: np.ndarray, oracle) -> np.ndarray:
    return oracle.f32_to_bf16(x.astype(np.float32))


def unpermute_v(v8_permuted: np.ndarray) -> np.ndarray:
    """Undo the reference's 16-token fragment permutation of its channel-major
    V codes (quant_v_int8_cuda_sm75.cu:22-26, 137-152): token s is stored at
    (s & ~15) | p(s & 15) with p moving bit 3 to bit 1 and bits 1, 2 to 2, 3."""
    t = np.arange(v8_permuted.shape[-1])
    w = t & 15
    dest = (t & ~15) | (w & 1) | (((w >> 3) & 1) << 1) | (((w >> 1) & 1) << 2) | (((w >> 2) & 1) << 3)
    return v8_permuted[..., dest]


def test_rotation_preserves_dot_products(oracle):
    rng = np.random.default_rng(3)
    for D in (64, 128):
        q = rng.standard_normal((1, 1, 64, D)).astype(np.float32)
        k = rng.standard_normal((1, 1, 64, D)).astype(np.float32)
        qb, kb = _bf16(q, oracle), _bf16(k, oracle)
        q8, qs, k8, ks, anc = oracle.per_warp_int8_hadamard(qb, kb, stabilize_k=False)
        assert anc is None
        qf = q8.astype(np.float32) * np.repeat(qs, 16, axis=2)[..., :64, None]
        kf = k8.astype(np.float32) * np.repeat(ks, 64, axis=2)[..., :64, None]
        exact = oracle.bf16_to_f32(qb)[0, 0] @ oracle.bf16_to_f32(kb)[0, 0].T
        approx = qf[0, 0] @ kf[0, 0].T
        # Orthonormal rotation: only the INT8 rounding separates the two.
        assert np.abs(approx - exact).max() < 0.02 * np.abs(exact).max() + 0.05
        # Not the identity: the codes differ from the unrotated ones.
        q8_plain, _ = oracle.sage_quant(qb, 16, block=64)
        assert (q8_plain != q8).mean() > 0.5


def test_rotation_matches_hadamard_matrix(oracle):
    """Row 0 of the codes equals the quantized H_D diag(sign) x / sqrt(D) built
    from the Sylvester matrix (the butterfly order only moves roundings)."""
    D = 128
    x = np.zeros((1, 1, 16, D), np.float32)
    x[0, 0, 0, 5] = 1.0                     # one basis vector: rotated = +-column / sqrt(D)
    q8, qs = oracle.rot_quant(_bf16(x, oracle), 16, block=64)
    h = np.array([[(-1) ** bin(i & j).count("1") for j in range(D)] for i in range(D)], np.float32)
    signs = [0x1035997B, 0x8087F5EE, 0xEE2E4E1A, 0x71132418]
    s5 = 1.0 if (signs[5 >> 5] >> (5 & 31)) & 1 else -1.0
    want = np.rint(h[:, 5] * s5 / np.sqrt(D) * 127.0 / (1.0 / np.sqrt(D)))
    np.testing.assert_array_equal(q8[0, 0, 0], want.astype(np.int8))


def test_k_anchor_choice(oracle):
    rng = np.random.default_rng(5)
    k_plain = _bf16(rng.standard_normal((1, 2, 300, 128)), oracle)
    assert (oracle.k_anchor(k_plain) == -1).all()        # centring only adds energy
    k_off = _bf16(rng.standard_normal((1, 2, 300, 128)) + rng.standard_normal((1, 2, 1, 128)) * 3,
                  oracle)
    a = oracle.k_anchor(k_off)
    samples = {s * 299 // 8 for s in range(9)}
    assert all(int(v) in samples for v in a.ravel())    # one of the nine sampled rows
    # NHD input gives the same choice.
    assert (oracle.k_anchor(np.ascontiguousarray(k_off.transpose(0, 2, 1, 3)), layout="NHD") == a).all()


def test_quant_v_round_trip(oracle):
    rng = np.random.default_rng(7)
    v = rng.standard_normal((1, 2, 100, 64)).astype(np.float32) * np.linspace(0.1, 3, 64)
    v[0, 1, :, 7] = 0.0                        # all-zero channel: scale floor 1e-12
    vb = _bf16(v, oracle)
    codes, scale = oracle.quant_v(vb)
    assert codes.shape == (1, 2, 64, 128) and scale.shape == (1, 2, 64)
    assert (codes[..., 100:] == 0).all()
    assert scale[0, 1, 7] == np.float32(1e-12)
    vf = oracle.bf16_to_f32(vb)
    rec = codes[..., :100].transpose(0, 1, 3, 2).astype(np.float32) * scale[:, :, None, :]
    assert np.abs(rec - vf).max() <= scale.max() * 0.5 * (1 + 1e-5)
    assert np.abs(codes).max() == 127


def test_w8a8_attention_close_to_fp32(oracle):
    """The u8 P / INT8 V quantization keeps the output within the W8A8
    reference's own error of fp32 attention on the same inputs."""
    rng = np.random.default_rng(11)
    B, H, L, D = 1, 2, 256, 128
    q = _bf16(rng.standard_normal((B, H, L, D)) * 1.5, oracle)
    k = _bf16(rng.standard_normal((B, H, L, D)) + rng.standard_normal((B, H, 1, D)) * 2, oracle)
    v = _bf16(rng.standard_normal((B, H, L, D)), oracle)
    out = oracle.bf16_to_f32(oracle.w8a8attn(q, k, v))
    qt, kt, vt = (torch.from_numpy(oracle.bf16_to_f32(t)) for t in (q, k, v))
    ref = torch.softmax(qt @ kt.transpose(-1, -2) * D ** -0.5, -1) @ vt
    m = oracle.metrics(out, ref.numpy())
    assert m["cosine"] > 0.999 and m["rel_l2"] < 0.05, m
    # Causal: row 0 attends to key 0 only -> its output is V[0] up to codes.
    oc = oracle.bf16_to_f32(oracle.w8a8attn(q, k, v, is_causal=True))
    np.testing.assert_allclose(oc[0, :, 0], oracle.bf16_to_f32(v)[0, :, 0], atol=0.03)


def test_masked_keys_carry_no_mass(oracle):
    """A single key whose anchored K is all zero (k_scale = 1e-7 / 127): the
    output is V itself.  The reference's -5e6 sentinel would give each of the
    63 padded keys p ~ 255 here and return V / 64; masked keys carry no mass
    in this build (identical results whenever c > ~2.6e-5)."""
    rng = np.random.default_rng(13)
    q = _bf16(rng.standard_normal((1, 1, 5, 128)), oracle)
    k = _bf16(rng.standard_normal((1, 1, 1, 128)) + 2.0, oracle)
    v = _bf16(rng.standard_normal((1, 1, 1, 128)), oracle)
    _, _, k8, ks, anc = oracle.per_warp_int8_hadamard(q, k)
    assert anc[0, 0] == 0 and (k8 == 0).all()
    out = oracle.bf16_to_f32(oracle.w8a8attn(q, k, v))
    np.testing.assert_allclose(out[0, 0], np.repeat(oracle.bf16_to_f32(v)[0, 0], 5, 0), rtol=0.02,
                               atol=0.02)


@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: p.stem)
def test_oracle_matches_reference_kernels(oracle, path):
    f = np.load(path)
    fp16, stab, causal = (bool(x) for x in f["meta"])
    q, k, v = f["q"], f["k"], f["v"]
    D = q.shape[-1]
    q8, qs, k8, ks, anc = oracle.per_warp_int8_hadamard(q, k, fp16=fp16, stabilize_k=stab)
    if stab:
        np.testing.assert_array_equal(anc, f["anchors"])
    for got, want in ((q8, f["q8"]), (k8, f["k8"])):
        diff = np.abs(got.astype(np.int32) - want.astype(np.int32))
        assert diff.max() <= 1 and (diff > 0).mean() < 1e-3
    for got, want in ((qs, f["qs"]), (ks, f["ks"])):
        np.testing.assert_allclose(got, want.view(np.float32), rtol=3e-7, atol=0)
    v8, vs = oracle.quant_v(v, fp16=fp16)
    want_v8 = unpermute_v(f["v8_permuted"])
    diff = np.abs(v8.astype(np.int32) - want_v8.astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).mean() < 1e-3
    np.testing.assert_allclose(vs, f["vs"].view(np.float32), rtol=3e-7, atol=0)
    # Attention on the reference's own codes: only the exp2 / reciprocal
    # approximations and the summation order differ.
    o = oracle.w8a8_attn(f["q8"], f["k8"], want_v8, f["vs"].view(np.float32),
                         f["qs"].view(np.float32), f["ks"].view(np.float32), sm_scale=D ** -0.5,
                         is_causal=causal)
    to_f = oracle.f16_to_f32 if fp16 else oracle.bf16_to_f32
    ref = to_f(f["out"])
    m = oracle.metrics(o, ref)
    assert m["cosine"] > 0.99999 and m["rel_l2"] < 5e-3, m


@pytest.mark.parametrize("head_dim", [64, 128])
def test_reference_self_test_inputs(oracle, head_dim):
    """The reference's W8A8 self-test (turing_sage/__init__.py:573-610): integer
    ramps Q [1,4,129,D], K/V [1,2,151,D] in bf16 (GQA 2:1) stay within
    rtol 0.12 / atol 0.09 of fp32 SDPA through the W8A8 arithmetic."""
    qv = torch.arange(4 * 129 * head_dim, dtype=torch.float32)
    kv = torch.arange(2 * 151 * head_dim, dtype=torch.float32)
    q = (((qv % 29) - 14) / 16).reshape(1, 4, 129, head_dim).to(torch.bfloat16)
    k = ((((kv * 3) % 31) - 15) / 16).reshape(1, 2, 151, head_dim).to(torch.bfloat16)
    v = ((((kv * 5) % 37) - 18) / 16).reshape_as(k).to(torch.bfloat16)
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    out = oracle.bf16_to_f32(oracle.w8a8attn(bits(q), bits(k), bits(v)))
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(),
                                                           enable_gqa=True)
    assert torch.allclose(torch.from_numpy(out), ref, rtol=0.12, atol=0.09)
