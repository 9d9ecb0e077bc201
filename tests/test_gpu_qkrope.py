"""GPU parity of the fused RMSNorm + RoPE + INT8 Q/K prologue
(``quant_qk_rms_rope_int8_cuda`` / ``turing_utils::qk_rms_rope_int8``)
through the C ABI.

Against the CPU oracle the codes and scales are bit-exact (both use a
correctly rounded reciprocal square root and IEEE divides, and the kernel
sums squares in the reference's order).  Against the reference kernel's own
outputs (tests/golden/qkrope_*.npz) the bar is the fast-math one: codes
within one (at most 0.2 % different), scales within 2 ulp.  Cases: both
layouts and dtypes, head dims 64/128, head and row norm scope, interleaved
and split-half RoPE, partial and no rotation, batch / sequence broadcast
frequencies, GQA head counts, different Q/K lengths, ragged tails, strided
(fused QKV) inputs, and the prequantize -> attention route."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import bf16_bits, from_bits
from test_oracle_qkrope import oracle_case

pytestmark = pytest.mark.gpu

import comfyui_turing_utils_kernel  # noqa: E402,F401
from comfyui_turing_utils_kernel import turing_sage  # noqa: E402
from comfyui_turing_utils_kernel.turing_sage import quant  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden"


def _freqs(fb, fs, pairs, seed, dt):
    g = torch.Generator().manual_seed(seed)
    ang = torch.rand((fb, fs, 1, pairs, 1, 1), generator=g) * 6.283
    c, s = torch.cos(ang), torch.sin(ang)
    return torch.cat([torch.cat([c, -s], -1), torch.cat([s, c], -1)], -2).to(dt)


def _run(q, k, qn, kn, fr, *, rot, layout, scope, split):
    return quant.rms_rope_per_warp_int8(q.cuda(), k.cuda(), qn.cuda(), kn.cuda(),
                                        None if fr is None else fr.cuda(), epsilon=1e-6,
                                        rot_dim=rot, tensor_layout=layout, norm_scope=scope,
                                        split_half=split, rotate_qk=False, stabilize_k=False)


def _oracle(oracle, q, k, qn, kn, fr, *, rot, layout, scope, split):
    fp16 = q.dtype == torch.float16
    kw = dict(eps=1e-6, rot_dim=rot, layout=layout, norm_scope=scope, split_half=split,
              fp16=fp16)
    fb = None if fr is None else bf16_bits(fr)
    q8, qs = oracle.qk_rms_rope_int8(bf16_bits(q), bf16_bits(qn), fb, tile_tokens=16, **kw)
    k8, ks = oracle.qk_rms_rope_int8(bf16_bits(k), bf16_bits(kn), fb, tile_tokens=64, **kw)
    return q8, qs, k8, ks


def _exact(got, want):
    for g, w in zip(got, want):
        g = g.cpu().numpy()
        assert g.shape == w.shape and g.dtype == w.dtype
        assert np.array_equal(g.view(np.uint8) if g.dtype == np.int8 else g.view(np.uint32),
                              w.view(np.uint8) if w.dtype == np.int8 else w.view(np.uint32))


CASES = [
    # dt, layout, B, hq, hk, lq, lk, D, scope, split, rot, fb, fs
    (torch.bfloat16, "HND", 2, 3, 3, 129, 129, 128, "head", False, 128, 1, 129),
    (torch.float16, "HND", 1, 4, 2, 64, 64, 128, "head", True, 128, 1, 64),
    (torch.bfloat16, "NHD", 2, 2, 2, 33, 33, 64, "head", False, 64, 2, 33),
    (torch.float16, "NHD", 1, 6, 3, 200, 200, 64, "row", True, 48, 1, 1),
    (torch.bfloat16, "HND", 1, 5, 5, 17, 300, 128, "row", False, 0, 1, 1),
    (torch.bfloat16, "NHD", 3, 2, 1, 1, 1, 128, "head", True, 64, 3, 1),
    (torch.float16, "HND", 1, 2, 2, 1000, 1000, 128, "row", False, 128, 1, 1000),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c[1:])))
def test_bit_exact_against_oracle(oracle, case):
    dt, layout, B, hq, hk, lq, lk, D, scope, split, rot, fb, fs = case
    g = torch.Generator().manual_seed(lq * 7 + hq + D)
    qs_ = (B, hq, lq, D) if layout == "HND" else (B, lq, hq, D)
    ks_ = (B, hk, lk, D) if layout == "HND" else (B, lk, hk, D)
    q = (torch.randn(qs_, generator=g) * 2 + 0.3).to(dt)
    k = (torch.randn(ks_, generator=g) * 0.7).to(dt)
    qn = (torch.rand((D if scope == "head" else hq * D,), generator=g) + 0.5).to(dt)
    kn = (torch.rand((D if scope == "head" else hk * D,), generator=g) + 0.5).to(dt)
    fr = _freqs(fb, fs, rot // 2, lq, dt) if rot else None
    kw = dict(rot=rot, layout=layout, scope=scope, split=split)
    _exact(_run(q, k, qn, kn, fr, **kw), _oracle(oracle, q, k, qn, kn, fr, **kw))


@pytest.mark.parametrize("scope", ["head", "row"])
def test_nan_zero_and_large_tokens(oracle, scope):
    """A NaN element poisons its token's RMS (its codes become -127, as the
    reference's clamp of NaN gives) without touching the tile's scale; an
    all-zero token quantizes to zeros; large magnitudes normalize away."""
    g = torch.Generator().manual_seed(33)
    q = (torch.randn((1, 2, 80, 128), generator=g)).to(torch.bfloat16)
    k = (torch.randn((1, 2, 80, 128), generator=g) * 3e4).to(torch.bfloat16)
    q[0, 1, 5, 17] = float("nan")
    q[0, 0, 9] = 0.0
    k[0, 0, 70, 3] = float("nan")
    n = 128 if scope == "head" else 256
    qn = (torch.rand((n,), generator=g) + 0.5).to(torch.bfloat16)
    kn = (torch.rand((n,), generator=g) + 0.5).to(torch.bfloat16)
    fr = _freqs(1, 80, 64, 34, torch.bfloat16)
    kw = dict(rot=128, layout="HND", scope=scope, split=False)
    got = _run(q, k, qn, kn, fr, **kw)
    want = _oracle(oracle, q, k, qn, kn, fr, **kw)
    _exact(got, want)
    if scope == "head":
        assert (got[0][0, 1, 5].cpu() == -127).all() and (got[0][0, 0, 9].cpu() == 0).all()


def test_strided_fused_qkv_views(oracle):
    """Q and K as head slices of one [B, L, 3, H, D] projection buffer."""
    g = torch.Generator().manual_seed(11)
    qkv = torch.randn((2, 90, 3, 4, 128), generator=g).to(torch.bfloat16)
    q, k = qkv[:, :, 0], qkv[:, :, 1]          # NHD views, token stride 3*4*128
    qn = (torch.rand((128,), generator=g) + 0.5).to(torch.bfloat16)
    kn = (torch.rand((128,), generator=g) + 0.5).to(torch.bfloat16)
    fr = _freqs(1, 90, 64, 12, torch.bfloat16)
    kw = dict(rot=128, layout="NHD", scope="head", split=False)
    got = quant.rms_rope_per_warp_int8(qkv.cuda()[:, :, 0], qkv.cuda()[:, :, 1], qn.cuda(),
                                       kn.cuda(), fr.cuda(), epsilon=1e-6, rot_dim=128,
                                       tensor_layout="NHD", norm_scope="head", split_half=False,
                                       rotate_qk=False, stabilize_k=False)
    _exact(got, _oracle(oracle, q.contiguous(), k.contiguous(), qn, kn, fr, **kw))


@pytest.mark.parametrize("name", sorted(p.stem for p in GOLDEN.glob("qkrope_*.npz")))
def test_matches_reference_kernel(oracle, name):
    f = np.load(GOLDEN / f"{name}.npz")
    rot, split, row, fp16, nhd = (int(v) for v in f["params"])
    dt = torch.float16 if fp16 else torch.bfloat16
    q, k, qn, kn = (from_bits(f[n], dt) for n in ("q", "k", "qn", "kn"))
    fr = from_bits(f["freqs"], dt) if rot else None
    got = _run(q, k, qn, kn, fr, rot=rot, layout="NHD" if nhd else "HND",
               scope="row" if row else "head", split=bool(split))
    for g, w in ((got[0], f["q8"]), (got[2], f["k8"])):
        d = np.abs(g.cpu().numpy().astype(np.int16) - w.astype(np.int16))
        assert d.max() <= 1 and (d > 0).mean() <= 2e-3, (d.max(), (d > 0).mean())
    for g, w in ((got[1], f["qs"]), (got[3], f["ks"])):
        u = np.abs(g.cpu().numpy().view(np.int32).astype(np.int64) -
                   w.view(np.int32).astype(np.int64))
        assert u.max() <= 2, u.max()
    _exact(got, oracle_case(oracle, f))


def test_custom_op_and_prequantized_attention(oracle):
    """prequantize_rms_rope_qk -> prequantize_sageattn_from_qk -> attention
    equals the dequantize-then-attention reference on the same codes."""
    g = torch.Generator().manual_seed(21)
    B, H, L, D = 1, 2, 256, 64
    q = torch.randn((B, H, L, D), generator=g).to(torch.bfloat16).cuda()
    k = torch.randn((B, H, L, D), generator=g).to(torch.bfloat16).cuda()
    v = torch.randn((B, H, L, D), generator=g).to(torch.bfloat16).cuda()
    qn = (torch.rand((D,), generator=g) + 0.5).to(torch.bfloat16)
    kn = (torch.rand((D,), generator=g) + 0.5).to(torch.bfloat16)
    fr = _freqs(1, L, 32, 22, torch.bfloat16)
    assert turing_sage.fused_qk_preprocessing_available()
    qk = turing_sage.prequantize_rms_rope_qk(q, k, qn, kn, fr, epsilon=1e-6, rot_dim=64)
    op = torch.ops.turing_utils.qk_rms_rope_int8(q, k, qn.cuda(), kn.cuda(), fr.cuda(), 1e-6, 64,
                                                 "HND", "head", False, False, False)
    for a, b in zip((qk.query_int8, qk.query_scale, qk.key_int8, qk.key_scale), op):
        assert torch.equal(a, b)
    pre = turing_sage.prequantize_sageattn_from_qk(qk, v)
    out = turing_sage.sageattn_from_prequantized(pre)
    assert out.shape == (B, H, L, D)
    want = oracle.dequant_attention_reference(qk.query_int8.cpu(), qk.query_scale.cpu(),
                                              qk.key_int8.cpu(), qk.key_scale.cpu(), v.cpu(),
                                              sm_scale=D ** -0.5)
    m = oracle.metrics(out.float().cpu(), want)
    assert m["cosine"] >= oracle.NORTH_STAR_COSINE and m["rel_l2"] <= oracle.NORTH_STAR_REL_L2, m


def test_rejections():
    q = torch.randn((1, 1, 64, 128), device="cuda", dtype=torch.bfloat16)
    w = torch.ones(128, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="head_dim 64 or 128"):
        turing_sage.prequantize_rms_rope_qk(q[..., :96], q[..., :96], w[:96], w[:96], None,
                                            epsilon=1e-6, rot_dim=0)
    with pytest.raises(RuntimeError, match="rot_dim must be even"):
        quant.rms_rope_per_warp_int8(q, q, w, w, None, epsilon=1e-6, rot_dim=3,
                                     tensor_layout="HND", norm_scope="head", split_half=False,
                                     rotate_qk=False, stabilize_k=False)


def test_no_watchdog_errors():
    from comfyui_turing_utils_kernel import _lib

    assert _lib.device_error() == 0


@pytest.mark.parametrize("layout,D", [("HND", 128), ("NHD", 64)])
def test_row_sum_squares_and_given_rrms_match_row_scope(layout, D):
    """The tensor-parallel route: per-token sums of squares over the heads
    (tb_row_sum_squares, the row pass's reduction order), RRMS formed on the
    host as the correctly rounded 1/sqrt(sum / (H*D) + eps), then the prologue
    with that RRMS (norm_scope 2) — the same codes and scales as the row-scope
    prologue that computes its own RRMS."""
    g = torch.Generator().manual_seed(D + len(layout))
    H, L = 5, 150
    shape = (2, H, L, D) if layout == "HND" else (2, L, H, D)
    q = (torch.randn(shape, generator=g) * 1.3).to(torch.bfloat16).cuda()
    k = (torch.randn(shape, generator=g) * 0.9).to(torch.bfloat16).cuda()
    wq = (torch.rand((H * D,), generator=g) + 0.5).to(torch.bfloat16).cuda()
    wk = (torch.rand((H * D,), generator=g) + 0.5).to(torch.bfloat16).cuda()
    fr = _freqs(1, L, D // 2, 7, torch.bfloat16).cuda()
    kw = dict(epsilon=1e-6, rot_dim=D, tensor_layout=layout, norm_scope="row", split_half=False,
              rotate_qk=False, stabilize_k=False)
    own = quant.rms_rope_per_warp_int8(q, k, wq, wk, fr, **kw)

    def rrms(t):
        s = quant.row_sum_squares(t, tensor_layout=layout).cpu().numpy()
        x = (s / np.float32(H * D)).astype(np.float32) + np.float32(1e-6)
        return torch.from_numpy((1.0 / np.sqrt(x.astype(np.float64))).astype(np.float32)).cuda()

    given = quant.rms_rope_per_warp_int8(q, k, wq, wk, fr, query_rrms=rrms(q), key_rrms=rrms(k),
                                         **kw)
    for a, b in zip(own, given):
        assert torch.equal(a, b)


ROT_CASES = [
    # dt, layout, B, hq, hk, lq, lk, D, scope, split, rot, fb, fs, stabilize, K offset
    (torch.bfloat16, "HND", 1, 2, 2, 150, 150, 128, "row", False, 128, 1, 150, True, 2.0),
    (torch.float16, "NHD", 2, 3, 1, 70, 90, 64, "head", True, 48, 1, 1, True, 1.5),
    (torch.bfloat16, "HND", 1, 2, 2, 100, 100, 128, "head", False, 0, 1, 1, True, 3.0),
    (torch.bfloat16, "NHD", 1, 4, 2, 33, 129, 128, "row", True, 128, 1, 1, False, 0.0),
    (torch.float16, "HND", 2, 1, 1, 1, 1, 64, "head", False, 64, 2, 1, True, 0.0),
]


def _rot_inputs(case, seed):
    dt, layout, B, hq, hk, lq, lk, D, scope, split, rot, fb, fs, stab, off = case
    g = torch.Generator().manual_seed(seed)
    qs_ = (B, hq, lq, D) if layout == "HND" else (B, lq, hq, D)
    ks_ = (B, hk, lk, D) if layout == "HND" else (B, lk, hk, D)
    os_ = (1, hk, 1, D) if layout == "HND" else (1, 1, hk, D)
    q = (torch.randn(qs_, generator=g) * 1.5 + 0.2).to(dt)
    k = (torch.randn(ks_, generator=g) + torch.randn(os_, generator=g) * off).to(dt)
    qn = (torch.rand((D if scope == "head" else hq * D,), generator=g) + 0.5).to(dt)
    kn = (torch.rand((D if scope == "head" else hk * D,), generator=g) + 0.5).to(dt)
    fr = _freqs(fb, fs, rot // 2, seed + 1, dt) if rot else None
    return q, k, qn, kn, fr


@pytest.mark.parametrize("case", ROT_CASES, ids=lambda c: "-".join(map(str, c[1:])))
def test_rotated_prologue_bit_exact_against_oracle(oracle, case):
    """rotate_qk (+ stabilize_k): normalized + rotated values written once,
    the K anchor from nine processed samples, then the randomized-Hadamard
    quantizer — codes and scales equal the oracle's (qk_preprocess.cu:252-753)."""
    dt, layout, B, hq, hk, lq, lk, D, scope, split, rot, fb, fs, stab, off = case
    q, k, qn, kn, fr = _rot_inputs(case, seed=lq * 5 + hk + D)
    got = quant.rms_rope_per_warp_int8(q.cuda(), k.cuda(), qn.cuda(), kn.cuda(),
                                       None if fr is None else fr.cuda(), epsilon=1e-6,
                                       rot_dim=rot, tensor_layout=layout, norm_scope=scope,
                                       split_half=split, rotate_qk=True, stabilize_k=stab)
    want = oracle.qk_rms_rope_rotated_int8(
        bf16_bits(q), bf16_bits(k), bf16_bits(qn), bf16_bits(kn),
        None if fr is None else bf16_bits(fr), eps=1e-6, rot_dim=rot, layout=layout,
        norm_scope=scope, split_half=split, fp16=dt == torch.float16, stabilize_k=stab)
    _exact(got, want[:4])


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("qkrot_*.npz")), ids=lambda p: p.stem)
def test_rotated_prologue_matches_reference_kernel(oracle, path):
    f = np.load(path)
    rot, split, row, fp16, nhd, stab = (int(v) for v in f["params"])
    dt = torch.float16 if fp16 else torch.bfloat16
    q, k, qn, kn = (from_bits(f[n], dt).cuda() for n in ("q", "k", "qn", "kn"))
    fr = from_bits(f["freqs"], dt).cuda() if rot else None
    got = quant.rms_rope_per_warp_int8(q, k, qn, kn, fr, epsilon=1e-6, rot_dim=rot,
                                       tensor_layout="NHD" if nhd else "HND",
                                       norm_scope="row" if row else "head",
                                       split_half=bool(split), rotate_qk=True,
                                       stabilize_k=bool(stab))
    for g, w in ((got[0], f["q8"]), (got[2], f["k8"])):
        d = np.abs(g.cpu().numpy().astype(np.int16) - w.astype(np.int16))
        assert d.max() <= 1 and (d > 0).mean() <= 2e-3, (d.max(), (d > 0).mean())


def test_rotated_prologue_feeds_w8a8(oracle):
    """prequantize_rms_rope_qk(rotate_qk, stabilize_k) ->
    prequantize_sol_sageattn_from_qk(use_w8a8, force_dense) ->
    sol_sparse_sageattn_from_prequantized, the plugin's W8A8 route with the
    fused prologue (attention/stable.py:388-460, 501-518): the output equals the
    oracle's W8A8 attention on the oracle's codes."""
    case = (torch.bfloat16, "HND", 1, 2, 2, 200, 200, 128, "row", False, 128, 1, 200, True, 2.0)
    q, k, qn, kn, fr = _rot_inputs(case, seed=77)
    v = torch.randn((1, 2, 200, 128), generator=torch.Generator().manual_seed(78)).to(torch.bfloat16)
    qk = turing_sage.prequantize_rms_rope_qk(q.cuda(), k.cuda(), qn.cuda(), kn.cuda(), fr.cuda(),
                                            epsilon=1e-6, rot_dim=128, norm_scope="row",
                                            rotate_qk=True, stabilize_k=True)
    assert qk.route_original_basis
    pre = turing_sage.prequantize_sol_sageattn_from_qk(qk, v.cuda(), use_w8a8=True,
                                                       force_dense=True)
    out = turing_sage.sol_sparse_sageattn_from_prequantized(pre)
    q8, qs, k8, ks, _ = oracle.qk_rms_rope_rotated_int8(
        bf16_bits(q), bf16_bits(k), bf16_bits(qn), bf16_bits(kn), bf16_bits(fr), eps=1e-6,
        rot_dim=128, norm_scope="row", stabilize_k=True)
    v8, vs = oracle.quant_v(bf16_bits(v))
    want = oracle.w8a8_attn(q8, k8, v8, vs, qs, ks, sm_scale=128 ** -0.5)
    m = oracle.metrics(out.float().cpu().numpy(), want)
    assert m["cosine"] >= 0.99999 and m["rel_l2"] <= 5e-3, m
