"""CPU oracle of the fused RMSNorm + RoPE + INT8 Q/K prologue
(sage/qk_preprocess.cu) against the reference kernel's own outputs
(tests/golden/qkrope_*.npz, made by tests/golden/make_golden.py on a B200).

The reference extension is built with fast-math: its reciprocal square root
and divides are the hardware approximations, the oracle's are correctly
rounded.  A normalized value therefore differs only where it lands on a
rounding boundary of the 16-bit dtype, so the bar is: codes within one, at
most 0.2 % of them different; scales within 2 ulp."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("qkrope_*.npz"))


def _ulp(a, b):
    return np.abs(a.view(np.int32).astype(np.int64) - b.view(np.int32).astype(np.int64))


def oracle_case(oracle, f):
    rot, split, row, fp16, nhd = (int(v) for v in f["params"])
    layout = "NHD" if nhd else "HND"
    kw = dict(eps=1e-6, rot_dim=rot, layout=layout, norm_scope="row" if row else "head",
              split_half=bool(split), fp16=bool(fp16))
    fr = f["freqs"] if rot else None
    q8, qs = oracle.qk_rms_rope_int8(f["q"], f["qn"], fr, tile_tokens=16, **kw)
    k8, ks = oracle.qk_rms_rope_int8(f["k"], f["kn"], fr, tile_tokens=64, **kw)
    return q8, qs, k8, ks


def test_fixtures_present():
    assert len(CASES) >= 4, CASES


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_kernel(oracle, name):
    f = np.load(GOLDEN / f"{name}.npz")
    q8, qs, k8, ks = oracle_case(oracle, f)
    for got, want in ((q8, f["q8"]), (k8, f["k8"])):
        d = np.abs(got.astype(np.int16) - want.astype(np.int16))
        assert d.max() <= 1, d.max()
        assert (d > 0).mean() <= 2e-3, (d > 0).mean()
    assert _ulp(qs, f["qs"]).max() <= 2 and _ulp(ks, f["ks"]).max() <= 2


def test_identity_rotation_equals_no_rope(oracle):
    """RoPE with cos = 1, sin = 0 leaves the normalized values unchanged."""
    rng = np.random.default_rng(5)
    x = oracle.f32_to_bf16(rng.standard_normal((1, 2, 40, 64)).astype(np.float32))
    w = oracle.f32_to_bf16((rng.random(64) + 0.5).astype(np.float32))
    eye = np.zeros((1, 1, 1, 32, 2, 2), np.float32)
    eye[..., 0, 0] = eye[..., 1, 1] = 1.0
    a = oracle.qk_rms_rope_int8(x, w, oracle.f32_to_bf16(eye), tile_tokens=64, eps=1e-6,
                                rot_dim=64)
    b = oracle.qk_rms_rope_int8(x, w, None, tile_tokens=64, eps=1e-6, rot_dim=0)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_scale_invariance_of_the_norm(oracle):
    """RMSNorm removes a power-of-two gain exactly (eps aside)."""
    rng = np.random.default_rng(6)
    xf = rng.standard_normal((1, 1, 64, 128)).astype(np.float32)
    w = oracle.f32_to_bf16(np.ones(128, np.float32))
    a = oracle.qk_rms_rope_int8(oracle.f32_to_bf16(xf), w, None, tile_tokens=16, eps=0.0,
                                rot_dim=0)
    b = oracle.qk_rms_rope_int8(oracle.f32_to_bf16(xf * 8), w, None, tile_tokens=16, eps=0.0,
                                rot_dim=0)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


ROT_FIXTURES = sorted(GOLDEN.glob("qkrot_*.npz"))


def rotated_case(oracle, f):
    rot, split, row, fp16, nhd, stab = (int(v) for v in f["params"])
    return oracle.qk_rms_rope_rotated_int8(
        f["q"], f["k"], f["qn"], f["kn"], f["freqs"] if rot else None, eps=1e-6, rot_dim=rot,
        layout="NHD" if nhd else "HND", norm_scope="row" if row else "head",
        split_half=bool(split), fp16=bool(fp16), stabilize_k=bool(stab))


@pytest.mark.parametrize("path", ROT_FIXTURES, ids=lambda p: p.stem)
def test_rotated_oracle_matches_reference_kernel(oracle, path):
    """The prologue's Hadamard-rotated form with the K anchor against the
    reference kernel's own outputs (quant_qk_rms_rope_int8_cuda, rotate=True):
    fast-math bar as above; anchors identical."""
    f = np.load(path)
    q8, qs, k8, ks, anchors = rotated_case(oracle, f)
    if int(f["params"][5]):
        np.testing.assert_array_equal(anchors, f["anchors"])
    for got, want in ((q8, f["q8"]), (k8, f["k8"])):
        d = np.abs(got.astype(np.int16) - want.astype(np.int16))
        assert d.max() <= 1 and (d > 0).mean() <= 2e-3, (d.max(), (d > 0).mean())
    assert _ulp(qs, f["qs"]).max() <= 2 and _ulp(ks, f["ks"]).max() <= 2


def test_rotated_prologue_anchor_and_rotation(oracle):
    """Row scope: the anchor the prologue picks from its own nine processed
    samples is the raw-key anchor rule applied to the processed keys; the
    rotation keeps Q.K of the processed values up to the INT8 rounding."""
    rng = np.random.default_rng(21)
    B, H, L, D = 1, 2, 90, 128
    q = oracle.f32_to_bf16(rng.standard_normal((B, H, L, D)).astype(np.float32))
    k = oracle.f32_to_bf16((rng.standard_normal((B, H, L, D))
                            + rng.standard_normal((B, H, 1, D)) * 2).astype(np.float32))
    w = oracle.f32_to_bf16((rng.random(H * D) + 0.5).astype(np.float32))
    ang = rng.random((1, L, 1, D // 2, 1, 1)) * 6.283
    fr = oracle.f32_to_bf16(np.concatenate([np.concatenate([np.cos(ang), -np.sin(ang)], -1),
                                            np.concatenate([np.sin(ang), np.cos(ang)], -1)],
                                           -2).astype(np.float32))
    for rot in (0, D):
        kw = dict(eps=1e-6, rot_dim=rot, norm_scope="row")
        kp = oracle.qk_processed(k, w, fr if rot else None, **kw)
        idx, vals = oracle.qk_anchor_processed(k, w, fr if rot else None, **kw)
        idx2, vals2 = oracle.k_anchor(kp, with_values=True)
        np.testing.assert_array_equal(idx, idx2)
        np.testing.assert_array_equal(vals, vals2)
        if rot == 0:
            assert (idx >= 0).all()   # the common offset survives normalization: centring pays
    kw = dict(eps=1e-6, rot_dim=D, norm_scope="row")
    q8, qs, k8, ks, _ = oracle.qk_rms_rope_rotated_int8(q, k, w, w, fr, stabilize_k=False, **kw)
    qp = oracle.bf16_to_f32(oracle.qk_processed(q, w, fr, **kw))[0, 0]
    kpf = oracle.bf16_to_f32(kp)[0, 0]
    qf = q8[0, 0].astype(np.float32) * np.repeat(qs[0, 0], 16)[:L, None]
    kf = k8[0, 0].astype(np.float32) * np.repeat(ks[0, 0], 64)[:L, None]
    exact = qp @ kpf.T
    assert np.abs(qf @ kf.T - exact).max() < 0.02 * np.abs(exact).max() + 0.05
