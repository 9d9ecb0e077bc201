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
