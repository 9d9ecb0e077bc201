"""CPU checks of the ConvRot oracle against the reference's own known answers
(kernel/scripts/validate_compatible.py:43-76) and against the mathematics of
the transform (convrot_quant.cu:104-116, 350-444)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_bits, make_activation


def test_rotation_is_the_kron_hadamard(oracle):
    h = oracle.hadamard256_matrix()
    assert np.allclose(h @ h.T, np.eye(256))
    assert np.allclose(h, h.T)
    x = make_activation(4, 512, seed=1)
    rot_bits, gmax = oracle.convrot_rotate_bf16(bf16_bits(x))
    xf = x.float().numpy().astype(np.float64)
    exact = np.concatenate([xf[:, g * 256:(g + 1) * 256] @ h.T for g in range(2)], axis=1)
    got = oracle.bf16_to_f32(rot_bits).astype(np.float64)
    # bf16 storage: within one bf16 ulp of the exact rotation
    assert np.all(np.abs(got - exact) <= np.abs(exact) * 2.0 ** -8 + 1e-30)
    np.testing.assert_allclose(gmax, np.abs(exact.reshape(4, 2, 256)).max(-1), rtol=1e-5)


@pytest.mark.parametrize("hidden", [256, 5376, 7168, 14336])
def test_staged_equals_rowbuffer(oracle, hidden):
    """Port of validate_compatible.py:43-65: staged == row-buffer codes exactly,
    scales within rtol 1e-6 / atol 5e-8 (SwiGLU input, INT8 and INT4)."""
    g = torch.Generator().manual_seed(4100 + hidden)
    x = torch.randn((3, hidden * 2), generator=g).to(torch.bfloat16)
    for int4 in (False, True):
        sq, ss = oracle.convrot_quantize(bf16_bits(x), int4=int4, act="swiglu", staged=True)
        rq, rs = oracle.convrot_quantize(bf16_bits(x), int4=int4, act="swiglu", staged=False)
        assert np.array_equal(sq, rq)
        np.testing.assert_allclose(rs, ss, rtol=1e-6, atol=5e-8)
        if int4:
            u = oracle.unpack_int4(rq, hidden)
            assert u.min() >= -7 and u.max() <= 7


def test_int4_zero_input_scale_floor(oracle):
    """validate_compatible.py:67-76: zero input -> zero codes, scale exactly 1e-10."""
    zero = np.zeros((2, 512), np.uint16)
    for staged in (False, True):
        packed, scale = oracle.convrot_quantize(zero, int4=True, act="swiglu", staged=staged)
        assert not np.any(oracle.unpack_int4(packed, 256))
        assert np.all(scale == np.float32(1.0e-10))
    q, s = oracle.convrot_quantize(np.zeros((2, 256), np.uint16))
    assert not np.any(q) and np.all(s == np.float32(1.0e-30))


def test_int8_codes_follow_the_scale(oracle):
    x = make_activation(16, 5120, seed=7)
    q, s = oracle.convrot_quantize(bf16_bits(x))
    rot, _ = oracle.convrot_rotate_bf16(bf16_bits(x))
    r = oracle.bf16_to_f32(rot)
    amax = np.abs(r).max(1, keepdims=True)
    # scale from the fp32 absmax: within a bf16 ulp of the bf16 absmax / 127
    np.testing.assert_allclose(s, amax / 127.0, rtol=2 ** -7)
    rs = oracle.bf16_to_f32(oracle.f32_to_bf16(s))
    approx = r / rs
    assert np.max(np.abs(q - approx)) <= 0.5 + 128 * 2 ** -8
    assert q.max() <= 127 and q.min() >= -128


def test_nonfinite_and_huge_inputs(oracle):
    x = np.zeros((3, 256), np.uint16)
    x[0, 5] = 0x7FC0  # NaN: the whole group rotates to NaN -> code -128
    x[1, :] = 0x7F7F  # bf16 max: absmax clipped to the bf16 finite max
    x[2, 3] = 0x3F80  # 1.0
    q, s = oracle.convrot_quantize(x)
    assert np.all(q[0] == -128)
    assert np.isfinite(s[1, 0])
    assert q[2].max() <= 127
