"""The float identities the sm_100a kernels rely on for bit-exact results,
checked exhaustively (or on dense grids) in numpy float32 on the CPU.

* Scores: an INT32 score s with |s| < 2^22 becomes the float 1.5 * 2^23 + s by
  an integer add to the bits of 1.5 * 2^23 (sage_attn.cu magic_pair, the Sage
  softmax), and subtracting 1.5 * 2^23 back gives float(s) exactly (the W8A8
  softmax takes float(s) with cvt.rn.f32.s32, exact for |s| < 2^24), so its
  fma(s, c, -m) is the reference's fmaf of the exact score.
* Rounding: v + 1.5 * 2^23 rounds v to the nearest integer, ties to even, for
  |v| < 2^22 (w8a8_quant.cu / convrot.cu code_bits, the W8A8 u8 codes of P),
  i.e. it equals cvt.rni.
* INT8 code -> fp16: the bits 0x6400 | (c ^ 0x80) are the fp16 1024 + (c + 128);
  minus 1152 gives c exactly (w8a8_quant.cu v_codes_kernel).
* u8 saturation: min(p + 1.5 * 2^23, 1.5 * 2^23 + 255) - 1.5 * 2^23 is
  rni_sat_u8(p) for p in [0, 2^22); sage_attn.cu u8_code_pair takes the same
  codes as min(fp16(rni(p)), 255), rni(p) <= 256 being exact in fp16.
* Codebook table lookup: three byte permutes of a 16-byte table map four
  4-bit codes to their bytes (elementwise.cu codebook_decode_lut_kernel).
* PV on the fp16 tensor path: every u8 x s8 product and every sum of 16 of
  them is an integer below 2^24, exact in fp32 and in fp16 operands.
"""
from __future__ import annotations

import numpy as np

MAGIC = np.float32(12582912.0)          # 1.5 * 2^23
MAGIC_BITS = np.uint32(0x4B400000)


def test_score_to_float_through_the_magic_constant():
    s = np.arange(-(1 << 21), 1 << 21, 7, dtype=np.int64)
    s = np.concatenate([s, [-(1 << 22) + 1, (1 << 22) - 1, -127 * 127 * 128, 127 * 127 * 128]])
    bits = (s.astype(np.int64) + int(MAGIC_BITS)).astype(np.uint32)
    t = bits.view(np.float32)
    np.testing.assert_array_equal(t - MAGIC, s.astype(np.float32))


def test_magic_add_is_round_half_even():
    v = np.concatenate([np.arange(-300.0, 300.0, 0.125, dtype=np.float32),
                        np.float32([0.5, 1.5, 2.5, -0.5, -1.5, 126.5, 127.5, 254.5, 255.49998])])
    got = (v + MAGIC) - MAGIC
    np.testing.assert_array_equal(got, np.rint(v).astype(np.float32))
    # The low byte of the sum is the two's-complement INT8 code.
    codes = (v[np.abs(v) <= 127] + MAGIC).view(np.uint32) & 0xFF
    want = np.rint(v[np.abs(v) <= 127]).astype(np.int64) & 0xFF
    np.testing.assert_array_equal(codes.astype(np.int64), want)


def test_int8_code_to_fp16_exactly():
    c = np.arange(-128, 128, dtype=np.int64)
    biased = (0x6400 | ((c & 0xFF) ^ 0x80)).astype(np.uint16).view(np.float16)
    got = biased - np.float16(1152.0)
    np.testing.assert_array_equal(got.astype(np.float64), c.astype(np.float64))


def test_u8_saturating_code():
    p = np.concatenate([np.linspace(0.0, 300.0, 240001, dtype=np.float32),
                        np.float32([255.49998, 255.5, 255.50002, 1e6])])
    r = np.minimum(p + MAGIC, np.float32(12583167.0)) - MAGIC
    want = np.clip(np.rint(p), 0, 255).astype(np.float32)
    np.testing.assert_array_equal(r, want)


def test_pv_partial_sums_are_exact():
    # The largest |u8 x s8| product and the largest 16-term and 64-term sums.
    assert 255 * 128 * 16 < 2 ** 24 and 255 * 128 * 64 < 2 ** 24
    rng = np.random.default_rng(0)
    p = rng.integers(0, 256, size=(1000, 16)).astype(np.float32)
    v = rng.integers(-128, 128, size=(1000, 16)).astype(np.float32)
    exact = (p.astype(np.int64) * v.astype(np.int64)).sum(axis=1)
    acc = np.zeros(1000, np.float32)
    for j in range(16):                 # any order of fp32 adds gives the integer
        acc = acc + p[:, j] * v[:, j]
    np.testing.assert_array_equal(acc.astype(np.int64), exact)
    # Every code is exact in fp16 (an fp16 integer needs <= 11 significant bits).
    assert (np.arange(-128, 256).astype(np.float16).astype(np.int64) == np.arange(-128, 256)).all()


def _exp2_poly(x: np.ndarray) -> np.ndarray:
    """sage_attn.cu exp2_poly_pair restated in float32: clamp at -120,
    n = rint(x) through the 1.5 * 2^23 constant, f = x - n in [-0.5, 0.5],
    2^f by the degree-3 minimax polynomial (Horner with fused multiply-adds,
    emulated in float64 with one float32 rounding each), 2^n added to the
    exponent field."""
    x = np.maximum(x.astype(np.float32), np.float32(-120.0))
    r2 = (x + MAGIC).astype(np.float32)
    f = (x - (r2 - MAGIC).astype(np.float32)).astype(np.float32)

    def fma(a, b, c):
        return (a.astype(np.float64) * b.astype(np.float64) + np.float64(c)).astype(np.float32)

    q = fma(f, np.full_like(f, np.float32(0.0551716685295105)), np.float32(0.2426111251115799))
    q = fma(q, f, np.float32(0.6932609677314758))
    q = fma(q, f, np.float32(0.9999280571937561))
    n_bits = (r2.view(np.uint32).astype(np.uint64) << np.uint64(23)) & np.uint64(0xFFFFFFFF)
    bits = (q.view(np.uint32).astype(np.uint64) + n_bits) & np.uint64(0xFFFFFFFF)
    return bits.astype(np.uint32).view(np.float32)


def test_fma_pipe_exp2_matches_exp2_within_the_p_rounding():
    """The FMA-pipe 2^x that takes one pair of scores in sixteen off the MUFU
    unit: relative error <= 8e-5 on every representable x in [-100, 8] at a
    2^-12 step (the softmax arguments: at most 8 above the reference point),
    far below the 2^-9 rounding of the 16-bit P it feeds."""
    x = np.arange(-100.0, 8.0, 2.0 ** -12, dtype=np.float64).astype(np.float32)
    got = _exp2_poly(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got - want) / want
    assert rel.max() <= 8e-5, rel.max()
    # Below the clamp the result is 2^-120 (0 for every later use of p).
    assert _exp2_poly(np.array([-300.0, -121.0], np.float32)).max() <= np.float32(2.0 ** -119)


def _byte_perm(x, y, s):
    """CUDA __byte_perm: byte i of the result is byte (s >> 4i) & 7 of y:x,
    or that byte's sign replicated when bit 3 of the selector nibble is set."""
    b = [(x >> (8 * i)) & 0xFF for i in range(4)] + [(y >> (8 * i)) & 0xFF for i in range(4)]
    r = 0
    for i in range(4):
        sel = (s >> (4 * i)) & 0xF
        v = b[sel & 7]
        if sel & 8:
            v = 0xFF if v & 0x80 else 0
        r |= v << (8 * i)
    return r


def test_codebook_lut_lookup_by_byte_permutes():
    """codebook_decode_lut_kernel (elementwise.cu) maps four 4-bit codes to
    their decoded bytes with three byte permutes of a 16-byte table: entries
    code & 7 of the low and the high halves, then the high pick where code >= 8.
    Equal to a direct table lookup for random tables and codes."""
    import random

    rng = random.Random(7)
    for _ in range(5000):
        table = [rng.randrange(256) for _ in range(16)]
        lut = [sum(table[4 * j + i] << (8 * i) for i in range(4)) for j in range(4)]
        w = rng.getrandbits(32)
        for part in (w, w >> 16):
            sel = part & 0x7777
            lo = _byte_perm(lut[0], lut[1], sel)
            hi = _byte_perm(lut[2], lut[3], sel)
            got = _byte_perm(lo, hi, 0x3210 | ((part >> 1) & 0x4444))
            want = sum(table[(part >> (4 * i)) & 0xF] << (8 * i) for i in range(4))
            assert got == want
