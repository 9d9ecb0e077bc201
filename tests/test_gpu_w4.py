"""GPU parity of the 4-bit-weight linears through the C ABI.

* Signed-nibble W4A8 (``turing_w4a8_linear``; reference w4a8.cu:34-72,
  1000-1086, bindings.cpp:167-259): the shape list and input ranges of the
  reference's own check (kernel/scripts/validate_compatible.py:78-121), N and
  K tails included.  The output must equal, bit for bit, the oracle's INT32
  contraction of the unpacked weights followed by the (acc * a_s) * w_s + bias
  epilogue, and it must meet the reference's tolerance (rtol = atol = 0.01)
  against the fp32 dequantize-then-matmul result.  The 17x72x80 fixture holds
  the reference kernel's own output for the same inputs.
* W4A4 (``turing_int4_linear``): packed INT4 activations as the INT4 ConvRot
  quantizers write them, packed INT4 weights; bit-exact against the oracle.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import bf16_bits

pytestmark = pytest.mark.gpu

import comfyui_turing_utils_kernel as kernel  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden"

W4A8_CASES = [(7, 13, 64), (3, 16, 12), (1, 8, 16), (17, 72, 80), (33, 128, 128),
              (129, 264, 256), (513, 520, 508), (513, 520, 64), (8193, 8, 16)]


def _w4a8_inputs(m, n, k, seed, bias):
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand((m,), generator=g) * 0.02 + 0.001
    w_s = torch.rand((n,), generator=g) * 0.03 + 0.001
    b = (torch.randn((n,), generator=g) * 0.1).to(torch.bfloat16) if bias else None
    return a, w, a_s, w_s, b


def _expected(oracle, a, w, a_s, w_s, b):
    acc = oracle.int8_gemm_rows(a.numpy(), w.numpy())
    return oracle.dequant_bf16(acc, a_s.numpy(), w_s.numpy(),
                               None if b is None else b.float().numpy())


@pytest.mark.parametrize("index,case", list(enumerate(W4A8_CASES)))
def test_w4a8_matches_oracle_and_reference_tolerance(oracle, index, case):
    m, n, k = case
    a, w, a_s, w_s, b = _w4a8_inputs(m, n, k, 4300 + index, bias=index % 2 == 0)
    packed = torch.from_numpy(oracle.pack_int4(w.numpy()))
    out = kernel.turing_w4a8_linear(a.cuda(), packed.cuda(), a_s.cuda(), w_s.cuda(),
                                    None if b is None else b.cuda())
    assert out.shape == (m, n) and out.dtype == torch.bfloat16
    assert np.array_equal(bf16_bits(out), _expected(oracle, a, w, a_s, w_s, b))
    ref = oracle.dequant_matmul_reference(a.numpy(), w.numpy(), a_s.numpy(), w_s.numpy(),
                                          None if b is None else b.float().numpy())
    torch.testing.assert_close(out.float().cpu(), ref, rtol=0.01, atol=0.01)


def test_w4a8_reference_kernel_fixture():
    d = np.load(GOLDEN / "w4a8_17x72x80.npz")
    out = kernel.turing_w4a8_linear(torch.from_numpy(d["a"]).cuda(),
                                    torch.from_numpy(d["w_packed"]).cuda(),
                                    torch.from_numpy(d["a_s"]).cuda(),
                                    torch.from_numpy(d["w_s"]).cuda())
    assert np.array_equal(bf16_bits(out), d["out"])


def test_w4a8_custom_op_and_tile_policies(oracle):
    a, w, a_s, w_s, b = _w4a8_inputs(64, 96, 256, 77, bias=True)
    packed = torch.from_numpy(oracle.pack_int4(w.numpy())).cuda()
    want = _expected(oracle, a, w, a_s, w_s, b)
    out = torch.ops.turing_utils.w4a8_linear(a.cuda(), packed, a_s.cuda(), w_s.cuda(), b.cuda())
    assert np.array_equal(bf16_bits(out), want)
    for policy in range(6):
        out = kernel._C.turing_w4a8_linear(a.cuda(), packed, a_s.cuda(), w_s.cuda(), b.cuda(),
                                           tile_policy=policy)
        assert np.array_equal(bf16_bits(out), want)


@pytest.mark.parametrize("case", [(5, 8, 16), (37, 13, 80), (256, 520, 512), (1000, 264, 1024)])
def test_int4_linear_matches_oracle(oracle, case):
    m, n, k = case
    g = torch.Generator().manual_seed(m * 31 + n)
    a = torch.randint(-7, 8, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand((m,), generator=g) * 0.5 + 0.01
    w_s = torch.rand((n,), generator=g) * 0.03 + 0.001
    b = (torch.randn((n,), generator=g) * 0.1).to(torch.bfloat16)
    a_p = torch.from_numpy(oracle.pack_int4(a.numpy()))
    w_p = torch.from_numpy(oracle.pack_int4(w.numpy()))
    out = kernel.turing_int4_linear(a_p.cuda(), w_p.cuda(), a_s.cuda(), w_s.cuda(), b.cuda())
    assert out.shape == (m, n)
    assert np.array_equal(bf16_bits(out), _expected(oracle, a, w, a_s, w_s, b))


def test_int4_linear_on_convrot_int4_codes(oracle):
    """The packed codes and per-token scales straight from the INT4 ConvRot
    quantizer feed the W4A4 linear; the result equals the oracle applied to
    the oracle's own unpacked codes."""
    from conftest import make_activation

    x = make_activation(96, 512, seed=5)
    q, s = kernel.turing_bf16_int4_convrot_quantize(x.cuda())
    g = torch.Generator().manual_seed(6)
    w = torch.randint(-8, 8, (136, 512), generator=g, dtype=torch.int8)
    w_s = torch.rand((136,), generator=g) * 0.01 + 0.001
    out = kernel.turing_int4_linear(q, torch.from_numpy(oracle.pack_int4(w.numpy())).cuda(),
                                    s.reshape(-1), w_s.cuda())
    a = torch.from_numpy(oracle.unpack_int4(q.cpu().numpy(), 512))
    assert np.array_equal(bf16_bits(out), _expected(oracle, a, w, s.reshape(-1).cpu(), w_s, None))


def test_w4_linears_across_weight_chunks(oracle, monkeypatch):
    """A chunk cap far below N x K splits the expanded weight into several
    decode + GEMM rounds (the last one short); W4A8 and W4A4 outputs stay
    bit-exact against the oracle."""
    from comfyui_turing_utils_kernel import _C

    monkeypatch.setattr(_C, "_WEIGHT_CHUNK_BYTES", 300 * 512)
    m, n, k = 130, 1000, 512
    assert _C._weight_chunk_rows(n, k) == 256
    g = torch.Generator().manual_seed(91)
    a = torch.randint(-7, 8, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand((m,), generator=g) * 0.5 + 0.01
    w_s = torch.rand((n,), generator=g) * 0.03 + 0.001
    b = (torch.randn((n,), generator=g) * 0.1).to(torch.bfloat16)
    want = _expected(oracle, a, w, a_s, w_s, b)
    w_p = torch.from_numpy(oracle.pack_int4(w.numpy())).cuda()
    out = kernel.turing_w4a8_linear(a.cuda(), w_p, a_s.cuda(), w_s.cuda(), b.cuda())
    assert np.array_equal(bf16_bits(out), want)
    a_p = torch.from_numpy(oracle.pack_int4(a.numpy())).cuda()
    out = kernel.turing_int4_linear(a_p, w_p, a_s.cuda(), w_s.cuda(), b.cuda())
    assert np.array_equal(bf16_bits(out), want)


def test_no_watchdog_errors():
    from comfyui_turing_utils_kernel import _lib

    assert _lib.device_error() == 0
