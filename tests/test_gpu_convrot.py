"""GPU parity: ConvRot quantizers (sm_100a, through the C ABI) vs the CPU oracle.

Bit-exact bar: INT8 / packed INT4 codes and fp32 scales for the plain
rotation (every size below, including the config-1 and config-4 shapes).
SwiGLU / GELU fused variants call CUDA's expf / tanhf on the GPU while the
oracle calls the C library's; those agree to a few ulp, so the fused variants
allow codes to differ by at most 1 in at most 1e-4 of the elements (the
reference's own GPU-vs-GPU staged/row-buffer check is exact and is ported as
such below)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_bits, make_activation

pytestmark = pytest.mark.gpu

import comfyui_turing_utils_kernel as kernel  # noqa: E402


def _codes_equal_or_close(got, want, frac=1e-4):
    diff = np.abs(got.astype(np.int16) - want.astype(np.int16))
    assert diff.max() <= 1, diff.max()
    assert (diff > 0).mean() <= frac


def _nibbles(packed, hidden, oracle):
    return oracle.unpack_int4(packed, hidden)


@pytest.mark.parametrize("rows,hidden", [(1, 256), (3, 512), (7, 5376), (5, 7168), (2, 14336),
                                         (33, 256), (4096, 5120)])
@pytest.mark.parametrize("int4", [False, True])
def test_rowbuffer_plain_bit_exact(oracle, rows, hidden, int4):
    x = make_activation(rows, hidden, seed=rows * 7 + hidden)
    want_q, want_s = oracle.convrot_quantize(bf16_bits(x), int4=int4)
    fn = kernel.turing_bf16_int4_convrot_quantize if int4 else kernel.turing_bf16_int8_convrot_quantize
    q, s = fn(x.cuda())
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), want_q)
    assert np.array_equal(s.cpu().numpy(), want_s)


def test_config4_down_projection_width(oracle):
    """32760 x 13824 (54 groups per row): check a seeded row sample bit-exact."""
    x = make_activation(32760, 13824, seed=44)
    q, s = kernel.turing_bf16_int4_convrot_quantize(x.cuda())
    rows = torch.randperm(32760, generator=torch.Generator().manual_seed(1))[:64].numpy()
    want_q, want_s = oracle.convrot_quantize(bf16_bits(x[rows]), int4=True)
    assert np.array_equal(q.cpu().numpy()[rows], want_q)
    assert np.array_equal(s.cpu().numpy()[rows], want_s)


@pytest.mark.parametrize("hidden", [256, 5376, 7168, 14336])
@pytest.mark.parametrize("int4", [False, True])
def test_swiglu_staged_equals_rowbuffer_and_oracle(oracle, hidden, int4):
    """Port of validate_compatible.py:43-65 (GPU staged == GPU row-buffer codes
    exactly; scales rtol 1e-6 / atol 5e-8), plus the oracle within +-1."""
    g = torch.Generator().manual_seed(4100 + hidden)
    x = torch.randn((3, hidden * 2), generator=g).to(torch.bfloat16)
    staged = kernel.turing_swiglu_int4_convrot_quantize if int4 else kernel.turing_swiglu_int8_convrot_quantize
    row = kernel.turing_bf16_int4_convrot_quantize if int4 else kernel.turing_bf16_int8_convrot_quantize
    sq, ss = staged(x.cuda(), 256)
    rq, rs = row(x.cuda(), 256, swiglu=True)
    assert torch.equal(sq, rq)
    torch.testing.assert_close(rs, ss, rtol=1e-6, atol=5e-8)
    want_q, want_s = oracle.convrot_quantize(bf16_bits(x), int4=int4, act="swiglu")
    got = rq.cpu().numpy()
    if int4:
        _codes_equal_or_close(_nibbles(got, hidden, oracle), _nibbles(want_q, hidden, oracle))
    else:
        _codes_equal_or_close(got, want_q)
    np.testing.assert_allclose(rs.cpu().numpy(), want_s, rtol=1e-5)


@pytest.mark.parametrize("int4", [False, True])
@pytest.mark.parametrize("staged", [False, True])
def test_gelu_variants(oracle, int4, staged):
    x = make_activation(9, 13824, seed=5)
    if staged:
        fn = kernel.turing_gelu_int4_convrot_quantize if int4 else kernel.turing_gelu_int8_convrot_quantize
    else:
        fn = kernel.turing_bf16_gelu_int4_convrot_quantize if int4 else kernel.turing_bf16_gelu_int8_convrot_quantize
    q, s = fn(x.cuda())
    want_q, want_s = oracle.convrot_quantize(bf16_bits(x), int4=int4, act="gelu", staged=staged)
    got = q.cpu().numpy()
    if int4:
        _codes_equal_or_close(_nibbles(got, 13824, oracle), _nibbles(want_q, 13824, oracle))
    else:
        _codes_equal_or_close(got, want_q)
    np.testing.assert_allclose(s.cpu().numpy(), want_s, rtol=1e-5)


def test_staged_fp16_input(oracle):
    x = make_activation(6, 2 * 1024, seed=9).to(torch.float16)
    q, s = kernel.turing_swiglu_int8_convrot_quantize(x.cuda())
    want_q, want_s = oracle.convrot_quantize(bf16_bits(x), act="swiglu", staged=True, fp16=True)
    _codes_equal_or_close(q.cpu().numpy(), want_q)
    np.testing.assert_allclose(s.cpu().numpy(), want_s, rtol=1e-5)


def test_int4_zero_input_scale_floor():
    zero = torch.zeros((2, 512), device="cuda", dtype=torch.bfloat16)
    for fn in (lambda: kernel.turing_swiglu_int4_convrot_quantize(zero, 256),
               lambda: kernel.turing_bf16_int4_convrot_quantize(zero, 256, swiglu=True)):
        packed, scale = fn()
        assert torch.count_nonzero(packed) == 0
        assert torch.equal(scale, torch.full_like(scale, 1.0e-10))


def test_nonfinite_inputs(oracle):
    bits = np.zeros((3, 512), np.uint16)
    bits[0, 5] = 0x7FC0
    bits[1, :] = 0x7F7F
    bits[2, 300] = 0xFF80  # -inf
    x = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)
    q, s = kernel.turing_bf16_int8_convrot_quantize(x.cuda())
    want_q, want_s = oracle.convrot_quantize(bits)
    assert np.array_equal(q.cpu().numpy(), want_q)
    assert np.array_equal(s.cpu().numpy(), want_s)


def test_no_watchdog_errors():
    from comfyui_turing_utils_kernel import _lib

    assert _lib.device_error() == 0


GOLDEN = __import__("pathlib").Path(__file__).parent / "golden"


def _fixture(name):
    path = GOLDEN / f"{name}.npz"
    if not path.exists():
        pytest.skip(f"golden fixture {name} not present")
    return dict(np.load(path))


@pytest.mark.parametrize("name", ["plain_5120", "plain_256", "edge_512"])
def test_plain_matches_reference_kernel_outputs(name):
    """Codes and scale bits equal the reference kernel's own outputs
    (convrot_quant.cu:350-444 run on a B200 by tests/golden/make_golden.py)."""
    from conftest import from_bits

    f = _fixture(f"convrot_{name}")
    x = from_bits(f["x"]).cuda()
    for int4, tag in ((False, "8"), (True, "4")):
        fn = kernel.turing_bf16_int4_convrot_quantize if int4 else kernel.turing_bf16_int8_convrot_quantize
        q, s = fn(x)
        assert np.array_equal(q.cpu().numpy(), f[f"q{tag}"])
        assert np.array_equal(s.cpu().numpy().reshape(-1).view(np.uint32),
                              f[f"s{tag}"].reshape(-1).view(np.uint32))


@pytest.mark.parametrize("name,act", [("gelu_13824", "gelu"), ("swiglu_5376", "swiglu")])
def test_fused_activation_matches_reference_kernel_outputs(name, act):
    """Row-buffer, staged and staged-fp16 forms with the fused activation:
    codes and scale bits equal the reference kernel's outputs, since both call
    CUDA's expf / tanhf on the same operation tree (convrot_quant.cu:137-291)."""
    from conftest import from_bits

    f = _fixture(f"convrot_{name}")
    x = from_bits(f["x"]).cuda()
    x16 = x.float().to(torch.float16)
    for int4, tag in ((False, "8"), (True, "4")):
        if act == "gelu":
            row = kernel.turing_bf16_gelu_int4_convrot_quantize if int4 else kernel.turing_bf16_gelu_int8_convrot_quantize
            staged = kernel.turing_gelu_int4_convrot_quantize if int4 else kernel.turing_gelu_int8_convrot_quantize
            row_out = row(x)
        else:
            row = kernel.turing_bf16_int4_convrot_quantize if int4 else kernel.turing_bf16_int8_convrot_quantize
            staged = kernel.turing_swiglu_int4_convrot_quantize if int4 else kernel.turing_swiglu_int8_convrot_quantize
            row_out = row(x, 256, swiglu=True)
        for (q, s), key in ((row_out, ""), (staged(x), f"_staged_{tag}"), (staged(x16), f"_staged16_{tag}")):
            qk = f"q{tag}" if key == "" else f"q{key}"
            sk = f"s{tag}" if key == "" else f"s{key}"
            assert np.array_equal(q.cpu().numpy(), f[qk]), (qk, int(np.sum(q.cpu().numpy() != f[qk])))
            assert np.array_equal(s.cpu().numpy().reshape(-1).view(np.uint32),
                                  f[sk].reshape(-1).view(np.uint32)), sk
