"""GPU parity of the dense W8A8-PV attention path through the C ABI:
randomized-Hadamard Q/K INT8 (``quant_qk_per_warp_int8_rotated[_anchored]_cuda``),
channel-wise INT8 V (``quantize_v_int8_sm75``), the W8A8 attention
(``sol_sparse_online_w8a8_prequantized_attn`` force_dense) and the public
``w8a8attn`` / ``turing_utils::w8a8_attention``.

Against the CPU oracle the codes, scales and anchors are bit-exact.  The
attention output on identical codes agrees with the oracle's fp32 result to
cosine >= 0.99999 and relative L2 <= 5e-3: the u8 codes of P are the same
except where 2^x lands within an ulp of a rounding tie (MUFU ex2 against the C
library's exp2f), and the fp32 sums run in another order.  Masked keys carry
no mass in either (the reference's -5e6 sentinel differs only for degenerate
scales; the single-key case below is one).  The error against
fp32 attention is the W8A8 algorithm's own, so it is checked against the
oracle's error of the same inputs.  Against the reference kernel's outputs
(tests/golden/w8a8_*.npz) the fast-math bar of the other quantizers applies.
Cases: both dtypes and layouts, head dims 64/128, anchored and plain K, GQA,
different Q/K lengths with ragged tails, causal, strided V, NaN/inf V, and
sampled rows of the configs[1] shape."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import bf16_bits, from_bits
from test_oracle_w8a8 import unpermute_v

pytestmark = pytest.mark.gpu

import comfyui_turing_utils_kernel  # noqa: E402,F401
from comfyui_turing_utils_kernel import _lib, _sage_qattn_sm75 as qattn, turing_sage  # noqa: E402
from comfyui_turing_utils_kernel.turing_sage import core, quant  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden"


def _inputs(B, hq, hk, lq, lk, D, dt, seed, offset=2.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn((B, hq, lq, D), generator=g) * 1.5).to(dt)
    k = (torch.randn((B, hk, lk, D), generator=g)
         + torch.randn((B, hk, 1, D), generator=g) * offset).to(dt)
    v = torch.randn((B, hk, lk, D), generator=g).to(dt)
    return q, k, v


def _metrics(got, want):
    g = np.asarray(got, np.float64).ravel()
    w = np.asarray(want, np.float64).ravel()
    return {"cos": float(g @ w / (np.linalg.norm(g) * np.linalg.norm(w) + 1e-30)),
            "rel": float(np.linalg.norm(g - w) / (np.linalg.norm(w) + 1e-30))}


QK_CASES = [  # dtype, layout, B, hq, hk, lq, lk, D, stabilize, K offset
    (torch.bfloat16, "HND", 1, 2, 2, 200, 200, 128, True, 2.0),
    (torch.bfloat16, "NHD", 2, 4, 2, 77, 130, 128, True, 3.0),
    (torch.float16, "HND", 1, 3, 1, 64, 65, 64, False, 0.0),
    (torch.float16, "NHD", 1, 2, 2, 300, 17, 64, True, 1.0),
    (torch.bfloat16, "HND", 1, 1, 1, 1, 1, 128, True, 0.0),
    (torch.bfloat16, "HND", 1, 2, 2, 129, 250, 128, True, 0.0),   # no offset: anchor -1
]


@pytest.mark.parametrize("case", QK_CASES, ids=lambda c: "-".join(map(str, c[1:])))
def test_rotated_quant_bit_exact(oracle, case):
    dt, layout, B, hq, hk, lq, lk, D, stab, off = case
    q, k, _ = _inputs(B, hq, hk, lq, lk, D, dt, seed=lq * 3 + lk + D, offset=off)
    if layout == "NHD":
        q, k = (t.transpose(1, 2).contiguous() for t in (q, k))
    got = quant.per_warp_int8_hadamard(q.cuda(), k.cuda(), tensor_layout=layout,
                                       stabilize_k=stab)
    want = oracle.per_warp_int8_hadamard(bf16_bits(q), bf16_bits(k), layout=layout,
                                         fp16=dt == torch.float16, stabilize_k=stab)
    for g, w in zip(got, want[:4]):
        np.testing.assert_array_equal(g.cpu().numpy(), w)
    if stab:
        a = torch.empty((B, hk), dtype=torch.int32, device="cuda")
        from comfyui_turing_utils_kernel import _sage_fused_sm75 as fused
        qo, ko = torch.empty_like(q, dtype=torch.int8, device="cuda"), \
            torch.empty_like(k, dtype=torch.int8, device="cuda")
        qs, ks = (torch.empty_like(t) for t in got[1::2])
        fused.quant_qk_per_warp_int8_rotated_anchored_cuda(
            q.cuda(), k.cuda(), qo, ko, qs, ks, a, 64, 16, 64, 0 if layout == "NHD" else 1)
        np.testing.assert_array_equal(a.cpu().numpy(), want[4])
        if off == 0.0:
            assert (want[4] == -1).all() or lk < 3


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D,L", [(128, 300), (64, 64), (128, 1)])
def test_quantize_v_bit_exact(oracle, dt, D, L):
    g = torch.Generator().manual_seed(D + L)
    v = (torch.randn((2, 3, L, D), generator=g) * torch.linspace(0.05, 4, D)).to(dt)
    if L > 10:
        v[0, 1, 3, 5] = float("nan")
        v[1, 2, :, 9] = 0.0
    want_codes, want_scale = oracle.quant_v(bf16_bits(v), fp16=dt == torch.float16)
    vd = v.cuda()
    lpad = (L + 63) // 64 * 64
    codes = torch.full((2, 3, D, lpad), 99, dtype=torch.int8, device="cuda")
    scale = torch.empty((2, 3, D), dtype=torch.float32, device="cuda")
    qattn.quantize_v_int8_sm75(vd, codes, scale)
    np.testing.assert_array_equal(codes.cpu().numpy(), want_codes)
    np.testing.assert_array_equal(scale.cpu().numpy(), want_scale)
    f16 = torch.empty((2, 3, L, D), dtype=torch.float16, device="cuda")
    scale2 = torch.empty_like(scale)
    qattn.quantize_v_codes(vd, f16, scale2)
    np.testing.assert_array_equal(f16.float().cpu().numpy(),
                                  want_codes[..., :L].transpose(0, 1, 3, 2).astype(np.float32))
    np.testing.assert_array_equal(scale2.cpu().numpy(), want_scale)
    # Strided V (a slice of a fused buffer, NHD-like strides) gives the same codes.
    big = torch.zeros((2, L, 3, 2 * D), dtype=dt, device="cuda")
    big[..., :D] = vd.transpose(1, 2)
    qattn.quantize_v_int8_sm75(big[..., :D].transpose(1, 2), codes, scale)
    np.testing.assert_array_equal(codes.cpu().numpy(), want_codes)


def test_quantize_v_infinite_channel(oracle):
    v = torch.randn((1, 1, 70, 64)).to(torch.bfloat16)
    v[0, 0, 4, 2] = float("inf")
    want_codes, want_scale = oracle.quant_v(bf16_bits(v))
    codes = torch.empty((1, 1, 64, 128), dtype=torch.int8, device="cuda")
    scale = torch.empty((1, 1, 64), dtype=torch.float32, device="cuda")
    qattn.quantize_v_int8_sm75(v.cuda(), codes, scale)
    np.testing.assert_array_equal(codes.cpu().numpy(), want_codes)
    np.testing.assert_array_equal(scale.cpu().numpy(), want_scale)


ATTN_CASES = [  # dtype, hq, hk, lq, lk, D, causal
    (torch.bfloat16, 2, 2, 200, 200, 128, False),
    (torch.bfloat16, 4, 2, 77, 333, 128, False),
    (torch.float16, 2, 1, 256, 130, 128, False),
    (torch.bfloat16, 1, 1, 300, 300, 128, True),
    (torch.float16, 2, 2, 513, 513, 128, True),
    (torch.bfloat16, 1, 1, 5, 1, 128, False),
]


@pytest.mark.parametrize("case", ATTN_CASES, ids=lambda c: "-".join(map(str, c[1:])))
def test_attention_on_identical_codes(oracle, case):
    dt, hq, hk, lq, lk, D, causal = case
    q, k, v = _inputs(1, hq, hk, lq, lk, D, dt, seed=lq + 7 * lk + hq)
    q8, qs, k8, ks, _ = oracle.per_warp_int8_hadamard(bf16_bits(q), bf16_bits(k),
                                                      fp16=dt == torch.float16)
    v8, vs = oracle.quant_v(bf16_bits(v), fp16=dt == torch.float16)
    want = oracle.w8a8_attn(q8, k8, v8, vs, qs, ks, sm_scale=D ** -0.5, is_causal=causal)
    codes = torch.from_numpy(np.ascontiguousarray(v8[..., :lk].transpose(0, 1, 3, 2))).to(
        torch.float16).cuda()
    out = torch.empty((1, hq, lq, D), dtype=dt, device="cuda")
    qattn.w8a8_attn(torch.from_numpy(q8).cuda(), torch.from_numpy(k8).cuda(), codes,
                    torch.from_numpy(vs).cuda(), out, torch.from_numpy(qs).cuda(),
                    torch.from_numpy(ks).cuda(), D ** -0.5, int(causal))
    m = _metrics(out.float().cpu().numpy(), want)
    assert m["cos"] >= 0.99999 and m["rel"] <= 5e-3, m
    assert _lib.device_error() == 0


@pytest.mark.parametrize("dt,layout,D,causal,stab", [
    (torch.bfloat16, "HND", 128, False, True),
    (torch.float16, "NHD", 128, False, False),
    (torch.bfloat16, "HND", 64, False, True),
    (torch.bfloat16, "NHD", 96, True, True),
])
def test_w8a8attn_pipeline(oracle, dt, layout, D, causal, stab):
    q, k, v = _inputs(1, 2, 2, 260, 260, D, dt, seed=D + int(causal))
    if layout == "NHD":
        q, k, v = (t.transpose(1, 2).contiguous() for t in (q, k, v))
    got = turing_sage.w8a8attn(q.cuda(), k.cuda(), v.cuda(), tensor_layout=layout,
                               is_causal=causal, stabilize_k=stab)
    assert got.shape == q.shape and got.dtype == dt
    want_bits = oracle.w8a8attn(bf16_bits(q), bf16_bits(k), bf16_bits(v), layout=layout,
                                fp16=dt == torch.float16, is_causal=causal, stabilize_k=stab)
    want = from_bits(want_bits, dt).float().numpy()
    m = _metrics(got.float().cpu().numpy(), want)
    assert m["cos"] >= 0.99999 and m["rel"] <= 5e-3, m
    # Error against fp32 attention: the W8A8 algorithm's own, not more.
    qf, kf, vf = (t.float() for t in (q, k, v))
    if layout == "NHD":
        qf, kf, vf = (t.transpose(1, 2) for t in (qf, kf, vf))
    exact = torch.nn.functional.scaled_dot_product_attention(qf, kf, vf, is_causal=causal)
    if layout == "NHD":
        exact = exact.transpose(1, 2)
    e_gpu = _metrics(got.float().cpu().numpy(), exact.numpy())["rel"]
    e_orc = _metrics(want, exact.numpy())["rel"]
    assert e_gpu <= 1.05 * e_orc + 1e-4, (e_gpu, e_orc)
    # Custom op and compiled wrapper run the same kernels.
    op = torch.ops.turing_utils.w8a8_attention(q.cuda(), k.cuda(), v.cuda(), layout, causal, -1.0,
                                               0, True, stab)
    torch.testing.assert_close(op, got, rtol=0, atol=0)
    comp = turing_sage.w8a8attn_compiled(q.cuda(), k.cuda(), v.cuda(), tensor_layout=layout,
                                         is_causal=causal, stabilize_k=stab)
    torch.testing.assert_close(comp, got, rtol=0, atol=0)


def test_split_prequantize_and_reference_layout_codes(oracle):
    """prequantize_sol_sageattn -> sol_sparse_sageattn_from_prequantized equals
    w8a8attn; the low-level entry also takes int8 channel-major V codes."""
    q, k, v = _inputs(1, 2, 2, 190, 190, 128, torch.bfloat16, seed=4)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    pre = turing_sage.prequantize_sol_sageattn(qd, kd, vd, use_w8a8=True, force_dense=True)
    out, selected, possible = turing_sage.sol_sparse_sageattn_from_prequantized(
        pre, return_stats=True)
    ref = turing_sage.w8a8attn(qd, kd, vd)
    torch.testing.assert_close(out, ref, rtol=0, atol=0)
    assert selected.dtype == torch.int64 and int(selected.sum()) == 0
    codes = torch.empty((1, 2, 128, 192), dtype=torch.int8, device="cuda")
    vs = torch.empty((1, 2, 128), dtype=torch.float32, device="cuda")
    qattn.quantize_v_int8_sm75(vd, codes, vs)
    out2 = torch.empty_like(qd)
    qattn.sol_sparse_online_w8a8_prequantized_attn(
        pre.query_int8, pre.key_int8, codes, vs, out2, pre.query_scale, pre.key_scale, None, None,
        None, None, None, pre.sparse_query_blocks, pre.exact_kv_blocks, 0.0, 1, pre.sm_scale, 0, 1,
        64, 0, 1)
    torch.testing.assert_close(out2, ref, rtol=0, atol=0)
    with pytest.raises(RuntimeError, match="force_dense"):
        qattn.sol_sparse_online_w8a8_prequantized_attn(
            pre.query_int8, pre.key_int8, codes, vs, out2, pre.query_scale, pre.key_scale, None,
            None, None, None, None, pre.sparse_query_blocks, pre.exact_kv_blocks, 1.0, 1,
            pre.sm_scale, 0, 0, 64, 0, 1)
    with pytest.raises(ValueError, match="dense W8A8"):
        turing_sage.prequantize_sol_sageattn(qd, kd, vd, use_w8a8=False)


def test_configs1_shape_sampled_rows(oracle):
    """configs[1] shape (B=1, H=40, L=32760, D=128): the kernel's output at 4
    sampled 16-row tiles of 2 heads against the oracle run on those tiles."""
    B, H, L, D = 1, 40, 32760, 128
    g = torch.Generator(device="cuda").manual_seed(1000)
    q = torch.randn((B, H, L, D), generator=g, device="cuda").to(torch.bfloat16)
    k = (torch.randn((B, H, L, D), generator=g, device="cuda")
         + torch.randn((B, H, 1, D), generator=g, device="cuda") * 2.0).to(torch.bfloat16)
    v = torch.randn((B, H, L, D), generator=g, device="cuda").to(torch.bfloat16)
    pre = core.prequantize_sol_sageattn(q, k, v, use_w8a8=True, force_dense=True)
    out = core.sol_sparse_sageattn_from_prequantized(pre)
    del q, k
    for h in (0, 39):
        tiles = [0, 700, 1500, 2047]
        rows = np.concatenate([np.arange(16 * t, min(16 * t + 16, L)) for t in tiles])
        q8 = pre.query_int8[:, h:h + 1, rows].cpu().numpy()
        qs = pre.query_scale[:, h:h + 1, tiles].cpu().numpy()
        k8 = pre.key_int8[:, h:h + 1].cpu().numpy()
        ks = pre.key_scale[:, h:h + 1].cpu().numpy()
        v8 = pre.value_int8[:, h:h + 1].float().cpu().numpy().astype(np.int8)
        v8 = np.ascontiguousarray(np.pad(v8.transpose(0, 1, 3, 2), ((0, 0), (0, 0), (0, 0),
                                                                     (0, 32768 - L))))
        vs = pre.value_scale[:, h:h + 1].cpu().numpy()
        want = oracle.w8a8_attn(q8, k8, v8, vs, qs, ks, sm_scale=D ** -0.5)
        m = _metrics(out[:, h:h + 1, rows].float().cpu().numpy(), want)
        assert m["cos"] >= 0.99999 and m["rel"] <= 5e-3, (h, m)
    assert _lib.device_error() == 0


FIXTURES = sorted(GOLDEN.glob("w8a8_*.npz"))


@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: p.stem)
def test_against_reference_kernels(path):
    f = np.load(path)
    fp16, stab, causal = (bool(x) for x in f["meta"])
    dt = torch.float16 if fp16 else torch.bfloat16
    q, k, v = (from_bits(f[n], dt).cuda() for n in ("q", "k", "v"))
    q8, qs, k8, ks = quant.per_warp_int8_hadamard(q, k, stabilize_k=stab)
    for got, want in ((q8, f["q8"]), (k8, f["k8"])):
        diff = np.abs(got.cpu().numpy().astype(np.int32) - want.astype(np.int32))
        assert diff.max() <= 1 and (diff > 0).mean() < 1e-3
    for got, want in ((qs, f["qs"]), (ks, f["ks"])):
        np.testing.assert_allclose(got.cpu().numpy(), want.view(np.float32), rtol=3e-7, atol=0)
    D = q.shape[-1]
    lpad = (k.shape[2] + 63) // 64 * 64
    codes = torch.empty((1, k.shape[1], D, lpad), dtype=torch.int8, device="cuda")
    vs = torch.empty((1, k.shape[1], D), dtype=torch.float32, device="cuda")
    qattn.quantize_v_int8_sm75(v, codes, vs)
    diff = np.abs(codes.cpu().numpy().astype(np.int32)
                  - unpermute_v(f["v8_permuted"]).astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).mean() < 1e-3
    out = turing_sage.w8a8attn(q, k, v, is_causal=causal, stabilize_k=stab)
    m = _metrics(out.float().cpu().numpy(), from_bits(f["out"], dt).float().numpy())
    assert m["cos"] >= 0.9999 and m["rel"] <= 2e-2, m


def test_no_watchdog_errors():
    assert _lib.device_error() == 0


def test_preflight_self_tests():
    """The plugin's preflight_bundled / preflight_bundled_w8a8 entry points
    (attention/stable.py:521-558) pass on the B200."""
    dev = torch.device("cuda:0")
    turing_sage.preflight(dev)
    turing_sage.preflight_w8a8(dev)
    with pytest.raises(RuntimeError, match="not built"):
        turing_sage.preflight_sparse(dev)
    assert _lib.device_error() == 0
