"""TEST INFRASTRUCTURE ONLY: time the reference's own CUDA kernels beside this
repository's on the same B200, on the same inputs.

The reference kernels are the ones oracle/ref/build_ref.py compiles from the
reference checkout into oracle/_ref (the sm75 `mma.sync` code built for
sm_100a, unmodified).  This is the same-box bar the sm_100a kernels must beat.
Ops, at BASELINE configs[0]'s and configs[1]'s shapes:

* ConvRot INT8 quantize of X [4096, 5120] bf16
  (reference `turing_bf16_int8_convrot_quantize`, convrot_quant.cu:566-589);
* INT8 linear [4096, 5120] x [13824, 5120]^T + epilogue
  (reference `turing_int8_linear`, w4a8.cu:1185-1219);
* Sage Q per-warp + K per-block INT8 quantizers and the Sage attention
  (reference `qk_int8_sv_f16_accum_f32_attn`, qk_int_sv_f16_cuda_sm75.cu:984-1123)
  at B=1, H=40, L=32760, D=128, bf16, K + per-channel offset N(0, 2);
* the dense W8A8 path: rotated anchored Q/K + channel-wise V quantizers and
  `sol_sparse_online_w8a8_prequantized_attn` with force_dense=1
  (sol_sparse_cuda_sm75.cu:709-1394).

After a 1 s warm-up of the GPU, each op: 2 untimed calls, then 5 calls each
bracketed by CUDA events on the current stream, with a 256 MB buffer written between calls (outside the
events) so no call finds the previous call's operands in the 126 MB L2.  The
median is reported.  One JSON line per op on stdout:
{"op", "reference_ms", "ours_ms", "speedup", ...}.

    python oracle/ref/time_reference.py
"""
from __future__ import annotations

import json
import statistics
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "comfyui-turing-utils_b200"))

from oracle import refkernels as R  # noqa: E402

_FLUSH = None


def timed(fn, warm: int = 2, reps: int = 5) -> float:
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        _FLUSH.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    return statistics.median(times)


def report(op: str, ref_ms: float, ours_ms: float, ops: float | None = None, **extra) -> None:
    rec = {"op": op, "reference_ms": round(ref_ms, 4), "ours_ms": round(ours_ms, 4),
           "speedup": round(ref_ms / ours_ms, 2), **extra}
    if ops is not None:
        rec["reference_tops"] = round(ops / (ref_ms * 1e-3) / 1e12, 1)
        rec["ours_tops"] = round(ops / (ours_ms * 1e-3) / 1e12, 1)
    print(json.dumps(rec), flush=True)


def attention(dev, S) -> None:
    from comfyui_turing_utils_kernel import _sage_fused_sm75 as F
    from comfyui_turing_utils_kernel import _sage_qattn_sm75 as A

    B, H, L, D = 1, 40, 32760, 128
    g = torch.Generator(device=dev).manual_seed(1000)
    q = torch.randn((B, H, L, D), generator=g, device=dev).to(torch.bfloat16)
    k = (torch.randn((B, H, L, D), generator=g, device=dev)
         + torch.randn((B, H, 1, D), generator=g, device=dev) * 2.0).to(torch.bfloat16)
    v = torch.randn((B, H, L, D), generator=g, device=dev).to(torch.bfloat16)
    ops = 4.0 * B * H * L * L * D
    q8 = torch.empty(q.shape, dtype=torch.int8, device=dev)
    k8 = torch.empty(k.shape, dtype=torch.int8, device=dev)
    qs = torch.empty((B, H, (L + 63) // 64 * 4), dtype=torch.float32, device=dev)
    ks = torch.empty((B, H, (L + 63) // 64), dtype=torch.float32, device=dev)
    o = torch.empty_like(q)
    scale = D ** -0.5

    def sage_quant(M):
        return lambda: (M.quant_per_warp_int8_cuda(q, q8, qs, 64, 16, 1),
                        M.quant_per_block_int8_cuda(k, k8, ks, 64, 1))

    report("sage quant (Q per warp, K per block)", timed(sage_quant(S)), timed(sage_quant(F)))
    # Both attentions read the same codes (the reference's quantizer ran last
    # in each timing loop above, so q8/k8/qs/ks hold its codes).
    S.quant_per_warp_int8_cuda(q, q8, qs, 64, 16, 1)
    S.quant_per_block_int8_cuda(k, k8, ks, 64, 1)
    ref_ms = timed(lambda: S.qk_int8_sv_f16_accum_f32_attn(q8, k8, v, o, qs, ks, 1, 0, 2, scale, 0))
    o_ref = o.clone()
    ours_ms = timed(lambda: A.qk_int8_sv_f16_accum_f32_attn(q8, k8, v, o, qs, ks, 1, 0, 2, scale, 0))
    cos = torch.nn.functional.cosine_similarity(o.float().flatten(), o_ref.float().flatten(), dim=0)
    report("Sage INT8 attention (qk_int8_sv_f16_accum_f32_attn)", ref_ms, ours_ms, ops,
           output_cosine_vs_reference=round(float(cos), 6))

    anchors = torch.empty((B, H), dtype=torch.int32, device=dev)
    lpad = (L + 63) // 64 * 64
    v8 = torch.empty((B, H, D, lpad), dtype=torch.int8, device=dev)
    vs = torch.empty((B, H, D), dtype=torch.float32, device=dev)
    vcodes = torch.empty((B, H, L, D), dtype=torch.float16, device=dev)
    vs_ours = torch.empty((B, H, D), dtype=torch.float32, device=dev)

    def ref_w8a8_quant():
        S.quant_qk_per_warp_int8_rotated_anchored_cuda(q, k, q8, k8, qs, ks, anchors, 64, 16, 64, 1)
        S.quantize_v_int8_sm75(v, v8, vs)

    def our_w8a8_quant():
        F.quant_qk_per_warp_int8_rotated_anchored_cuda(q, k, q8, k8, qs, ks, anchors, 64, 16, 64, 1)
        A.quantize_v_codes(v, vcodes, vs_ours)

    report("W8A8 quant (rotated anchored Q/K, channel-wise V)", timed(ref_w8a8_quant),
           timed(our_w8a8_quant))
    ref_w8a8_quant()
    our_w8a8_quant()
    he = torch.empty((0, 0, 0, 0), dtype=torch.float16, device=dev)
    fe = torch.empty((0, 0, 0), dtype=torch.float32, device=dev)
    sq = torch.zeros(((L + 63) // 64,), dtype=torch.uint8, device=dev)
    ek = torch.zeros(((L + 63) // 64,), dtype=torch.uint8, device=dev)
    ref_ms = timed(lambda: S.sol_sparse_online_w8a8_prequantized_attn(
        q8, k8, v8, vs, o, qs, ks, he, he, he, fe, fe, sq, ek, 0.0, 1, scale, 0, 1, 128, 0, 1))
    o_ref = o.clone()
    ours_ms = timed(lambda: A.w8a8_attn(q8, k8, vcodes, vs_ours, o, qs, ks, scale, 0))
    cos = torch.nn.functional.cosine_similarity(o.float().flatten(), o_ref.float().flatten(), dim=0)
    report("dense W8A8 attention (sol_sparse_online_w8a8_prequantized_attn, force_dense)",
           ref_ms, ours_ms, ops, output_cosine_vs_reference=round(float(cos), 6))


def linear(dev, Lib) -> None:
    from comfyui_turing_utils_kernel import _C

    M, K, N = 4096, 5120, 13824
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
    w = torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
    w_s = torch.rand((N,), generator=g, device=dev) * 4e-3 + 1e-3
    bias = (torch.randn((N,), generator=g, device=dev) * 0.02).float()
    xq = torch.empty((M, K), dtype=torch.int8, device=dev)
    xs = torch.empty((M, 1), dtype=torch.float32, device=dev)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    ref_ms = timed(lambda: R.check(Lib.ref_bf16_convrot(R.ptr(x), M, K, 0, 0, 0, R.ptr(xq),
                                                        R.ptr(xs), R.stream()), "convrot"))
    ours_ms = timed(lambda: _C.turing_bf16_int8_convrot_quantize(x))
    oq, os_ = _C.turing_bf16_int8_convrot_quantize(x)
    report("ConvRot INT8 quantize (turing_bf16_int8_convrot_quantize)", ref_ms, ours_ms,
           codes_equal=bool(torch.equal(oq, xq)), scales_equal=bool(torch.equal(os_, xs)),
           gbs_ours=round((2 * M * K + M * K + 4 * M) / (ours_ms * 1e-3) / 1e9, 1))
    ref_ms = timed(lambda: R.check(Lib.ref_int8_linear(R.ptr(xq), R.ptr(w), R.ptr(xs), R.ptr(w_s),
                                                       R.ptr(bias), R.ptr(out), M, N, K,
                                                       R.stream()), "int8 linear"))
    ours_ms = timed(lambda: _C.turing_int8_linear(xq, w, xs.view(M), w_s, bias))
    mine = _C.turing_int8_linear(xq, w, xs.view(M), w_s, bias)
    torch.cuda.synchronize()
    # Where the two outputs differ, which one the oracle's epilogue
    # ((float(acc) * a_s) * w_s + bias, one bf16 rounding) agrees with, on
    # 16 sampled rows.
    import numpy as np

    import oracle

    differ = (mine != out)
    # The sampled rows: 8 random ones plus up to 8 rows where the outputs differ.
    diff_rows = torch.nonzero(differ.any(dim=1)).flatten()[:8].cpu()
    rows = torch.cat([torch.randperm(M, generator=torch.Generator().manual_seed(3))[:8],
                      diff_rows]).unique().numpy()
    q_np = xq.cpu().numpy()
    acc = oracle.int8_gemm_rows(q_np, w.cpu().numpy(), rows)
    want = oracle.dequant_bf16(acc, xs.cpu().numpy()[rows], w_s.cpu().numpy(),
                               bias.cpu().numpy())

    def bits(t):
        return t.cpu().view(torch.int16).numpy().view(np.uint16)[rows]

    ulp = (mine.float() - out.float()).abs() / out.float().abs().clamp_min(1e-30)
    report("INT8 linear (turing_int8_linear)", ref_ms, ours_ms, 2.0 * M * N * K,
           outputs_equal=bool(torch.equal(mine, out)),
           outputs_differing_frac=round(float(differ.float().mean()), 6),
           max_rel_diff=float(ulp.max()),
           sampled_rows=int(rows.size), rows_with_differences=int(differ.any(dim=1).sum()),
           ours_equal_oracle_rows=bool(np.array_equal(bits(mine), want)),
           reference_equal_oracle_rows=bool(np.array_equal(bits(out), want)),
           reference_mismatches_vs_oracle=int((bits(out) != want).sum()),
           ours_mismatches_vs_oracle=int((bits(mine) != want).sum()))


def warm(dev, seconds: float = 1.0) -> None:
    """Bring the GPU out of its idle clocks before the first timing."""
    import time

    a = torch.randn((4096, 4096), device=dev, dtype=torch.bfloat16)
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        for _ in range(20):
            a = torch.matmul(a, a) * 1e-2
        torch.cuda.synchronize()


def main() -> None:
    dev = torch.device("cuda:0")
    warm(dev)
    linear(dev, R.linear())
    attention(dev, R.sage())


if __name__ == "__main__":
    main()
