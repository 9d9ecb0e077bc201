"""TEST INFRASTRUCTURE ONLY: time the reference's own CUDA kernels on a B200.

The kernels are the ones oracle/ref/build_ref.py compiles from the reference
checkout into oracle/_ref (the sm75 `mma.sync` code built for sm_100a).  This
is the same-box baseline the sm_100a kernels are compared with: the Sage INT8
attention and the dense W8A8 attention at configs[1]'s shape
(B=1, H=40, L=32760, D=128, bf16, K + per-channel offset N(0, 2)) and the
ConvRot quantizer + INT8 linear at configs[0]'s shape (X [4096, 5120],
W [13824, 5120]).  Each kernel: 2 untimed calls, then CUDA events around 5
calls on the current stream.  One JSON line per kernel on stdout.

    python oracle/ref/time_reference.py
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import refkernels as R  # noqa: E402


def timed(fn, warm: int = 2, reps: int = 5) -> float:
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def report(name: str, ms: float, ops: float | None = None, **extra) -> None:
    rec = {"kernel": name, "ms": round(ms, 4), **extra}
    if ops is not None:
        rec["tops"] = round(ops / (ms * 1e-3) / 1e12, 1)
    print(json.dumps(rec), flush=True)


def attention(dev, S) -> None:
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

    def sage_quant():
        S.quant_per_warp_int8_cuda(q, q8, qs, 64, 16, 1)
        S.quant_per_block_int8_cuda(k, k8, ks, 64, 1)

    report("reference sage quant (Q per warp, K per block)", timed(sage_quant))
    report("reference qk_int8_sv_f16_accum_f32_attn (Sage)",
           timed(lambda: S.qk_int8_sv_f16_accum_f32_attn(q8, k8, v, o, qs, ks, 1, 0, 2, scale, 0)),
           ops)

    anchors = torch.empty((B, H), dtype=torch.int32, device=dev)
    lpad = (L + 63) // 64 * 64
    v8 = torch.empty((B, H, D, lpad), dtype=torch.int8, device=dev)
    vs = torch.empty((B, H, D), dtype=torch.float32, device=dev)

    def w8a8_quant():
        S.quant_qk_per_warp_int8_rotated_anchored_cuda(q, k, q8, k8, qs, ks, anchors, 64, 16, 64, 1)
        S.quantize_v_int8_sm75(v, v8, vs)

    report("reference W8A8 quant (rotated anchored Q/K, channel V)", timed(w8a8_quant))
    he = torch.empty((0, 0, 0, 0), dtype=torch.float16, device=dev)
    fe = torch.empty((0, 0, 0), dtype=torch.float32, device=dev)
    sq = torch.zeros(((L + 63) // 64,), dtype=torch.uint8, device=dev)
    ek = torch.zeros(((L + 63) // 64,), dtype=torch.uint8, device=dev)
    report("reference sol_sparse_online_w8a8_prequantized_attn (dense W8A8)",
           timed(lambda: S.sol_sparse_online_w8a8_prequantized_attn(
               q8, k8, v8, vs, o, qs, ks, he, he, he, fe, fe, sq, ek, 0.0, 1, scale, 0, 1, 128, 0,
               1)), ops)


def linear(dev, Lib) -> None:
    M, K, N = 4096, 5120, 13824
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
    w = torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
    w_s = torch.rand((N,), generator=g, device=dev) * 4e-3 + 1e-3
    bias = (torch.randn((N,), generator=g, device=dev) * 0.02).float()
    xq = torch.empty((M, K), dtype=torch.int8, device=dev)
    xs = torch.empty((M, 1), dtype=torch.float32, device=dev)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    report("reference bf16_rowbuffer_convrot_quantize (INT8)",
           timed(lambda: R.check(Lib.ref_bf16_convrot(R.ptr(x), M, K, 0, 0, 0, R.ptr(xq), R.ptr(xs),
                                                      R.stream()), "convrot")))
    report("reference turing_int8_linear (CUTLASS sm75 tiles)",
           timed(lambda: R.check(Lib.ref_int8_linear(R.ptr(xq), R.ptr(w), R.ptr(xs), R.ptr(w_s),
                                                     R.ptr(bias), R.ptr(out), M, N, K,
                                                     R.stream()), "int8 linear")),
           2.0 * M * N * K)


def main() -> None:
    dev = torch.device("cuda:0")
    linear(dev, R.linear())
    attention(dev, R.sage())


if __name__ == "__main__":
    main()
