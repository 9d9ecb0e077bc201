"""Generate the golden fixtures under tests/golden/ by running the REFERENCE's
own CUDA kernels (built from its sources by oracle/ref/build_ref.py into
oracle/_ref) on seeded CPU-generated inputs, on a B200.

    python tests/golden/make_golden.py [out_dir] [--only norm|qkrope|qkrot|w8a8]

Each fixture is a compressed .npz holding the inputs (as raw bits) and the
reference's outputs.  tests/test_oracle_golden.py checks the CPU oracle
against them; nothing at run time reads the reference checkout.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from oracle import refkernels as R  # noqa: E402


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16) \
        if t.dtype in (torch.bfloat16, torch.float16) else t.detach().cpu().numpy()


def act(rows, cols, seed, outliers=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((rows, cols), generator=g)
    if outliers:
        idx = torch.randperm(cols, generator=g)[: max(1, int(round(cols * 0.005)))]
        x[:, idx] *= 20.0
    return x.to(torch.bfloat16)


def norm_fixtures(dev, L) -> dict:
    """Segmented RMSNorm+AdaLN and LayerNorm+AdaLN (segmented_rms_adaln.cu)."""
    fx = {}
    codes = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}
    for dtype, tag in ((torch.bfloat16, "bf16"), (torch.float16, "f16"), (torch.float32, "f32")):
        g = torch.Generator().manual_seed(91 + codes[dtype])
        rows, hidden, mod_rows = 13, (5120 if dtype != torch.float32 else 2048), 3
        x = (torch.randn((rows, hidden), generator=g) * 3 + 0.5).to(dtype)
        w = (torch.rand((hidden,), generator=g) + 0.5).to(dtype)
        sc = (torch.randn((mod_rows, hidden), generator=g) * 0.1).to(dtype)
        sh = (torch.randn((mod_rows, hidden), generator=g) * 0.1).to(dtype)
        # Row 11 lies in no segment and row 12 names an out-of-range modulation
        # row: both fall back to modulation row 0.
        seg = torch.tensor([[0, 4, 2], [4, 9, 0], [9, 11, 1], [12, 13, 7]], dtype=torch.int32)
        out = torch.empty((rows, hidden), dtype=dtype, device=dev)
        xd, wd, scd, shd, segd = (t.to(dev) for t in (x, w, sc, sh, seg))
        R.check(L.ref_segmented_rms_adaln(R.ptr(xd), R.ptr(wd), R.ptr(scd), R.ptr(shd), R.ptr(segd),
                                          R.ptr(out), rows, hidden, mod_rows, 4, codes[dtype],
                                          1e-6, R.stream()), "segmented_rms_adaln")
        torch.cuda.synchronize()
        fx[f"rms_adaln_{tag}"] = {"x": bits(x), "w": bits(w), "scale": bits(sc), "shift": bits(sh),
                                  "segments": seg.numpy(), "out": bits(out)}
        batch, seq, hid, steps = 2, 9, 1536, 4
        x = (torch.randn((batch, seq, hid), generator=g) * 2 + 3.0).to(dtype)
        sc = (torch.randn((batch, steps, hid), generator=g) * 0.1).to(dtype)
        sh = (torch.randn((batch, steps, hid), generator=g) * 0.1).to(dtype)
        out = torch.empty((batch, seq, hid), dtype=dtype, device=dev)
        xd, scd, shd = (t.to(dev) for t in (x, sc, sh))
        R.check(L.ref_layer_norm_adaln(R.ptr(xd), R.ptr(scd), R.ptr(shd), R.ptr(out), batch, seq,
                                       hid, steps, codes[dtype], 1e-6, R.stream()),
                "layer_norm_adaln")
        torch.cuda.synchronize()
        fx[f"ln_adaln_{tag}"] = {"x": bits(x), "scale": bits(sc), "shift": bits(sh),
                                 "out": bits(out)}
    return fx


def rope_freqs(fb, fs, pairs, seed, dtype):
    """[fb, fs, 1, pairs, 2, 2] rotation matrices [[cos, -sin], [sin, cos]]."""
    g = torch.Generator().manual_seed(seed)
    ang = torch.rand((fb, fs, 1, pairs, 1, 1), generator=g) * 6.283
    c, s = torch.cos(ang), torch.sin(ang)
    return torch.cat([torch.cat([c, -s], -1), torch.cat([s, c], -1)], -2).to(dtype)


# (name, dtype, layout, B, Hq, Hk, Lq, Lk, D, scope, split, rot_dim, fb, fs)
QKROPE_CASES = [
    ("bf16_hnd_d128_head", torch.bfloat16, "HND", 1, 3, 3, 150, 150, 128, "head", False, 128, 1, 150),
    ("f16_nhd_d64_row_split", torch.float16, "NHD", 2, 4, 2, 77, 77, 64, "row", True, 32, 2, 77),
    ("bf16_hnd_d64_norope", torch.bfloat16, "HND", 2, 2, 2, 70, 200, 64, "head", False, 0, 1, 1),
    ("bf16_nhd_d128_row", torch.bfloat16, "NHD", 1, 5, 5, 64, 64, 128, "row", False, 96, 1, 1),
]


def qkrope_fixtures(dev, S) -> dict:
    """Fused RMSNorm + RoPE + INT8 Q/K (sage/qk_preprocess.cu:566-753)."""
    fx = {}
    for i, (name, dt, layout, B, hq, hk, lq, lk, D, scope, split, rot, fb, fs) in \
            enumerate(QKROPE_CASES):
        g = torch.Generator().manual_seed(300 + i)
        qshape = (B, hq, lq, D) if layout == "HND" else (B, lq, hq, D)
        kshape = (B, hk, lk, D) if layout == "HND" else (B, lk, hk, D)
        q = (torch.randn(qshape, generator=g) * 1.5 + 0.2).to(dt)
        k = (torch.randn(kshape, generator=g) * 0.8 - 0.3).to(dt)
        nq, nk = (D if scope == "head" else hq * D), (D if scope == "head" else hk * D)
        qn = (torch.rand((nq,), generator=g) + 0.5).to(dt)
        kn = (torch.rand((nk,), generator=g) + 0.5).to(dt)
        fr = rope_freqs(fb, fs, rot // 2, 400 + i, dt) if rot else torch.empty(0, dtype=dt)
        qd, kd, qnd, knd, frd = (t.to(dev) for t in (q, k, qn, kn, fr))
        q8 = torch.empty(qshape, dtype=torch.int8, device=dev)
        k8 = torch.empty(kshape, dtype=torch.int8, device=dev)
        qs = torch.empty((B, hq, (lq + 63) // 64 * 4), dtype=torch.float32, device=dev)
        ks = torch.empty((B, hk, (lk + 63) // 64), dtype=torch.float32, device=dev)
        qr = torch.empty((B, lq) if scope == "row" else (0,), dtype=torch.float32, device=dev)
        kr = torch.empty((B, lk) if scope == "row" else (0,), dtype=torch.float32, device=dev)
        e_i = torch.empty(0, dtype=torch.int32, device=dev)
        e_f = torch.empty(0, dtype=torch.float32, device=dev)
        S.quant_qk_rms_rope_int8_cuda(qd, kd, q8, k8, qs, ks, qnd, knd, frd, qr, kr, e_i, e_f,
                                      1e-6, rot, 64, 16, 64, 1 if layout == "HND" else 0,
                                      1 if scope == "row" else 0, split, False)
        torch.cuda.synchronize()
        fx[f"qkrope_{name}"] = {
            "q": bits(q), "k": bits(k), "qn": bits(qn), "kn": bits(kn), "freqs": bits(fr),
            "params": np.array([rot, int(split), int(scope == "row"), int(dt == torch.float16),
                                int(layout == "NHD")], np.int64),
            "q8": bits(q8), "qs": bits(qs), "k8": bits(k8), "ks": bits(ks)}
    return fx


QKROT_CASES = [
    # name, dtype, layout, B, hq, hk, lq, lk, D, scope, split, rot, fb, fs, stabilize, K offset
    ("bf16_hnd_d128_row_anchor", torch.bfloat16, "HND", 1, 2, 2, 150, 150, 128, "row", False,
     128, 1, 150, True, 2.0),
    ("f16_nhd_d64_head_split", torch.float16, "NHD", 2, 3, 1, 70, 90, 64, "head", True, 48, 1,
     1, True, 1.5),
    ("bf16_hnd_d128_head_plain", torch.bfloat16, "HND", 1, 2, 2, 100, 100, 128, "head", False,
     0, 1, 1, False, 0.0),
]


def qkrot_fixtures(dev, S) -> dict:
    """The fused prologue's Hadamard-rotated form with the K anchor
    (sage/qk_preprocess.cu:252-415, 417-753, rotate=True)."""
    fx = {}
    for i, (name, dt, layout, B, hq, hk, lq, lk, D, scope, split, rot, fb, fs, stab, off) in \
            enumerate(QKROT_CASES):
        g = torch.Generator().manual_seed(700 + i)
        qshape = (B, hq, lq, D) if layout == "HND" else (B, lq, hq, D)
        kshape = (B, hk, lk, D) if layout == "HND" else (B, lk, hk, D)
        oshape = (1, hk, 1, D) if layout == "HND" else (1, 1, hk, D)
        q = (torch.randn(qshape, generator=g) * 1.5 + 0.2).to(dt)
        k = (torch.randn(kshape, generator=g) + torch.randn(oshape, generator=g) * off).to(dt)
        nq, nk = (D if scope == "head" else hq * D), (D if scope == "head" else hk * D)
        qn = (torch.rand((nq,), generator=g) + 0.5).to(dt)
        kn = (torch.rand((nk,), generator=g) + 0.5).to(dt)
        fr = rope_freqs(fb, fs, rot // 2, 800 + i, dt) if rot else torch.empty(0, dtype=dt)
        qd, kd, qnd, knd, frd = (t.to(dev) for t in (q, k, qn, kn, fr))
        q8 = torch.empty(qshape, dtype=torch.int8, device=dev)
        k8 = torch.empty(kshape, dtype=torch.int8, device=dev)
        qs = torch.empty((B, hq, (lq + 63) // 64 * 4), dtype=torch.float32, device=dev)
        ks = torch.empty((B, hk, (lk + 63) // 64), dtype=torch.float32, device=dev)
        qr = torch.empty((B, lq) if scope == "row" else (0,), dtype=torch.float32, device=dev)
        kr = torch.empty((B, lk) if scope == "row" else (0,), dtype=torch.float32, device=dev)
        ai = torch.empty((B, hk) if stab else (0,), dtype=torch.int32, device=dev)
        av = torch.empty((B, hk, D) if stab else (0,), dtype=torch.float32, device=dev)
        S.quant_qk_rms_rope_int8_cuda(qd, kd, q8, k8, qs, ks, qnd, knd, frd, qr, kr, ai, av,
                                      1e-6, rot, 64, 16, 64, 1 if layout == "HND" else 0,
                                      1 if scope == "row" else 0, split, True)
        torch.cuda.synchronize()
        rec = {"q": bits(q), "k": bits(k), "qn": bits(qn), "kn": bits(kn), "freqs": bits(fr),
               "params": np.array([rot, int(split), int(scope == "row"), int(dt == torch.float16),
                                   int(layout == "NHD"), int(stab)], np.int64),
               "q8": bits(q8), "qs": bits(qs), "k8": bits(k8), "ks": bits(ks)}
        if stab:
            rec["anchors"], rec["anchor_values"] = bits(ai), bits(av)
        fx[f"qkrot_{name}"] = rec
    return fx


def w8a8_fixtures(dev, S) -> dict:
    """Dense W8A8-PV path: rotated (anchored) Q/K INT8 (sage/fused.cu:201-639),
    channel-wise INT8 V (quant_v_int8_cuda_sm75.cu:58-246) and the force_dense
    attention (sol_sparse_cuda_sm75.cu:709-1394, 2767-2932).  v8 is stored as
    the reference writes it (16-token permuted)."""
    fx = {}
    cases = [  # name, dtype, Hq, Hk, Lq, Lk, D, stabilize_k, causal, K offset
        ("w8a8_bf16_d128_anchor", torch.bfloat16, 2, 2, 200, 200, 128, True, False, 2.0),
        ("w8a8_f16_d64_gqa", torch.float16, 4, 2, 130, 190, 64, False, False, 0.0),
        ("w8a8_bf16_d128_causal", torch.bfloat16, 1, 1, 300, 300, 128, True, True, 1.0),
    ]
    for i, (name, dt, hq, hk, lq, lk, d, stab, causal, off) in enumerate(cases):
        g = torch.Generator().manual_seed(9100 + i)
        q = (torch.randn((1, hq, lq, d), generator=g) * 1.5).to(dt)
        k = (torch.randn((1, hk, lk, d), generator=g)
             + torch.randn((1, hk, 1, d), generator=g) * off).to(dt)
        v = torch.randn((1, hk, lk, d), generator=g).to(dt)
        qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
        q8 = torch.empty(q.shape, dtype=torch.int8, device=dev)
        k8 = torch.empty(k.shape, dtype=torch.int8, device=dev)
        qs = torch.empty((1, hq, (lq + 63) // 64 * 4), dtype=torch.float32, device=dev)
        ks = torch.empty((1, hk, (lk + 63) // 64), dtype=torch.float32, device=dev)
        rec = {"q": bits(q), "k": bits(k), "v": bits(v)}
        if stab:
            anchors = torch.empty((1, hk), dtype=torch.int32, device=dev)
            S.quant_qk_per_warp_int8_rotated_anchored_cuda(qd, kd, q8, k8, qs, ks, anchors, 64, 16,
                                                           64, 1)
        else:
            S.quant_qk_per_warp_int8_rotated_cuda(qd, kd, q8, k8, qs, ks, 64, 16, 64, 1)
        lpad = (lk + 63) // 64 * 64
        v8 = torch.empty((1, hk, d, lpad), dtype=torch.int8, device=dev)
        vs = torch.empty((1, hk, d), dtype=torch.float32, device=dev)
        S.quantize_v_int8_sm75(vd, v8, vs)
        o = torch.empty(q.shape, dtype=dt, device=dev)
        he = torch.empty((0, 0, 0, 0), dtype=torch.float16, device=dev)
        fe = torch.empty((0, 0, 0), dtype=torch.float32, device=dev)
        sq = torch.zeros(((lq + 63) // 64,), dtype=torch.uint8, device=dev)
        ek = torch.zeros(((lk + 63) // 64,), dtype=torch.uint8, device=dev)
        S.sol_sparse_online_w8a8_prequantized_attn(q8, k8, v8, vs, o, qs, ks, he, he, he, fe, fe,
                                                   sq, ek, 0.0, 1, d ** -0.5, 0, 1, 64,
                                                   int(causal), 1)
        torch.cuda.synchronize()
        rec.update({"q8": bits(q8), "qs": bits(qs), "k8": bits(k8), "ks": bits(ks),
                    "v8_permuted": bits(v8), "vs": bits(vs), "out": bits(o),
                    "meta": np.array([int(dt == torch.float16), int(stab), int(causal)], np.int32)})
        if stab:
            rec["anchors"] = bits(anchors)
        fx[name] = rec
    return fx


def main(out_dir: Path, only: str = "") -> None:
    out_dir.mkdir(parents=True, exist_ok=True)
    if only == "qkrope":
        fx = qkrope_fixtures(torch.device("cuda:0"), R.sage())
        for name, rec in fx.items():
            np.savez_compressed(out_dir / f"{name}.npz", **rec)
        print(f"wrote {len(fx)} fixtures to {out_dir}")
        return
    if only == "qkrot":
        fx = qkrot_fixtures(torch.device("cuda:0"), R.sage())
        for name, rec in fx.items():
            np.savez_compressed(out_dir / f"{name}.npz", **rec)
        print(f"wrote {len(fx)} fixtures to {out_dir}")
        return
    if only == "w8a8":
        fx = w8a8_fixtures(torch.device("cuda:0"), R.sage())
        for name, rec in fx.items():
            np.savez_compressed(out_dir / f"{name}.npz", **rec)
        print(f"wrote {len(fx)} fixtures to {out_dir}")
        return
    if only == "norm":
        fx = norm_fixtures(torch.device("cuda:0"), R.linear())
        for name, rec in fx.items():
            np.savez_compressed(out_dir / f"{name}.npz", **rec)
        print(f"wrote {len(fx)} fixtures to {out_dir}")
        return
    dev = torch.device("cuda:0")
    L = R.linear()
    S = R.sage()
    fx = {}

    # --- ConvRot row-buffer (plain / SwiGLU / GELU, INT8 / INT4) ---------------
    cases = {"plain_5120": (act(8, 5120, 1), 0, 0), "plain_256": (act(3, 256, 2), 0, 0),
             "swiglu_5376": (act(3, 2 * 5376, 3, False), 1, 0),
             "gelu_13824": (act(4, 13824, 4), 0, 1)}
    edge = np.zeros((3, 512), np.uint16)
    edge[0, 5], edge[1, :], edge[2, 300] = 0x7FC0, 0x7F7F, 0xFF80
    cases["edge_512"] = (torch.from_numpy(edge.view(np.int16)).view(torch.bfloat16), 0, 0)
    for name, (x, swiglu, gelu) in cases.items():
        hidden = x.shape[1] // (2 if swiglu else 1)
        rec = {"x": bits(x)}
        for int4 in (0, 1):
            q = torch.empty((x.shape[0], hidden // 2 if int4 else hidden), dtype=torch.int8, device=dev)
            s = torch.empty((x.shape[0], 1), dtype=torch.float32, device=dev)
            xd = x.to(dev)
            R.check(L.ref_bf16_convrot(R.ptr(xd), x.shape[0], hidden, swiglu, gelu, int4, R.ptr(q),
                                       R.ptr(s), R.stream()), "convrot")
            torch.cuda.synchronize()
            rec[f"q{4 if int4 else 8}"], rec[f"s{4 if int4 else 8}"] = bits(q), bits(s)
            if swiglu or gelu:
                for fp16 in (0, 1):
                    xs = x.to(torch.float16) if fp16 else x
                    xs = xs.to(dev)
                    r = torch.empty((x.shape[0], hidden), dtype=xs.dtype, device=dev)
                    pa = torch.empty((x.shape[0], hidden // 256), dtype=torch.float32, device=dev)
                    q2 = torch.empty_like(q)
                    s2 = torch.empty_like(s)
                    R.check(L.ref_staged_convrot(R.ptr(xs), fp16, x.shape[0], hidden, gelu, int4,
                                                 R.ptr(r), R.ptr(pa), R.ptr(q2), R.ptr(s2),
                                                 R.stream()), "staged convrot")
                    torch.cuda.synchronize()
                    tag = f"staged{'16' if fp16 else ''}_{4 if int4 else 8}"
                    rec[f"q_{tag}"], rec[f"s_{tag}"] = bits(q2), bits(s2)
        fx[f"convrot_{name}"] = rec

    # --- W8A8 linear / W4A8 / codebook / dequant ------------------------------
    for i, (m, n, k) in enumerate([(33, 128, 128), (129, 264, 256)]):
        g = torch.Generator().manual_seed(4300 + i)
        a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
        w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
        a_s = torch.rand((m,), generator=g) * 0.02 + 0.001
        w_s = torch.rand((n,), generator=g) * 4e-3 + 1e-3
        b = (torch.randn((n,), generator=g) * 0.02).to(torch.bfloat16).float()
        o = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        ad, wd, asd, wsd, bd = (t.to(dev) for t in (a, w, a_s, w_s, b))
        R.check(L.ref_int8_linear(R.ptr(ad), R.ptr(wd), R.ptr(asd), R.ptr(wsd), R.ptr(bd), R.ptr(o),
                                  m, n, k, R.stream()), "int8 linear")
        torch.cuda.synchronize()
        fx[f"int8_linear_{m}x{n}x{k}"] = {"a": a.numpy(), "w": w.numpy(), "a_s": a_s.numpy(),
                                          "w_s": w_s.numpy(), "bias": b.numpy(), "out": bits(o)}
    g = torch.Generator().manual_seed(4301)
    m, n, k = 17, 72, 80
    a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    packed = ((w[:, 0::2].int() & 0xF) | ((w[:, 1::2].int() & 0xF) << 4)).to(torch.uint8).view(torch.int8)
    a_s = torch.rand((m,), generator=g) * 0.02 + 0.001
    w_s = torch.rand((n,), generator=g) * 0.03 + 0.001
    o = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    ad, pd, asd, wsd = (t.to(dev) for t in (a, packed, a_s, w_s))
    R.check(L.ref_w4a8_linear(R.ptr(ad), R.ptr(pd), R.ptr(asd), R.ptr(wsd), None, R.ptr(o), m, n, k,
                              R.stream()), "w4a8")
    torch.cuda.synchronize()
    fx["w4a8_17x72x80"] = {"a": a.numpy(), "w_packed": packed.numpy(), "a_s": a_s.numpy(),
                           "w_s": w_s.numpy(), "out": bits(o)}
    for gsz in (16, 128):
        g = torch.Generator().manual_seed(4388 + gsz)
        m, n, k = 7, 24, 256
        a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
        codes = torch.randint(0, 16, (n, k), generator=g, dtype=torch.int32)
        packed = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).to(torch.uint8).view(torch.int8)
        cb = torch.linspace(-1.0, 1.0, 16)
        gs = (torch.rand((n, k // gsz), generator=g) * 64.0 + 4.0).to(torch.float8_e4m3fn).view(torch.uint8)
        a_s = torch.rand((m,), generator=g) * 0.01
        c_s = torch.rand((n,), generator=g) * 0.02
        b = torch.randn((n,), generator=g).to(torch.bfloat16).float()
        ws = torch.empty((n, k), dtype=torch.int8, device=dev)
        o = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        t = [x.to(dev) for x in (a, packed, a_s, gs, c_s, cb, b)]
        R.check(L.ref_codebook_linear(*[R.ptr(x) for x in t], R.ptr(ws), n, R.ptr(o), m, n, k, gsz,
                                      R.stream()), "codebook")
        torch.cuda.synchronize()
        fx[f"codebook_g{gsz}"] = {"a": a.numpy(), "w_packed": packed.numpy(), "a_s": a_s.numpy(),
                                  "gs": gs.numpy(), "c_s": c_s.numpy(), "codebook": cb.numpy(),
                                  "bias": b.numpy(), "w8": ws.cpu().numpy(), "out": bits(o)}
    g = torch.Generator().manual_seed(2)
    acc = torch.randint(-2 ** 24, 2 ** 24, (37, 64), generator=g, dtype=torch.int32)
    a_s = torch.rand((37,), generator=g) * 0.01
    w_s = torch.rand((64,), generator=g) * 0.02
    o = torch.empty((37, 64), dtype=torch.bfloat16, device=dev)
    t = [x.to(dev) for x in (acc, a_s, w_s)]
    R.check(L.ref_dequant(R.ptr(t[0]), R.ptr(t[1]), R.ptr(t[2]), 64, R.ptr(o), 37, 64, R.stream()),
            "dequant")
    torch.cuda.synchronize()
    fx["dequant_37x64"] = {"acc": acc.numpy(), "a_s": a_s.numpy(), "w_s": w_s.numpy(), "out": bits(o)}

    # --- Sage quantizers + attention (reference built with --use_fast_math) ---
    for layout, lid in (("HND", 1), ("NHD", 0)):
        g = torch.Generator().manual_seed(77 + lid)
        q = torch.randn((1, 2, 129, 128), generator=g).to(torch.bfloat16)
        k = (torch.randn((1, 2, 151, 128), generator=g) + 1.5).to(torch.bfloat16)
        v = torch.randn((1, 2, 151, 128), generator=g).to(torch.bfloat16)
        if layout == "NHD":
            q, k, v = (x.transpose(1, 2).contiguous() for x in (q, k, v))
        qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
        q8 = torch.empty(q.shape, dtype=torch.int8, device=dev)
        k8 = torch.empty(k.shape, dtype=torch.int8, device=dev)
        qs = torch.empty((1, 2, 12), dtype=torch.float32, device=dev)
        ks = torch.empty((1, 2, 3), dtype=torch.float32, device=dev)
        S.quant_per_warp_int8_cuda(qd, q8, qs, 64, 16, lid)
        S.quant_per_block_int8_cuda(kd, k8, ks, 64, lid)
        o = torch.empty(q.shape, dtype=torch.bfloat16, device=dev)
        S.qk_int8_sv_f16_accum_f32_attn(q8, k8, vd, o, qs, ks, lid, 0, 2, 128 ** -0.5, 0)
        torch.cuda.synchronize()
        fx[f"sage_{layout}"] = {"q": bits(q), "k": bits(k), "v": bits(v), "q8": bits(q8),
                                "qs": bits(qs), "k8": bits(k8), "ks": bits(ks), "out": bits(o)}

    for name, rec in fx.items():
        np.savez_compressed(out_dir / f"{name}.npz", **rec)
    print(f"wrote {len(fx)} fixtures to {out_dir}")


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    only = sys.argv[sys.argv.index("--only") + 1] if "--only" in sys.argv else ""
    if only:
        args = [a for a in args if a != only]
    main(Path(args[0]) if args else Path(__file__).resolve().parent, only)
