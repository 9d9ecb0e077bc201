"""Benchmark of the B200 quantized DiT path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload W] [--impl ours|reference]

Workloads (synthetic seeded inputs of the stated shapes
and distributions — the reference benchmarks on no public dataset):
  dit_block  configs[4] (default): one Wan2.1-14B-shaped DiT block, dim 5120,
             40 heads x 128, FFN 13824, L = 75600, 512 text tokens, W8A8
             ConvRot linears, Sage INT8 self- and cross-attention, AdaLN;
             over the torchrun ranks either all-to-all sequence parallel
             (--parallel a2a, default: token shards through every linear,
             head shards for self-attention) or Megatron tensor + sequence
             parallel (--parallel tp), over NCCL; a "parity" key checks 256
             sampled output tokens against the fp32 reference block.
             Metric: block tokens/s (L / block time, max over ranks),
             strong scaling.
  attention  configs[1]: Sage INT8 attention B=1, H=40, L=32760, D=128, HND,
             Q/K/V bf16 ~N(0,1), K + per-channel offset ~N(0,2), K mean
             smoothing, Q per 16-token warp tiles, K per 64-token blocks.
             Step = Q/K quantize + attention.
  attention_rope
             configs[1] shape through the fused Q/K prologue a Wan block uses:
             RMSNorm over the whole 5120-wide row (norm_scope "row") with an
             affine weight, interleaved RoPE over all 128 channels with
             per-token rotations, INT8 Q/K in one pass, then the attention.
             Step = prologue + attention; the prologue is reported against
             the HBM roofline beside the attention's.
  w8a8_attention
             configs[1] shape through the dense W8A8-PV backend (the loader's
             default): randomized-Hadamard Q/K INT8 with the conditional K
             anchor, channel-wise INT8 V, P as u8 codes.  Step = the three
             quantizers + attention.
  linear     configs[0]: ConvRot W8A8 linear, X [4096, 5120] bf16 with 0.5%
             outlier channels x20, W [13824, 5120] int8, per-channel scales,
             bf16 bias.  Step = ConvRot INT8 quantize + tcgen05 GEMM with the
             fused dequant/bias/bf16 epilogue.
  codebook   configs[2]: W4A8 grouped-codebook linear, X [8192, 5120].
  w4a4_ffn   configs[3]: W4A4 ConvRot FFN pair over 32760 tokens.
Metric of the other workloads: INT8 TOPS (whole job, all ranks) = algorithmic
ops / device time.

Multi-GPU (torchrun): every workload splits one config over the ranks
(strong scaling): dit_block as above; the linears their tokens (rows of X,
weights replicated), the attentions their 40 heads, with no data-path
collective.  Time = max over ranks of the per-rank device time.

--impl reference times the reference's CPU implementation of the same step
(the torch fp32 dequantize-then-matmul / dequantize-then-attention path of
kernel/scripts/validate_compatible.py plus the ConvRot CPU restatement of
oracle/) on the host cores, on a bounded sample of the workload; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG_DIR = ROOT / "comfyui-turing-utils_b200"
for _p in (str(ROOT), str(PKG_DIR)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "INT8 TOPS/GPU (W8A8 linear, Sage attn) and DiT-block tokens/s at 1/2/4/8 B200"
UNIT = "TOPS"
L2_FLUSH_BYTES = 256 << 20


def load_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        p = json.loads(path.read_text())
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def ncu_traffic(kernel: str, workload: str):
    """DRAM bytes per launch from the committed ncu summary (profiles/ncu_traffic.txt)."""
    path = ROOT / "profiles" / "ncu_traffic.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 3 and parts[0] == kernel and parts[1] == workload:
            return float(parts[2])
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------- workloads --

def _host(t: torch.Tensor) -> torch.Tensor:
    """A host copy of t, pinned when CUDA is present (the CPU-only reference
    arm has no pinned memory)."""
    t = t.cpu()
    return t.pin_memory() if torch.cuda.is_available() else t


class LinearWorkload:
    name = "linear"
    config = {"workload": "convrot_w8a8_linear (BASELINE configs[0])", "m": 4096, "k": 5120,
              "n": 13824, "rotation": 256, "activation": "per-token int8",
              "weight": "int8 per-channel"}

    def __init__(self, device, seed):
        import comfyui_turing_utils_kernel as kernel
        from comfyui_turing_utils_kernel import _C

        self.kernel, self._C = kernel, _C
        m, k, n = self.config["m"], self.config["k"], self.config["n"]
        self.ops = self.dom_ops = 2.0 * m * n * k
        g = torch.Generator().manual_seed(seed)
        x = torch.randn((m, k), generator=g)
        idx = torch.randperm(k, generator=g)[: int(round(k * 0.005))]
        x[:, idx] *= 20.0
        x = x.to(torch.bfloat16)
        self.x_host = x.pin_memory() if device.type == "cuda" else x
        self.x = self.x_host.to(device)
        self.w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8).to(device)
        self.w_s = (torch.rand((n,), generator=g) * 4e-3 + 1e-3).to(device)
        self.bias = (torch.randn((n,), generator=g) * 0.02).to(torch.bfloat16).to(device)
        self.bias_f32 = self.bias.float()
        self.out_host = torch.empty((m, n), dtype=torch.bfloat16,
                                    pin_memory=device.type == "cuda")
        self.launches_per_step = 2
        self.dominant = "gemm_i8"
        self.h2d_bytes = self.x_host.numel() * 2
        self.d2h_bytes = self.out_host.numel() * 2

    def step(self, ev=None):
        """One step on resident inputs; ev = (start, mid, end) events to time the
        quantizer and the GEMM separately."""
        if ev:
            ev[0].record()
        xq, xs = self._C.turing_bf16_int8_convrot_quantize(self.x)
        if ev:
            ev[1].record()
        out = self._C.turing_int8_linear(xq, self.w, xs, self.w_s, self.bias_f32)
        if ev:
            ev[2].record()
        return out

    def step_e2e(self):
        x = self.x_host.to(self.x.device, non_blocking=True)
        xq, xs = self.kernel.turing_bf16_int8_convrot_quantize(x)
        out = self.kernel.turing_int8_linear(xq, self.w, xs, self.w_s, self.bias)
        self.out_host.copy_(out, non_blocking=True)
        return out

    cpu_sample_desc = "rows of X, full N and K (ConvRot oracle + torch fp32 dequantize-then-matmul)"

    def aux_roofline(self, pro_ms, peaks):
        """The ConvRot prologue (event 0 -> 1 of a step) against HBM:
        2 B read + 1 B code written per element + a 4 B scale per row."""
        m, k = self.x.size(0), self.x.size(1)
        bytes_ = 3 * m * k + 4 * m
        achieved = bytes_ / (pro_ms * 1e-3) / 1e9
        return {"prologue": {"kernel": "convrot_rowbuffer", "bound": "hbm",
                             "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                             "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                             "algorithmic_bytes": bytes_, "ms": round(pro_ms, 4)}}

    def roofline(self, dom_ms, peaks):
        int8_peak = 2.0 * peaks["bf16_tflops"]
        achieved = self.dom_ops / (dom_ms * 1e-3) / 1e12
        return {"kernel": self.dominant, "bound": "tensor", "achieved": round(achieved, 1),
                "peak": round(int8_peak, 1), "unit": "TOPS", "frac": round(achieved / int8_peak, 4),
                "peak_source": f"2 x {peaks['source']} dense bf16 TFLOP/s (MEASURED_PEAKS.json "
                               "bf16_tflops); dense INT8 = 2 x BF16 on B200",
                "kernel_ms": round(dom_ms, 4)}

    def cpu_reference_step(self, rows: int):
        """Reference CPU path on a row sample: ConvRot restatement + fp32
        dequantize-then-matmul (validate_compatible.py:110-114)."""
        import numpy as np

        import oracle

        xs = self.x_host[:rows]
        q, s = oracle.convrot_quantize(xs.view(torch.int16).numpy().view(np.uint16))
        w = self.w_cpu
        out = (torch.from_numpy(q).float() @ w.t()) * torch.from_numpy(s) \
            * self.w_s_cpu[None, :] + self.bias_cpu[None, :]
        return out.to(torch.bfloat16), 2.0 * rows * self.config["n"] * self.config["k"]

    def prepare_cpu(self):
        self.w_cpu = self.w.cpu().float()
        self.w_s_cpu = self.w_s.cpu()
        self.bias_cpu = self.bias.cpu().float()


def _chunks(n, k):
    """Weight chunks (decode + GEMM rounds) of a staged W4 linear."""
    from comfyui_turing_utils_kernel._C import _weight_chunk_rows

    return -(-n // _weight_chunk_rows(n, k))


class CodebookWorkload:
    """grouped-codebook W4A8 linear.  The reference's fast
    path stores symmetric codebook weights (packed 4-bit indices, 16-entry fp32
    codebook, E4M3 group scales relative to an fp32 channel scale); the config's
    per-group zero points have no codebook form and run with the zero point
    fixed at 8 (codebook[i] = i - 8), which leaves the arithmetic unchanged."""

    name = "codebook"
    config = {"workload": "codebook_w4a8_linear (BASELINE configs[2])", "m": 8192, "k": 5120,
              "n": 5120, "group_size": 128, "rotation": 256,
              "activation": "per-token int8 (ConvRot)",
              "weight": "4-bit codebook indices, e4m3 group scales, fp32 channel scales",
              "zero_points": "not built; parity unpinned: the config's asymmetric per-group "
                             "zero points need a correction term, which the reference's Turing "
                             "fast path rejects (dispatch.py:690-702, correction is None) and "
                             "hands to comfy-kitchen (absent); measured on the symmetric "
                             "codebook layout the reference's kernel takes"}

    def __init__(self, device, seed):
        import comfyui_turing_utils_kernel as kernel
        from comfyui_turing_utils_kernel import _C

        self.kernel, self._C = kernel, _C
        m, k, n, gsz = (self.config[key] for key in ("m", "k", "n", "group_size"))
        self.ops = self.dom_ops = 2.0 * m * n * k
        g = torch.Generator().manual_seed(seed)
        x = torch.randn((m, k), generator=g).to(torch.bfloat16)
        self.x_host = x.pin_memory() if device.type == "cuda" else x
        self.x = self.x_host.to(device)
        idx = torch.randint(0, 16, (n, k), generator=g, dtype=torch.int32)
        packed = (idx[:, 0::2] | (idx[:, 1::2] << 4)).to(torch.uint8).view(torch.int8)
        self.w_packed = packed.to(device)
        group_abs = torch.rand((n, k // gsz), generator=g) * 9e-3 + 1e-3
        # Channel scale so that |codebook| * relative group scale spans +-127.
        self.c_s = (group_abs.amax(dim=1) * 8.0 / 127.0).to(device)
        rel = group_abs / self.c_s.cpu()[:, None]
        self.g_s = rel.to(torch.float8_e4m3fn).view(torch.uint8).to(device)
        self.codebook = (torch.arange(16, dtype=torch.float32) - 8.0).to(device)
        self.out_host = torch.empty((m, n), dtype=torch.bfloat16,
                                    pin_memory=device.type == "cuda")
        # quantize, then (decode, GEMM) per weight chunk
        self.launches_per_step = 1 + 2 * _chunks(n, k)
        self.dominant = "gemm_i8"
        self.h2d_bytes = self.x_host.numel() * 2
        self.d2h_bytes = self.out_host.numel() * 2

    def step(self, ev=None):
        if ev:
            ev[0].record()
        xq, xs = self._C.turing_bf16_int8_convrot_quantize(self.x)
        if ev:
            ev[1].record()
        out = self._C.turing_codebook_w4a8_linear(xq, self.w_packed, xs, self.g_s, self.c_s,
                                                  self.codebook, None, self.config["group_size"])
        if ev:
            ev[2].record()
        return out

    def step_e2e(self):
        x = self.x_host.to(self.x.device, non_blocking=True)
        xq, xs = self.kernel.turing_bf16_int8_convrot_quantize(x)
        out = self.kernel.turing_codebook_w4a8_linear(xq, self.w_packed, xs, self.g_s, self.c_s,
                                                      self.codebook, None,
                                                      self.config["group_size"])
        self.out_host.copy_(out, non_blocking=True)
        return out

    cpu_sample_desc = ("rows of X, full N and K (ConvRot oracle + oracle codebook decode + "
                       "torch fp32 dequantize-then-matmul)")

    def roofline(self, dom_ms, peaks):
        return LinearWorkload.roofline(self, dom_ms, peaks)

    def cpu_reference_step(self, rows: int):
        import numpy as np

        import oracle

        xs = self.x_host[:rows]
        q, s = oracle.convrot_quantize(xs.view(torch.int16).numpy().view(np.uint16))
        out = (torch.from_numpy(q).float() @ self.w_cpu.t()) * torch.from_numpy(s) \
            * self.c_s_cpu[None, :]
        return out.to(torch.bfloat16), 2.0 * rows * self.config["n"] * self.config["k"]

    def prepare_cpu(self):
        import oracle

        w8 = oracle.codebook_decode(self.w_packed.cpu().numpy(), self.g_s.cpu().numpy(),
                                    self.codebook.cpu().numpy(), self.config["group_size"])
        self.w_cpu = torch.from_numpy(w8).float()
        self.c_s_cpu = self.c_s.cpu()


class W4A4FFNWorkload:
    """the W4A4 ConvRot FFN pair.  INT4 activations use
    the reference's per-token scales (absmax / 7, convrot_quant.cu:409-433) and
    the weights per-channel scales (dispatch.py:907-909): the config's group-64
    fp16 scales are only validated by the reference, not used."""

    name = "w4a4_ffn"
    n_events = 4  # the step continues after the timed up projection
    config = {"workload": "w4a4_convrot_ffn (BASELINE configs[3])", "m": 32760, "dim": 5120,
              "ffn": 13824, "rotation": 256, "activation": "per-token int4 (ConvRot)",
              "weight": "int4 per-channel", "between": "GELU-tanh fused into the down "
              "projection's INT4 quantizer",
              "group_scales": "not built; parity unpinned: the config's group-64 fp16 scales "
                              "are only validated by the reference's route (dispatch.py:746-806 "
                              "requires quant_group_size == 64, then uses per-token activation "
                              "and per-channel weight scales); measured on that layout, with the "
                              "W4A4 GEMM pinned to the restated formula (comfy-kitchen absent)"}

    def __init__(self, device, seed):
        import comfyui_turing_utils_kernel as kernel
        from comfyui_turing_utils_kernel import _C

        self.kernel, self._C = kernel, _C
        m, d, f = self.config["m"], self.config["dim"], self.config["ffn"]
        self.ops = 2.0 * 2.0 * m * d * f
        self.dom_ops = 2.0 * m * d * f  # the up projection, timed on its own
        g = torch.Generator().manual_seed(seed)
        x = torch.randn((m, d), generator=g)
        idx = torch.randperm(d, generator=g)[: int(round(d * 0.005))]
        x[:, idx] *= 20.0
        x = x.to(torch.bfloat16)
        self.x_host = x.pin_memory() if device.type == "cuda" else x
        self.x = self.x_host.to(device)

        def pack(rows, cols):
            v = torch.randint(-8, 8, (rows, cols), generator=g, dtype=torch.int32)
            return ((v[:, 0::2] & 0xF) | ((v[:, 1::2] & 0xF) << 4)).to(torch.uint8).view(torch.int8)

        self.w_up = pack(f, d).to(device)
        self.w_down = pack(d, f).to(device)
        self.s_up = (torch.rand((f,), generator=g) * 4e-3 + 1e-3).to(device)
        self.s_down = (torch.rand((d,), generator=g) * 4e-3 + 1e-3).to(device)
        self.b_up = (torch.randn((f,), generator=g) * 0.02).to(device)
        self.b_down = (torch.randn((d,), generator=g) * 0.02).to(device)
        self.out_host = torch.empty((m, d), dtype=torch.bfloat16,
                                    pin_memory=device.type == "cuda")
        # quantize, W4A4 up (activation unpack + (unpack, GEMM) per weight chunk),
        # GELU quantize, W4A4 down (the same).
        self.launches_per_step = 1 + (1 + 2 * _chunks(f, d)) + 1 + (1 + 2 * _chunks(d, f))
        self.dominant = "gemm_i8"
        self.h2d_bytes = self.x_host.numel() * 2
        self.d2h_bytes = self.out_host.numel() * 2

    def _ffn(self, x, ev=None, public=False):
        K = self.kernel if public else self._C
        if ev:
            ev[0].record()
        q, s = K.turing_bf16_int4_convrot_quantize(x)
        if ev:
            ev[1].record()
        h = K.turing_int4_linear(q, self.w_up, s.reshape(-1), self.s_up, self.b_up)
        if ev:
            ev[2].record()
        q2, s2 = K.turing_bf16_gelu_int4_convrot_quantize(h)
        out = K.turing_int4_linear(q2, self.w_down, s2.reshape(-1), self.s_down, self.b_down)
        if ev:
            ev[3].record()
        return out

    def step(self, ev=None):
        return self._ffn(self.x, ev)

    def step_e2e(self):
        x = self.x_host.to(self.x.device, non_blocking=True)
        out = self._ffn(x, public=True)
        self.out_host.copy_(out, non_blocking=True)
        return out

    cpu_sample_desc = ("rows of X through both projections (ConvRot INT4 oracle, torch fp32 "
                       "dequantize-then-matmul, GELU-fused INT4 oracle)")

    def roofline(self, dom_ms, peaks):
        int8_peak = 2.0 * peaks["bf16_tflops"]
        achieved = self.dom_ops / (dom_ms * 1e-3) / 1e12
        return {"kernel": self.dominant, "bound": "tensor", "achieved": round(achieved, 1),
                "peak": round(int8_peak, 1), "unit": "TOPS", "frac": round(achieved / int8_peak, 4),
                "peak_source": f"2 x {peaks['source']} dense bf16 TFLOP/s (MEASURED_PEAKS.json "
                               "bf16_tflops); dense INT8 = 2 x BF16 on B200",
                "kernel_ms": round(dom_ms, 4),
                "timed": "W4A4 up projection (INT4 unpacks + tcgen05 INT8 GEMM)"}

    def cpu_reference_step(self, rows: int):
        import numpy as np

        import oracle

        def lin(q_packed, s, w, ws, b, k):
            a = torch.from_numpy(oracle.unpack_int4(q_packed, k)).float()
            return (a @ w.t()) * torch.from_numpy(np.reshape(s, (-1, 1))) * ws[None, :] + b[None, :]

        d, f = self.config["dim"], self.config["ffn"]
        xs = self.x_host[:rows]
        q, s = oracle.convrot_quantize(xs.view(torch.int16).numpy().view(np.uint16), int4=True)
        h = lin(q, s, self.w_up_cpu, self.s_up_cpu, self.b_up_cpu, d).to(torch.bfloat16)
        q2, s2 = oracle.convrot_quantize(h.view(torch.int16).numpy().view(np.uint16), int4=True,
                                         act="gelu")
        out = lin(q2, s2, self.w_down_cpu, self.s_down_cpu, self.b_down_cpu, f)
        return out.to(torch.bfloat16), 2.0 * 2.0 * rows * d * f

    def prepare_cpu(self):
        import oracle

        d, f = self.config["dim"], self.config["ffn"]
        self.w_up_cpu = torch.from_numpy(oracle.unpack_int4(self.w_up.cpu().numpy(), d)).float()
        self.w_down_cpu = torch.from_numpy(oracle.unpack_int4(self.w_down.cpu().numpy(), f)).float()
        self.s_up_cpu, self.s_down_cpu = self.s_up.cpu(), self.s_down.cpu()
        self.b_up_cpu, self.b_down_cpu = self.b_up.cpu(), self.b_down.cpu()


class AttentionWorkload:
    name = "attention"
    config = {"workload": "sage_int8_attention (BASELINE configs[1])", "batch": 1, "heads": 40,
              "seq_len": 32760, "head_dim": 128, "layout": "HND", "causal": False,
              "q_quant": "int8 per 16-token warp tile", "k_quant": "int8 per 64-token block",
              "k_smoothing": True, "pv": "bf16 P x bf16 V, fp32 accumulation"}

    def __init__(self, device, seed, heads=None):
        from comfyui_turing_utils_kernel import turing_sage
        from comfyui_turing_utils_kernel.turing_sage import core

        self.ts, self.core = turing_sage, core
        if heads is not None and heads != self.config["heads"]:
            # Fewer heads: a smaller case of the same kernel (profiling captures).
            self.config = dict(self.config, heads=heads,
                               workload=f"sage_int8_attention, configs[1] shape with {heads} heads")
            self.name = f"attention_h{heads}"  # no committed traffic figure for this size
        B, H, L, D = (self.config[k] for k in ("batch", "heads", "seq_len", "head_dim"))
        self.ops = 4.0 * B * H * L * L * D
        g = torch.Generator(device=device).manual_seed(seed)
        self.q = torch.randn((B, H, L, D), generator=g, device=device).to(torch.bfloat16)
        k = torch.randn((B, H, L, D), generator=g, device=device)
        k += torch.randn((B, H, 1, D), generator=g, device=device) * 2.0
        self.k = k.to(torch.bfloat16)
        del k
        self.v = torch.randn((B, H, L, D), generator=g, device=device).to(torch.bfloat16)
        self.host = [_host(t) for t in (self.q, self.k, self.v)]
        self.out_host = _host(torch.empty_like(self.host[0]))
        self.launches_per_step = 4  # Q quant, K token mean, K quant, attention
        self.dominant = "sage_attn"
        self.h2d_bytes = sum(t.numel() * 2 for t in self.host)
        self.d2h_bytes = self.out_host.numel() * 2

    def step(self, ev=None):
        if ev:
            ev[0].record()
        pre = self.core.prequantize_sageattn(self.q, self.k, self.v, smooth_k=True)
        if ev:
            ev[1].record()
        out = self.core.sageattn_from_prequantized(pre)
        if ev:
            ev[2].record()
        return out

    def step_e2e(self):
        dev = self.q.device
        q, k, v = (t.to(dev, non_blocking=True) for t in self.host)
        out = self.ts.sageattn(q, k, v, tensor_layout="HND", smooth_k=True)
        self.out_host.copy_(out, non_blocking=True)
        return out

    def roofline(self, dom_ms, peaks):
        int8_peak = 2.0 * peaks["bf16_tflops"]
        achieved = self.ops / (dom_ms * 1e-3) / 1e12
        # QK^T runs at the INT8 rate, PV at the 16-bit rate: mixed floor.
        half = self.ops / 2
        floor_ms = (half / (int8_peak * 1e12) + half / (peaks["bf16_tflops"] * 1e12)) * 1e3
        return {"kernel": self.dominant, "bound": "tensor", "achieved": round(achieved, 1),
                "peak": round(int8_peak, 1), "unit": "TOPS", "frac": round(achieved / int8_peak, 4),
                "peak_source": f"2 x {peaks['source']} dense bf16 TFLOP/s (MEASURED_PEAKS.json "
                               "bf16_tflops); dense INT8 = 2 x BF16 on B200",
                "mixed_floor_ms": round(floor_ms, 3),
                "frac_of_mixed_floor": round(floor_ms / dom_ms, 4),
                "kernel_ms": round(dom_ms, 4)}

    def prepare_cpu(self):
        self.q_cpu, self.k_cpu, self.v_cpu = (t[0].float() for t in self.host[:3])

    def cpu_reference_step(self, rows: int):
        """Reference CPU path (validate_compatible.py:540-546): fp32 SDPA of
        `rows` query rows of one head against all keys."""
        h = self._cpu_head = (getattr(self, "_cpu_head", -1) + 1) % self.config["heads"]
        q = self.q_cpu[h:h + 1, :rows]
        out = torch.nn.functional.scaled_dot_product_attention(
            q[None], self.k_cpu[h:h + 1][None], self.v_cpu[h:h + 1][None])
        return out, 4.0 * rows * self.config["seq_len"] * self.config["head_dim"]

    cpu_sample_desc = "query rows of one head (cycling heads) vs all 32760 keys, fp32 SDPA"


class AttentionRopeWorkload(AttentionWorkload):
    """configs[1] attention fed by the fused RMSNorm + RoPE + INT8 Q/K prologue
    (sage/qk_preprocess.cu; the Wan self-attention normalizes Q and K over the
    whole row and rotates every channel pair per token)."""
    name = "attention_rope"
    config = dict(AttentionWorkload.config,
                  workload="sage_int8_attention (BASELINE configs[1]) behind the fused "
                           "RMSNorm(row)+RoPE+INT8 Q/K prologue",
                  k_smoothing=False, norm_scope="row", rope="interleaved, rot_dim 128, "
                  "per-token 2x2 rotations [1, L, 1, 64, 2, 2] bf16")

    def __init__(self, device, seed, heads=None):
        super().__init__(device, seed, heads=heads)
        self.name = "attention_rope" if heads in (None, 40) else f"attention_rope_h{heads}"
        B, H, L, D = (self.config[k] for k in ("batch", "heads", "seq_len", "head_dim"))
        g = torch.Generator(device=device).manual_seed(seed + 1)
        self.qn = (torch.rand((H * D,), generator=g, device=device) + 0.5).to(torch.bfloat16)
        self.kn = (torch.rand((H * D,), generator=g, device=device) + 0.5).to(torch.bfloat16)
        ang = torch.rand((1, L, 1, D // 2, 1, 1), generator=g, device=device) * 6.283
        c, s_ = torch.cos(ang), torch.sin(ang)
        self.freqs = torch.cat([torch.cat([c, -s_], -1), torch.cat([s_, c], -1)], -2).to(
            torch.bfloat16)
        self.host += [_host(t) for t in (self.qn, self.kn, self.freqs)]
        self.h2d_bytes = sum(t.numel() * t.element_size() for t in self.host)
        self.launches_per_step = 3  # row RRMS, fused Q/K prologue, attention
        # Algorithmic bytes of the prologue: Q and K read once, INT8 codes and
        # fp32 scales written, the rotations and norm weights read.
        n = B * H * L * D
        self.prologue_bytes = (2 * n * 2 + 2 * n + 4 * B * H * ((L + 63) // 64) * 5
                               + self.freqs.numel() * 2 + 2 * H * D * 2)

    def _prologue(self, q, k, qn, kn, fr):
        return self.ts.prequantize_rms_rope_qk(q, k, qn, kn, fr, epsilon=1e-6, rot_dim=128,
                                               norm_scope="row")

    def step(self, ev=None):
        if ev:
            ev[0].record()
        qk = self._prologue(self.q, self.k, self.qn, self.kn, self.freqs)
        pre = self.ts.prequantize_sageattn_from_qk(qk, self.v)
        if ev:
            ev[1].record()
        out = self.core.sageattn_from_prequantized(pre)
        if ev:
            ev[2].record()
        return out

    def step_e2e(self):
        dev = self.q.device
        q, k, v, qn, kn, fr = (t.to(dev, non_blocking=True) for t in self.host)
        pre = self.ts.prequantize_sageattn_from_qk(self._prologue(q, k, qn, kn, fr), v)
        out = self.ts.sageattn_from_prequantized(pre)
        self.out_host.copy_(out, non_blocking=True)
        return out

    def aux_roofline(self, pro_ms, peaks):
        achieved = self.prologue_bytes / (pro_ms * 1e-3) / 1e9
        return {"prologue": {"kernel": "qk_rms_rope (+ row_rrms)", "bound": "hbm",
                             "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                             "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                             "algorithmic_bytes": self.prologue_bytes,
                             "ms": round(pro_ms, 4)}}

    def prepare_cpu(self):
        super().prepare_cpu()
        B, H, L, D = (self.config[k] for k in ("batch", "heads", "seq_len", "head_dim"))
        self.qn_cpu, self.kn_cpu = self.host[3].float().view(H, D), self.host[4].float().view(H, D)
        self.fr_cpu = self.host[5].float().view(L, D // 2, 2, 2)
        # Row RRMS over all heads (the reference's norm_scope "row").
        self.q_rrms_cpu = torch.rsqrt(self.q_cpu.pow(2).mean(dim=(0, 2)) + 1e-6)
        self.k_rrms_cpu = torch.rsqrt(self.k_cpu.pow(2).mean(dim=(0, 2)) + 1e-6)

    def _norm_rope(self, x, rrms, w, tokens):
        n = (x * rrms[tokens, None] * w).view(x.shape[0], -1, 2)
        f = self.fr_cpu[tokens]
        return torch.einsum("tprc,tpc->tpr", f, n).reshape(x.shape)

    def cpu_reference_step(self, rows: int):
        """RMSNorm + RoPE (fp32) of `rows` query rows and all keys of one head,
        then the fp32 SDPA of the attention arm."""
        H, L = self.config["heads"], self.config["seq_len"]
        h = self._cpu_head = (getattr(self, "_cpu_head", -1) + 1) % H
        qt, kt = torch.arange(rows), torch.arange(L)
        q = self._norm_rope(self.q_cpu[h, :rows], self.q_rrms_cpu, self.qn_cpu[h], qt)
        k = self._norm_rope(self.k_cpu[h], self.k_rrms_cpu, self.kn_cpu[h], kt)
        out = torch.nn.functional.scaled_dot_product_attention(q[None, None], k[None, None],
                                                               self.v_cpu[h][None, None])
        return out, 4.0 * rows * L * self.config["head_dim"]

    cpu_sample_desc = ("query rows of one head (cycling heads): fp32 row RMSNorm + RoPE of "
                       "those rows and all 32760 keys, then fp32 SDPA")


class W8A8AttentionWorkload(AttentionWorkload):
    """configs[1] attention through the dense W8A8-PV path (the loader's
    default ``w8a8`` backend, turing_sage/core.py:656-708): rotated and
    anchored INT8 Q/K, channel-wise INT8 V, P packed to u8 codes."""
    name = "w8a8_attention"
    config = dict(AttentionWorkload.config,
                  workload="w8a8_pv_attention (BASELINE configs[1] shape, dense W8A8 backend)",
                  k_smoothing="anchor row (conditional)", q_quant="int8 per 16-token warp tile, "
                  "randomized Hadamard", k_quant="int8 per 64-token block, randomized Hadamard",
                  pv="u8 P codes x int8 V codes (exact, fp16 tensor path), fp32 accumulation")

    def __init__(self, device, seed, heads=None):
        super().__init__(device, seed, heads=heads)
        self.name = "w8a8_attention" if heads in (None, 40) else f"w8a8_attention_h{heads}"
        # K anchor, rotated Q/K, V amax, V codes, V scale, attention.
        self.launches_per_step = 6

    def step(self, ev=None):
        if ev:
            ev[0].record()
        pre = self.core.prequantize_sol_sageattn(self.q, self.k, self.v, use_w8a8=True,
                                                 force_dense=True)
        if ev:
            ev[1].record()
        out = self.core.sol_sparse_sageattn_from_prequantized(pre)
        if ev:
            ev[2].record()
        return out

    def step_e2e(self):
        dev = self.q.device
        q, k, v = (t.to(dev, non_blocking=True) for t in self.host)
        out = self.ts.w8a8attn(q, k, v, tensor_layout="HND")
        self.out_host.copy_(out, non_blocking=True)
        return out


class DiTBlockWorkload:
    """one Wan2.1-14B-shaped DiT block (dim 5120, 40 heads
    of 128, FFN 13824, L = 75600 video tokens, 512 text tokens, batch 1) on
    W8A8 ConvRot linears, the fused Q/K prologue and Sage INT8 attention,
    tensor-parallel over the torchrun ranks (comfyui_turing_utils_kernel.
    dit_block).  Metric: block tokens/s = L / block time, max over ranks."""
    name = "dit_block"
    unit = "tokens/s"
    unit_scale = 1.0
    scaling = "strong"
    n_events = 4          # step start, self-attention start, end, step end
    dominant = "sage_attn"

    def __init__(self, device, world=1, rank=0, tokens=None, cpu_only=False, use_graph=True,
                 max_chunks=4, parallel="a2a"):
        from comfyui_turing_utils_kernel import dit_block as db

        self.db = db
        self.cfg = db.BlockConfig()
        self.L, self.Lc = tokens or 75600, 512
        self.world, self.rank = world, rank
        # "a2a": token shards for the linears, head shards for self-attention,
        # two all-to-alls per block (full weights on every rank); "tp":
        # Megatron tensor + sequence parallel.  One rank: the same block.
        self.parallel = parallel if world > 1 else "a2a"
        a2a = self.parallel == "a2a"
        self.plan = db.shard_plan(self.cfg, 1 if a2a else world, 0 if a2a else rank)
        self.nattn = self.cfg.heads // world if a2a else self.plan.nattn
        # The committed traffic figure is for all 40 heads at L = 75600; a
        # launch's bytes are proportional to its heads.
        self.traffic_scale = self.nattn / self.cfg.heads if self.L == 75600 else None
        self.ops = db.block_ops(self.cfg, self.L, self.Lc)  # whole block, all ranks
        self.work = float(self.L)                             # tokens per step
        self.config = {"workload": "Wan2.1-14B DiT block (BASELINE configs[4])",
                       "dim": self.cfg.dim, "heads": self.cfg.heads, "head_dim": self.cfg.head_dim,
                       "ffn": self.cfg.ffn, "tokens": self.L, "text_tokens": self.Lc, "batch": 1,
                       "block_tops_per_step": round(self.ops / 1e12, 2),
                       "linears": "W8A8 ConvRot, per-channel weights", "attention": "Sage INT8",
                       "norms": "LayerNorm+AdaLN; row RMSNorm + RoPE fused into Q/K INT8"}
        if cpu_only:
            return
        import torch.distributed as tdist

        self.weights = db.make_weights(self.cfg, self.plan, seed=0, device=device)
        x = self.full_x(device)
        # Each rank holds (and is timed on) its own tokens.
        self.seq = None
        if a2a:
            if world > 1:
                self.seq = db.SeqShards.make(self.L, world, rank, tdist.group.WORLD)
            t0, t1 = self.seq.bounds[rank] if self.seq else (0, self.L)
            self.rows = torch.arange(t0, t1)
        else:
            self.rows = db.local_rows(self.L, world, rank, db.token_chunks(self.L, world))
        self.x = x[self.rows.to(device)].contiguous()
        del x
        g = torch.Generator(device=device).manual_seed(3)
        self.ctx = torch.randn((self.Lc, self.cfg.dim), generator=g, device=device).to(torch.bfloat16)
        self.freqs = db.rope_freqs(self.L, self.cfg.head_dim, seed=2, device=device)
        self.kops = db.KernelOps()
        self.block = db.DiTBlock(self.cfg, self.weights, self.plan, self.kops,
                                 group=tdist.group.WORLD if world > 1 and not a2a else None,
                                 max_chunks=max_chunks, seq=self.seq)
        self.config["token_chunks"] = 1 if a2a else db.token_chunks(self.L, world, max_chunks)
        self.host = [t.cpu().pin_memory() for t in (self.x, self.ctx)]
        self.out_host = torch.empty_like(self.host[0]).pin_memory()
        self.h2d_bytes = sum(t.numel() * 2 for t in self.host)
        self.d2h_bytes = self.out_host.numel() * 2
        before = self.kops.launches
        self.block.forward(self.x, self.ctx, self.freqs, L=self.L)
        self.launches_per_step = self.kops.launches - before
        self.graph = None
        if use_graph:
            self._capture()

    def full_x(self, device):
        """All L tokens of the block input (seeded; every rank makes the same)."""
        g = torch.Generator(device=device).manual_seed(1)
        return torch.randn((self.L, self.cfg.dim), generator=g, device=device).to(torch.bfloat16)

    def parity(self, out, samples=256):
        """Multi-GPU numerics on a seeded sample of output tokens: each rank
        contributes the sampled rows it owns, rank 0 compares them (as the
        residual branches' sum, out - x) with the fp32 reference block at
        one rank (dit_block.reference_rows: dequantized weights, unquantized
        activations) and, when it holds the full weights (the all-to-all
        layout), with its own one-GPU kernel block, bit for bit."""
        import torch.distributed as tdist

        db, dev = self.db, self.x.device
        idx = torch.randperm(self.L, generator=torch.Generator().manual_seed(7))[:samples]
        idx = idx.sort().values
        pos = torch.full((self.L,), -1, dtype=torch.long)
        pos[self.rows] = torch.arange(self.rows.numel())
        mine = pos[idx] >= 0
        rows = torch.zeros((idx.numel(), self.cfg.dim), dtype=torch.float32, device=dev)
        rows[mine.to(dev)] = out[pos[idx][mine].to(dev)].float()
        if self.world > 1:
            tdist.all_reduce(rows)   # each sampled row is owned by exactly one rank
        if self.rank != 0:
            return None
        x = self.full_x(dev)
        full_w = self.weights if self.plan.world == 1 else db.make_weights(
            self.cfg, db.shard_plan(self.cfg, 1, 0), seed=0, device=dev)
        ref = db.reference_rows(self.cfg, full_w, x, self.ctx, self.freqs, idx.to(dev))
        xi = x[idx.to(dev)].float()
        d_out, d_ref = rows - xi, ref - xi
        res = {"sample_tokens": int(idx.numel()),
               "vs_fp32_reference": {
                   "rel_l2": round(float((d_out - d_ref).norm() / d_ref.norm()), 6),
                   "cos": round(float(torch.nn.functional.cosine_similarity(
                       d_out.flatten(), d_ref.flatten(), dim=0)), 6),
                   "on": "out - x (the three residual branches)",
                   "bound": "rel_l2 <= 3e-2, cos >= 0.999 (tests/test_gpu_dit_block.py)"}}
        if self.world > 1 and self.plan.world == 1:
            one = db.DiTBlock(self.cfg, self.weights, self.plan, db.KernelOps()).forward(
                x, self.ctx, self.freqs)[idx.to(dev)].float()
            res["vs_one_gpu_kernel_block"] = {
                "identical_tokens": int((one == rows).all(dim=1).sum()),
                "max_abs_diff": float((one - rows).abs().max())}
        return res

    def phases(self, calls: int):
        """Per-phase device time of `calls` eager block forwards
        (comfyui_turing_utils_kernel.profiling): ms per forward, max over
        ranks (every rank runs the same forwards and collectives)."""
        from comfyui_turing_utils_kernel import profiling

        prof = profiling.CudaPhaseProfiler(calls)
        saved, self.db.PROFILER = self.db.PROFILER, prof
        try:
            for _ in range(calls):
                self.block.forward(self.x, self.ctx, self.freqs, L=self.L)
            torch.cuda.synchronize()
        finally:
            self.db.PROFILER = saved
        names = sorted(prof.last_report)
        per = torch.tensor([prof.last_report[n][1] / calls for n in names], dtype=torch.float64,
                           device=self.x.device)
        if self.world > 1:
            import torch.distributed as tdist

            tdist.all_reduce(per, op=tdist.ReduceOp.MAX)
        return {"eager_forwards": calls, "ms_per_forward_max_over_ranks":
                {n: round(float(v), 4) for n, v in zip(names, per.tolist())}}

    def _capture(self):
        """Capture one block forward (kernels and NCCL collectives) in a CUDA
        graph; a step then replays it, without per-launch host work."""
        self.attn_events = (torch.cuda.Event(enable_timing=True),
                            torch.cuda.Event(enable_timing=True))
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self.block.forward(self.x, self.ctx, self.freqs, L=self.L)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.graph_out = self.block.forward(self.x, self.ctx, self.freqs, L=self.L)
        torch.cuda.synchronize()
        self._dom = None

    def dom_ms(self, ev):
        """Self-attention kernel time of a step.  Events recorded inside a
        graph cannot be timed, so in graph mode one eager block forward with
        the events around the same launch runs after the timed steps (every
        rank, so the collectives stay matched)."""
        if self.graph is None:
            return ev[1].elapsed_time(ev[2])
        if self._dom is None:
            self.kops.event_pair = self.attn_events
            self.block.forward(self.x, self.ctx, self.freqs, L=self.L)
            self.kops.event_pair = None
            torch.cuda.synchronize()
            self._dom = self.attn_events[0].elapsed_time(self.attn_events[1])
        return self._dom

    def parallelism(self, world):
        if world > 1 and self.parallel == "a2a":
            return (f"all-to-all sequence parallel x{world}: token shards "
                    f"{self.seq.sizes} (whole 64-token quantizer blocks) through every norm, "
                    f"linear and the cross-attention with full weights on each rank; "
                    f"{self.nattn} heads per rank for self-attention over all tokens; NCCL "
                    "all-to-all of the INT8 Q/K codes, scales and bf16 V to the head owners "
                    "and of the attention output back")
        return (f"tensor + sequence parallel x{world}: heads {list(self.plan.heads)}, FFN "
                f"columns {list(self.plan.ffn)}; each rank owns {self.x.size(0)} tokens; NCCL "
                "all-gather of the INT8 activations before Q/K/V, cross-Q and FFN-up, "
                "reduce-scatter (bf16) after O, cross-O and FFN-down, chunked to overlap the "
                "linears; all-reduce of the Q/K row sums of squares") if world > 1 else "1 GPU"

    def step(self, ev=None):
        if ev:
            ev[0].record()
        if self.graph is not None:
            self.graph.replay()
            out = self.graph_out
        else:
            if ev:
                self.kops.event_pair = (ev[1], ev[2])
            out = self.block.forward(self.x, self.ctx, self.freqs, L=self.L)
            self.kops.event_pair = None
        if ev:
            ev[3].record()
        return out

    def e2e_begin(self):
        """Starts a streaming run of step_e2e (graph mode): the first step's
        tokens go up on the input copy stream; later steps' inputs are copied
        in, and earlier steps' outputs copied out, on two copy streams while
        the block computes, through two device staging buffers each way."""
        if self.graph is None:
            return
        cur = torch.cuda.current_stream()
        if not hasattr(self, "_h2d"):
            self._h2d, self._d2h = torch.cuda.Stream(), torch.cuda.Stream()
            self._stage = [(torch.empty_like(self.x), torch.empty_like(self.ctx)) for _ in range(2)]
            self._outbuf = [torch.empty_like(self.graph_out) for _ in range(2)]
            self._ev = {k: [torch.cuda.Event() for _ in range(2)]
                        for k in ("in", "free", "out", "done")}
        for b in range(2):            # nothing pending on either buffer
            self._ev["free"][b].record(cur)
            self._ev["done"][b].record(cur)
        self._h2d.wait_stream(cur)
        with torch.cuda.stream(self._h2d):
            self._stage[0][0].copy_(self.host[0], non_blocking=True)
            self._stage[0][1].copy_(self.host[1], non_blocking=True)
            self._ev["in"][0].record()
        self._i = 0

    def e2e_finish(self):
        """The compute stream waits for the last copies (they are timed)."""
        if self.graph is None:
            return
        cur = torch.cuda.current_stream()
        cur.wait_stream(self._h2d)
        cur.wait_stream(self._d2h)

    def step_e2e(self):
        """Host tokens in, host tokens out, through the same block call (the
        captured graph reads its static input buffers).  Between e2e_begin
        and e2e_finish the copies of neighbouring steps overlap this step's
        compute (a serving loop's double buffering); every step still moves
        its whole input from pinned host memory and its whole output back."""
        if self.graph is not None:
            cur = torch.cuda.current_stream()
            ev, b, nb = self._ev, self._i % 2, (self._i + 1) % 2
            with torch.cuda.stream(self._h2d):      # the next step's input
                self._h2d.wait_event(ev["free"][nb])
                self._stage[nb][0].copy_(self.host[0], non_blocking=True)
                self._stage[nb][1].copy_(self.host[1], non_blocking=True)
                ev["in"][nb].record()
            cur.wait_event(ev["in"][b])
            self.x.copy_(self._stage[b][0])
            self.ctx.copy_(self._stage[b][1])
            ev["free"][b].record(cur)
            self.graph.replay()
            cur.wait_event(ev["done"][b])
            self._outbuf[b].copy_(self.graph_out)
            ev["out"][b].record(cur)
            with torch.cuda.stream(self._d2h):      # this step's output
                self._d2h.wait_event(ev["out"][b])
                self.out_host.copy_(self._outbuf[b], non_blocking=True)
                ev["done"][b].record()
            self._i += 1
            return self._outbuf[b]
        else:
            dev = self.x.device
            x, ctx = (t.to(dev, non_blocking=True) for t in self.host)
            out = self.block.forward(x, ctx, self.freqs, L=self.L)
        self.out_host.copy_(out, non_blocking=True)
        return out

    def roofline(self, dom_ms, peaks):
        int8_peak = 2.0 * peaks["bf16_tflops"]
        # The timed launch is the last self-attention launch of this rank's heads.
        a0, a1 = self.db.attention_launches(self.L)[-1]
        rows = a1 - a0
        ops = 4.0 * self.nattn * rows * self.L * self.cfg.head_dim
        achieved = ops / (dom_ms * 1e-3) / 1e12
        return {"kernel": f"sage_attn ({self.nattn} heads x {rows} query rows x {self.L} keys)",
                "bound": "tensor",
                "achieved": round(achieved, 1), "peak": round(int8_peak, 1), "unit": "TOPS",
                "frac": round(achieved / int8_peak, 4),
                "peak_source": f"2 x {peaks['source']} dense bf16 TFLOP/s (MEASURED_PEAKS.json)",
                "kernel_ms": round(dom_ms, 4)}

    def prepare_cpu(self):
        d, f, H, D = self.cfg.dim, self.cfg.ffn, self.cfg.heads, self.cfg.head_dim
        g = torch.Generator().manual_seed(5)
        # fp32 weights of every linear a token passes (values do not change the time).
        self.cpu_w = [torch.randn((n, k), generator=g) * 0.02
                      for n, k in ((3 * d, d), (d, d), (d, d), (d, d), (f, d), (d, f))]
        self.cpu_kv = [torch.randn((1, H, self.L, D), generator=g) for _ in range(2)]
        self.cpu_ckv = [torch.randn((1, H, self.Lc, D), generator=g) for _ in range(2)]

    def cpu_reference_step(self, rows: int):
        """`rows` tokens through the block's fp32 path: every linear, the
        self-attention of those query rows against all L keys and the
        cross-attention against the 512 text keys (LayerNorm, GELU and the
        per-block text K/V projection are under 0.1 % of the work)."""
        rows = min(rows, self.cpu_rows_cap)
        d, H, D = self.cfg.dim, self.cfg.heads, self.cfg.head_dim
        x = torch.randn((rows, d))
        wqkv, wo, wcq, wco, wup, wdown = self.cpu_w
        qkv = x @ wqkv.t()
        q = qkv[:, :d].reshape(rows, H, D).transpose(0, 1)[None]
        a = torch.nn.functional.scaled_dot_product_attention(q, *self.cpu_kv)
        x = x + a[0].transpose(0, 1).reshape(rows, d) @ wo.t()
        cq = (x @ wcq.t()).reshape(rows, H, D).transpose(0, 1)[None]
        a = torch.nn.functional.scaled_dot_product_attention(cq, *self.cpu_ckv)
        x = x + a[0].transpose(0, 1).reshape(rows, d) @ wco.t()
        x = x + torch.nn.functional.gelu(x @ wup.t(), approximate="tanh") @ wdown.t()
        return x, float(rows)  # tokens

    # Each sampled token attends to all 75600 keys: 32 tokens are ~0.1 s of CPU work.
    cpu_rows_cap = 32
    cpu_sample_desc = ("tokens through the fp32 block path (all linears; self-attention "
                       "against all 75600 keys; cross-attention against 512 text keys)")


WORKLOADS = {"linear": LinearWorkload, "attention": AttentionWorkload,
             "attention_rope": AttentionRopeWorkload, "w8a8_attention": W8A8AttentionWorkload,
             "dit_block": DiTBlockWorkload,
             "codebook": CodebookWorkload, "w4a4_ffn": W4A4FFNWorkload}


def _split(units: int, parts: int) -> list[int]:
    base, extra = divmod(units, parts)
    return [base + (1 if r < extra else 0) for r in range(parts)]


def make_workload(args, device, seed, world=1, rank=0):
    """The workload of this rank.  On several ranks the independent configs
    are sharded with no collective: the linears split their
    tokens (rows of X; the weights are replicated), the attentions their 40
    heads; the reported value is the whole config's work over the max-over-
    ranks step time ("scaling": "strong")."""
    if args.workload in ("attention", "attention_rope", "w8a8_attention"):
        if world == 1 or args.heads is not None:
            return WORKLOADS[args.workload](device, seed, heads=args.heads)
        heads = AttentionWorkload.config["heads"]
        if heads % world:
            raise ValueError(f"{heads} heads do not split evenly over {world} ranks")
        wl = WORKLOADS[args.workload](device, seed + rank, heads=heads // world)
        wl.name = args.workload                      # the committed traffic is per head
        wl.traffic_scale = 1.0 / world
        wl.config = dict(WORKLOADS[args.workload].config, heads_per_rank=heads // world)
        wl.work = wl.ops * world                     # whole config (wl.ops: this rank's heads)
        wl.scaling = "strong"
        wl.shard_desc = f"heads split over {world} ranks ({heads // world} each), no collective"
        return wl
    if args.workload == "dit_block":
        return DiTBlockWorkload(device, world, rank, tokens=args.tokens,
                                use_graph=not args.no_graph, max_chunks=args.chunks,
                                parallel=args.parallel)
    wl = WORKLOADS[args.workload](device, seed)
    if world > 1:
        m_full = wl.config["m"]
        sizes = _split(m_full, world)
        r0, m = sum(sizes[:rank]), sizes[rank]
        wl.x = wl.x[r0:r0 + m].contiguous()
        wl.x_host = wl.x_host[r0:r0 + m]
        wl.out_host = wl.out_host[r0:r0 + m]
        wl.dom_ops *= m / m_full                     # this rank's dominant kernel
        wl.h2d_bytes = wl.x_host.numel() * 2
        wl.d2h_bytes = wl.out_host.numel() * 2
        wl.config = dict(wl.config, m_per_rank=m)    # wl.ops stays the whole config's
        wl.scaling = "strong"
        wl.shard_desc = (f"tokens (rows of X) split over {world} ranks ({m} here), weights "
                         "replicated, no collective")
    return wl


def default_workload() -> str:
    # The metric's multi-GPU part is DiT-block tokens/s at 1/2/4/8 GPUs
    # (BASELINE configs[4]); the block contains the attention of configs[1] and
    # the W8A8 linears of configs[0] at full size.
    return "dit_block"


# ----------------------------------------------------------------- runners --

def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64,
                     device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_ours(args, world, rank, local):
    from comfyui_turing_utils_kernel import _lib

    device = torch.device("cuda", local)
    wl = make_workload(args, device, seed=1000 + rank, world=world, rank=rank)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    for _ in range(args.warmup):
        wl.step()
        flush.fill_(1.0)
    torch.cuda.synchronize()

    n_ev = getattr(wl, "n_events", 3)  # step start, dominant start, dominant end[, step end]
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(n_ev)] for _ in range(args.steps)]
    sampler = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize()
    with sampler:
        t_start = time.perf_counter()
        for i in range(args.steps):
            flush.fill_(1.0)  # L2 flush, outside the per-step events
            wl.step(events[i])
        torch.cuda.synchronize()
        # nvidia-smi samples every 200 ms: when the timed region is shorter
        # than ~1 s keep the same step running so the clock record covers the
        # kernels under load (reported as "region": "timed+soak").
        soak = time.perf_counter() - t_start < 1.2
        while time.perf_counter() - t_start < 1.2:
            for _ in range(20):
                wl.step()
            torch.cuda.synchronize()
    barrier(world)
    step_ms = [ev[0].elapsed_time(ev[-1]) for ev in events]
    dom_ms = [wl.dom_ms(ev) if hasattr(wl, "dom_ms") else ev[1].elapsed_time(ev[2])
              for ev in events]
    local_ms = sum(step_ms) / len(step_ms)
    ms = max_over_ranks(local_ms, world)
    dom_avg = sum(dom_ms) / len(dom_ms)

    # End to end through the public API with host buffers.
    begin, finish = (getattr(wl, "e2e_begin", lambda: None), getattr(wl, "e2e_finish", lambda: None))
    begin()
    for _ in range(max(1, args.warmup // 2)):
        wl.step_e2e()
    finish()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    begin()
    for _ in range(args.steps):
        wl.step_e2e()
    finish()
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    parity = None
    if hasattr(wl, "parity") and not args.no_parity:
        out = wl.step()
        torch.cuda.synchronize()
        parity = wl.parity(out)
        barrier(world)
    phases = wl.phases(args.phases) if args.phases and hasattr(wl, "phases") else None
    dev_err = _lib.device_error()

    peaks = load_peaks()
    roof = wl.roofline(dom_avg, peaks)
    roof["traffic"] = ncu_traffic(wl.dominant, wl.name)
    if getattr(wl, "traffic_scale", 1) is None:
        roof["traffic"] = None
    elif roof["traffic"] is not None and hasattr(wl, "traffic_scale"):
        roof["traffic"] = round(roof["traffic"] * wl.traffic_scale)
    if hasattr(wl, "aux_roofline"):
        pro = [ev[0].elapsed_time(ev[1]) for ev in events]
        roof.update(wl.aux_roofline(sum(pro) / len(pro), peaks))
    unit, scale = getattr(wl, "unit", UNIT), getattr(wl, "unit_scale", 1e12)
    # Whole-job throughput: independent shards add up (weak scaling); a
    # tensor-parallel workload's ops are already the whole job's.
    work = getattr(wl, "work", wl.ops)  # ops (TOPS) or tokens (tokens/s) per step
    job = work * (1 if getattr(wl, "scaling", "weak") == "strong" else world)
    result = {
        "metric": METRIC,
        "value": round(job / (ms * 1e-3) / scale, 2),
        "unit": unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": getattr(wl, "scaling", "weak"),
        "vs_baseline": None,
        "dtype": "int8",
        "data": "synthetic (seeded; BASELINE shapes and distributions)",
        "config": dict(wl.config, parallelism=wl.parallelism(world) if hasattr(wl, "parallelism")
                       else getattr(wl, "shard_desc", "1 GPU"),
                       l2="256 MB buffer written between steps; per-step CUDA events exclude it"),
        "impl": "ours",
        "roofline": roof,
        "e2e": {"value": round(job / (e2e_ms * 1e-3) / scale, 2), "unit": unit,
                "h2d_bytes_per_step": wl.h2d_bytes, "d2h_bytes_per_step": wl.d2h_bytes,
                "ms_per_step": round(e2e_ms, 4),
                **({"copies": "each step's input up from and output back to pinned host "
                              "memory on two copy streams, overlapping the neighbouring "
                              "steps' compute (double-buffered); first input and last "
                              "output inside the timed region"}
                   if hasattr(wl, "e2e_begin") and getattr(wl, "graph", None) is not None
                   else {})},
        "gpu_launches": wl.launches_per_step * args.steps,
        **({"block_tops": round(wl.ops / (ms * 1e-3) / 1e12, 1)} if wl.name == "dit_block" else {}),
        "clocks": dict(sampler.summary(), region="timed+soak" if soak else "timed"),
        "device_error": dev_err,
        **({"parity": parity} if parity is not None else {}),
        **({"phases": phases} if phases is not None else {}),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(wl, args)
    return result


def cpu_baseline(wl, args) -> dict:
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    wl.prepare_cpu()
    rows = min(args.cpu_rows, getattr(wl, "cpu_rows_cap", args.cpu_rows))
    wl.cpu_reference_step(min(rows, 16))  # warm-up
    # About 10 s of CPU work: repeat the row sample until the budget is used.
    t0 = time.perf_counter()
    ops, reps = 0.0, 0
    while time.perf_counter() - t0 < args.cpu_seconds:
        ops += wl.cpu_reference_step(rows)[1]
        reps += 1
    dt = time.perf_counter() - t0
    return {"value": round(ops / dt / getattr(wl, "unit_scale", 1e12), 5),
            "unit": getattr(wl, "unit", UNIT), "cores": cores, "kind": "port",
            "sample": f"{reps} x {rows} {wl.cpu_sample_desc}",
            "seconds": round(dt, 2)}


def run_reference(args, world, rank, local):
    """CPU reference arm (rank 0 only)."""
    device = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    if args.workload == "dit_block":
        wl = DiTBlockWorkload(device, world, rank, tokens=args.tokens, cpu_only=True)
    else:
        wl = make_workload(args, device, seed=1000)
    wl.prepare_cpu()
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    rows = min(args.cpu_rows, getattr(wl, "cpu_rows_cap", args.cpu_rows))
    for _ in range(args.warmup):
        wl.cpu_reference_step(min(rows, 16))
    times, total_ops = [], 0.0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        _, ops = wl.cpu_reference_step(rows)
        times.append(time.perf_counter() - t0)
        total_ops += ops
    unit, scale = getattr(wl, "unit", UNIT), getattr(wl, "unit_scale", 1e12)
    value = total_ops / sum(times) / scale
    ms = sum(times) / len(times) * 1e3
    sample = f"{rows} {wl.cpu_sample_desc} per step"
    return {
        "metric": METRIC, "value": round(value, 5), "unit": unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2),
        "higher_is_better": True, "scaling": getattr(wl, "scaling", "weak"),
        "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded; BASELINE shapes and distributions)",
        "config": dict(wl.config, parallelism="cpu"), "impl": "reference",
        "cpu_baseline": {"value": round(value, 5), "unit": unit, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 5), "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default=None, choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-rows", type=int, default=1024)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--chunks", type=int, default=4,
                    help="dit_block: most token chunks of the multi-GPU pipeline")
    ap.add_argument("--no-graph", action="store_true",
                    help="dit_block: launch the block eagerly instead of replaying a CUDA graph")
    ap.add_argument("--tokens", type=int, default=None,
                    help="dit_block video tokens (default: the config's 75600)")
    ap.add_argument("--parallel", default="a2a", choices=["a2a", "tp"],
                    help="dit_block on several GPUs: all-to-all sequence parallel (token "
                         "shards, head-sharded self-attention) or Megatron tensor parallel")
    ap.add_argument("--no-parity", action="store_true",
                    help="dit_block: skip the sampled-token check against the fp32 reference")
    ap.add_argument("--phases", type=int, default=0,
                    help="dit_block: after the timed region, time the block's phases (CUDA "
                         "events on the compute stream, so a collective counts with its "
                         "exposed time) over this many eager forwards; max over ranks")
    ap.add_argument("--heads", type=int, default=None,
                    help="attention heads (default: the config's 40); smaller cases for profiling")
    args = ap.parse_args()
    args.workload = args.workload or default_workload()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            if rank != 0:
                return
            result = run_reference(args, world, rank, local)
        else:
            result = run_ours(args, world, rank, local)
        if rank == 0:
            print(json.dumps(result), flush=True)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
