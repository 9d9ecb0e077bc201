"""Drop-in for the reference's pybind module ``comfyui_turing_utils_kernel._C``.

Same function names, argument names, defaults and checks as
kernel/csrc/bindings.cpp:851-935; the work goes through the C ABI of
libturing_b200.so (sm_100a kernels).  Outputs are allocated here with torch and
written in place by the kernels, on PyTorch's current stream of the input's
device (the reference's TorchOpContext, bindings.cpp:17-31).
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import call, float_dtype_code, ptr, stream_of


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_cuda_2d(t: torch.Tensor, name: str) -> None:
    # bindings.cpp:93-97
    _check(t.is_cuda, f"{name} must be a CUDA tensor")
    _check(t.dim() == 2, f"{name} must be 2D")
    _check(t.is_contiguous(), f"{name} must be contiguous")


def _require_blackwell(device: torch.device, what: str) -> None:
    major, _ = torch.cuda.get_device_capability(device)
    _check(major == 10, f"{what} requires an sm_100 (B200) device for this build")


def _as_f32_vec(t: torch.Tensor) -> torch.Tensor:
    return t.reshape(-1).to(torch.float32).contiguous()


# ------------------------------------------------------------------ linears

def turing_int8_linear(activation, weight, activation_scale, weight_scale, bias=None,
                       tile_policy=0, out=None):
    """bindings.cpp:371-421.  out (not in the reference): an existing bf16
    [M, N] destination with unit column stride, e.g. a row block of a larger
    buffer; its row stride is passed as the GEMM's ldo."""
    activation = activation.contiguous()
    weight = weight.contiguous()
    activation_scale = _as_f32_vec(activation_scale)
    weight_scale = _as_f32_vec(weight_scale)
    if bias is not None:
        bias = _as_f32_vec(bias)
    _check_cuda_2d(activation, "activation")
    _check_cuda_2d(weight, "weight")
    _check(activation.dtype == torch.int8 and weight.dtype == torch.int8,
           "Turing INT8 linear activation and weight must be int8")
    _check(activation.device == weight.device and activation.device == activation_scale.device
           and activation.device == weight_scale.device,
           "Turing INT8 linear tensors must use the same CUDA device")
    _check(weight.size(1) == activation.size(1), "INT8 linear K dimensions must match")
    _check(activation.size(1) % 16 == 0 and weight.size(0) % 8 == 0,
           "Turing INT8 linear requires K%16=0 and N%8=0")
    _check(activation_scale.numel() == activation.size(0),
           "activation_scale must contain one value per row")
    _check(weight_scale.numel() == weight.size(0),
           "weight_scale must contain one value per output channel")
    if bias is not None:
        _check(bias.is_cuda and bias.device == activation.device
               and bias.numel() == weight.size(0),
               "bias must contain one value per output channel on the same CUDA device")
    m, k = activation.shape
    n = weight.size(0)
    with torch.cuda.device(activation.device):
        _require_blackwell(activation.device, "turing_int8_linear")
        if out is None:
            out = torch.empty((m, n), dtype=torch.bfloat16, device=activation.device)
        else:
            _check(out.dtype == torch.bfloat16 and out.device == activation.device
                   and tuple(out.shape) == (m, n) and out.stride(1) == 1
                   and out.stride(0) >= n and out.stride(0) % 8 == 0
                   and out.data_ptr() % 16 == 0,
                   "out must be a 16-byte aligned bf16 [M, N] CUDA view with unit column stride "
                   "and a row stride that is a multiple of 8")
        call("tb_int8_linear", ptr(activation), ptr(weight), ptr(activation_scale),
             ptr(weight_scale), ptr(bias), ptr(out), m, n, k, out.stride(0), int(tile_policy),
             stream_of(activation))
    return out


def _pad_k16(activation, weight_packed):
    """Zero-pad K to a multiple of 16 (zero codes add nothing to the sums): the
    sm_100a GEMM reads K in 16-byte TMA rows, the reference accepts K % 4."""
    k = activation.size(1)
    pad = (-k) % 16
    if pad == 0:
        return activation, weight_packed
    return (torch.nn.functional.pad(activation, (0, pad)),
            torch.nn.functional.pad(weight_packed, (0, pad // 2)))


# Largest expanded int8 weight chunk (bytes) a staged W4 linear decodes before
# its GEMM.  One chunk covers every N x K of the configs (13824 x 5120 = 67.5
# MiB), so the GEMM runs once over all N-blocks instead of ending each chunk
# on a partial wave of tiles.
_WEIGHT_CHUNK_BYTES = 128 << 20


def _weight_chunk_rows(n, k):
    """Rows of the expanded weight per decode + GEMM round: all N when N x K
    int8 fits _WEIGHT_CHUNK_BYTES, else equal chunks rounded up to the GEMM's
    256-column tile.  Each output column depends only on its own weight row,
    so the chunking changes no result."""
    if n * k <= _WEIGHT_CHUNK_BYTES:
        return n
    chunks = -(-(n * k) // _WEIGHT_CHUNK_BYTES)
    rows = -(-n // chunks)
    return min(n, -(-rows // 256) * 256)


def _n_tail_linear(m, n, dev, run):
    """N-tail handling of bindings.cpp:205-259: the first N - N % 8 channels in
    one call, the last N % 8 channels padded with zero rows to 8 in a second,
    into an output of ceil(N / 8) * 8 columns that is sliced back to N."""
    padded_n = (n + 7) // 8 * 8
    out = torch.empty((m, padded_n), dtype=torch.bfloat16, device=dev)
    bulk = n // 8 * 8
    if bulk > 0:
        run(0, bulk, bulk, out)
    if bulk != n:
        run(bulk, n - bulk, 8, out)
    return out if padded_n == n else out.narrow(1, 0, n).contiguous()


def turing_w4a8_linear(activation, weight, activation_scale, weight_scale, bias=None,
                       tile_policy=0):
    """bindings.cpp:167-259: signed-nibble W4A8, weight [N, K/2] packed int8
    storage (low nibble = even column).  The weight rows are unpacked to int8
    in a bounded workspace and contracted by the tcgen05 INT8 GEMM."""
    activation = activation.contiguous()
    weight = weight.contiguous()
    activation_scale = _as_f32_vec(activation_scale)
    weight_scale = _as_f32_vec(weight_scale)
    if bias is not None:
        bias = _as_f32_vec(bias)
    _check_cuda_2d(activation, "activation")
    _check_cuda_2d(weight, "weight")
    _check(activation.dtype == torch.int8, "activation must be int8")
    _check(weight.dtype == torch.int8, "weight must be packed int8 storage")
    _check(activation.device == weight.device,
           "activation and weight must be on the same CUDA device")
    _check(activation_scale.is_cuda and weight_scale.is_cuda, "scales must be CUDA tensors")
    _check(activation_scale.device == activation.device
           and weight_scale.device == activation.device,
           "scales must be on the activation device")
    _check(activation.size(1) % 4 == 0, "activation K must be divisible by 4")
    _check(weight.size(1) * 2 == activation.size(1), "packed weight K must match activation K")
    _check(activation_scale.numel() == activation.size(0),
           "activation_scale must contain one value per row")
    _check(weight_scale.numel() == weight.size(0),
           "weight_scale must contain one value per output channel")
    if bias is not None:
        _check(bias.is_cuda and bias.device == activation.device,
               "bias must be on the activation device")
        _check(bias.numel() == weight.size(0), "bias must contain one value per output channel")
    dev = activation.device
    m = activation.size(0)
    n = weight.size(0)
    with torch.cuda.device(dev):
        _require_blackwell(dev, "turing_w4a8_linear")
        activation, weight = _pad_k16(activation, weight)
        k = activation.size(1)
        if m == 0 or n == 0:
            return torch.empty((m, n), dtype=torch.bfloat16, device=dev)

        def run(n0, count, width, out):
            w = weight.narrow(0, n0, count)
            ws = weight_scale.narrow(0, n0, count)
            b = None if bias is None else bias.narrow(0, n0, count)
            if width != count:
                w = torch.nn.functional.pad(w, (0, 0, 0, width - count))
                ws = torch.nn.functional.pad(ws, (0, width - count))
                b = None if b is None else torch.nn.functional.pad(b, (0, width - count))
            rows = _weight_chunk_rows(width, k)
            workspace = torch.empty((rows, k), dtype=torch.int8, device=dev)
            call("tb_w4a8_linear", ptr(activation), ptr(w.contiguous()), ptr(activation_scale),
                 ptr(ws.contiguous()), ptr(None if b is None else b.contiguous()), ptr(workspace),
                 rows, ptr(out.narrow(1, n0, width)), m, width, k, out.size(1),
                 int(tile_policy) if width == count else 1, stream_of(activation))

        return _n_tail_linear(m, n, dev, run)


def turing_int4_linear(activation, weight, activation_scale, weight_scale, bias=None):
    """W4A4 linear for the plugin's INT4 ConvRot path (in place of the
    comfy-kitchen int4_linear call, comfyui_turing_utils/quantization/
    dispatch.py:791-804): activation [M, K/2] and weight [N, K/2] packed signed
    4-bit codes (low nibble = even column), activation_scale [M] (absmax / 7),
    weight_scale [N]; returns bf16 [M, N] =
    bf16(((sum a4 * w4) * a_s) * w_s + bias)."""
    activation = activation.contiguous()
    weight = weight.contiguous()
    activation_scale = _as_f32_vec(activation_scale)
    weight_scale = _as_f32_vec(weight_scale)
    if bias is not None:
        bias = _as_f32_vec(bias)
    _check_cuda_2d(activation, "activation")
    _check_cuda_2d(weight, "weight")
    _check(activation.dtype == torch.int8, "activation must be packed int8 storage")
    _check(weight.dtype == torch.int8, "weight must be packed int8 storage")
    dev = activation.device
    _check(weight.device == dev and activation_scale.device == dev and weight_scale.device == dev,
           "W4A4 tensors must be on the activation device")
    _check(weight.size(1) == activation.size(1), "packed activation and weight K must match")
    _check(activation.size(1) % 2 == 0, "activation K must be divisible by 4")
    _check(activation_scale.numel() == activation.size(0),
           "activation_scale must contain one value per row")
    _check(weight_scale.numel() == weight.size(0),
           "weight_scale must contain one value per output channel")
    if bias is not None:
        _check(bias.is_cuda and bias.device == dev, "bias must be on the activation device")
        _check(bias.numel() == weight.size(0), "bias must contain one value per output channel")
    m = activation.size(0)
    n = weight.size(0)
    with torch.cuda.device(dev):
        _require_blackwell(dev, "turing_int4_linear")
        pad = (-activation.size(1)) % 8
        if pad:
            activation = torch.nn.functional.pad(activation, (0, pad))
            weight = torch.nn.functional.pad(weight, (0, pad))
        k = activation.size(1) * 2
        if m == 0 or n == 0:
            return torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        act_workspace = torch.empty((m, k), dtype=torch.int8, device=dev)

        def run(n0, count, width, out):
            w = weight.narrow(0, n0, count)
            ws = weight_scale.narrow(0, n0, count)
            b = None if bias is None else bias.narrow(0, n0, count)
            if width != count:
                w = torch.nn.functional.pad(w, (0, 0, 0, width - count))
                ws = torch.nn.functional.pad(ws, (0, width - count))
                b = None if b is None else torch.nn.functional.pad(b, (0, width - count))
            rows = _weight_chunk_rows(width, k)
            workspace = torch.empty((rows, k), dtype=torch.int8, device=dev)
            call("tb_int4_linear", ptr(activation), ptr(w.contiguous()), ptr(activation_scale),
                 ptr(ws.contiguous()), ptr(None if b is None else b.contiguous()),
                 ptr(act_workspace), ptr(workspace), rows, ptr(out.narrow(1, n0, width)), m,
                 width, k, out.size(1), stream_of(activation))

        return _n_tail_linear(m, n, dev, run)


def turing_int8_gemm_s32(activation, weight):
    """Exact INT32 accumulators [M, N] (the INT32 GEMM the plugin pairs with
    turing_dequantize_int8_bf16, dispatch.py:481-535)."""
    activation = activation.contiguous()
    weight = weight.contiguous()
    _check_cuda_2d(activation, "activation")
    _check_cuda_2d(weight, "weight")
    _check(activation.dtype == torch.int8 and weight.dtype == torch.int8,
           "INT8 GEMM activation and weight must be int8")
    _check(weight.size(1) == activation.size(1), "INT8 GEMM K dimensions must match")
    m, k = activation.shape
    n = weight.size(0)
    _check(k % 16 == 0 and n % 4 == 0, "INT8 GEMM requires K%16=0 and N%4=0")
    with torch.cuda.device(activation.device):
        _require_blackwell(activation.device, "turing_int8_gemm_s32")
        acc = torch.empty((m, n), dtype=torch.int32, device=activation.device)
        call("tb_int8_gemm_s32", ptr(activation), ptr(weight), ptr(acc), m, n, k, n,
             stream_of(activation))
    return acc


def turing_codebook_w4a8_linear(activation, weight, activation_scale, group_scale,
                                channel_scale, codebook, bias=None, group_size=16, chunk_rows=0,
                                tile_policy=0):
    """bindings.cpp:262-369.  On sm_100a every shape decodes through the bounded
    staged workspace (the reference's inline CUTLASS iterator is an sm75 tile
    policy; both forms are bit-exact with each other, validate_compatible.py:175-210)."""
    activation = activation.contiguous()
    weight = weight.contiguous()
    activation_scale = _as_f32_vec(activation_scale)
    group_scale = group_scale.contiguous()
    channel_scale = _as_f32_vec(channel_scale)
    codebook = _as_f32_vec(codebook)
    if bias is not None:
        bias = _as_f32_vec(bias)
    _check_cuda_2d(activation, "activation")
    _check_cuda_2d(weight, "weight")
    _check_cuda_2d(group_scale, "group_scale")
    _check(activation.dtype == torch.int8, "activation must be int8")
    _check(weight.dtype == torch.int8, "weight must use packed int8 storage")
    _check(group_scale.dtype == torch.uint8, "group_scale must contain raw float8_e4m3fn bytes")
    dev = activation.device
    _check(weight.device == dev and group_scale.device == dev and activation_scale.device == dev
           and channel_scale.device == dev and codebook.device == dev,
           "all codebook W4A8 tensors must use the same CUDA device")
    m, k = activation.shape
    n = weight.size(0)
    _check(m > 0 and n > 0 and k > 0, "codebook W4A8 dimensions must be positive")
    _check(k % 16 == 0 and n % 8 == 0,
           "codebook W4A8 requires K divisible by 16 and N divisible by 8")
    _check(weight.size(1) * 2 == k, "packed weight K must match activation K")
    _check(group_size >= 4 and k % group_size == 0
           and (16 % group_size == 0 or group_size % 16 == 0),
           "unsupported codebook W4A8 group_size")
    _check(group_scale.size(0) == n and group_scale.size(1) == k // group_size,
           "group_scale must have shape [N, K/group_size]")
    _check(activation_scale.numel() == m,
           "activation_scale must contain one value per activation row")
    _check(channel_scale.numel() == n, "channel_scale must contain one value per output channel")
    _check(codebook.numel() == 16, "codebook must contain 16 float32 values")
    if bias is not None:
        _check(bias.is_cuda and bias.device == dev, "bias must use the activation CUDA device")
        _check(bias.numel() == n, "bias must contain one value per output channel")
    _check(chunk_rows >= -1, "chunk_rows must be -1, 0, or a positive multiple of 8")
    inline_eligible = group_size == 16 and m > 8192 and chunk_rows <= 0
    _check(chunk_rows != -1 or inline_eligible,
           "forced inline codebook W4A8 requires group_size=16 and M>8192")
    if chunk_rows <= 0:
        chunk_rows = _weight_chunk_rows(n, k)
    else:
        _check(chunk_rows % 8 == 0, "chunk_rows must be divisible by 8")
        chunk_rows = min(n, chunk_rows)
    with torch.cuda.device(dev):
        _require_blackwell(dev, "turing_codebook_w4a8_linear")
        workspace = torch.empty((chunk_rows, k), dtype=torch.int8, device=dev)
        out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        call("tb_codebook_w4a8_linear", ptr(activation), ptr(weight), ptr(activation_scale),
             ptr(group_scale), ptr(channel_scale), ptr(codebook), ptr(bias), ptr(workspace),
             chunk_rows, ptr(out), m, n, k, int(group_size), 0, int(tile_policy),
             stream_of(activation))
    return out


def turing_dequantize_int8_bf16(accumulator, activation_scale, weight_scale, output_columns=-1):
    """bindings.cpp:423-467."""
    accumulator = accumulator.contiguous()
    activation_scale = _as_f32_vec(activation_scale)
    weight_scale = _as_f32_vec(weight_scale)
    _check_cuda_2d(accumulator, "accumulator")
    _check(accumulator.dtype == torch.int32, "accumulator must be int32")
    _check(activation_scale.is_cuda and weight_scale.is_cuda, "scales must be CUDA tensors")
    _check(accumulator.device == activation_scale.device
           and accumulator.device == weight_scale.device,
           "accumulator and scales must use the same CUDA device")
    rows, acc_cols = accumulator.shape
    if output_columns < 0:
        output_columns = acc_cols
    _check(rows > 0 and acc_cols > 0, "INT8 BF16 epilogue dimensions must be positive")
    _check(0 < output_columns <= acc_cols,
           "output_columns must be positive and no larger than the accumulator width")
    _check(activation_scale.numel() == rows,
           "activation_scale must contain one value per accumulator row")
    _check(weight_scale.numel() == 1 or weight_scale.numel() == output_columns,
           "weight_scale must be scalar or contain one value per output column")
    with torch.cuda.device(accumulator.device):
        _require_blackwell(accumulator.device, "INT8 BF16 epilogue")
        out = torch.empty((rows, output_columns), dtype=torch.bfloat16, device=accumulator.device)
        call("tb_dequantize_int8_bf16", ptr(accumulator), acc_cols, ptr(activation_scale),
             ptr(weight_scale), weight_scale.numel(), ptr(out), rows, output_columns,
             stream_of(accumulator))
    return out


def gated_residual_add_(x, y, gate=None):
    """x = bf16(x + y * gate) in place (gate [cols] or None), fp32 arithmetic
    with one rounding per operation: the DiT block's residual, which the model
    code around the plugin runs as ``x.addcmul_(y, gate)``.  Not a reference
    binding; x and y are bf16 row blocks with unit column stride."""
    _check(x.is_cuda and y.is_cuda, "gated_residual_add_: x and y must be CUDA tensors")
    _check(x.dtype == torch.bfloat16 and y.dtype == torch.bfloat16,
           "gated_residual_add_: x and y must be bfloat16")
    _check(x.dim() == 2 and x.shape == y.shape, "gated_residual_add_: x and y must be 2D, same shape")
    _check(x.stride(1) == 1 and y.stride(1) == 1, "gated_residual_add_: unit column stride required")
    if gate is not None:
        _check(gate.dtype == torch.bfloat16 and gate.numel() == x.size(1),
               "gated_residual_add_: gate must be bfloat16 with one value per column")
        gate = gate.reshape(-1).contiguous()
    with torch.cuda.device(x.device):
        call("tb_gated_residual_add", ptr(x), x.stride(0), ptr(y), y.stride(0), ptr(gate),
             x.size(0), x.size(1), stream_of(x))
    return x


# ---------------------------------------------------------- ConvRot quantizers

def _rowbuffer(input, group_size, swiglu, int4, gelu, forced_threads=0):
    input = input.contiguous()
    _check_cuda_2d(input, "input")
    label = "BF16 GELU row-buffer" if gelu else "BF16 row-buffer"
    _check(input.dtype == torch.bfloat16, f"{label} ConvRot input must be bfloat16")
    _check(group_size == 256, f"{label} ConvRot only supports group_size=256")
    rows, cols = input.shape
    _check(not swiglu or cols % 2 == 0, "SwiGLU BF16 row-buffer ConvRot input width must be even")
    hidden = cols // 2 if swiglu else cols
    _check(rows > 0 and hidden > 0 and hidden % group_size == 0,
           f"{label} ConvRot width must be positive and divisible by 256")
    with torch.cuda.device(input.device):
        _require_blackwell(input.device, f"{label} ConvRot")
        out = torch.empty((rows, hidden // 2 if int4 else hidden), dtype=torch.int8,
                          device=input.device)
        scales = torch.empty((rows, 1), dtype=torch.float32, device=input.device)
        s = stream_of(input)
        if gelu:
            call("tb_bf16_gelu_int4_convrot_quantize" if int4 else
                 "tb_bf16_gelu_int8_convrot_quantize",
                 ptr(input), rows, hidden, ptr(out), ptr(scales), s)
        elif int4:
            call("tb_bf16_int4_convrot_quantize", ptr(input), rows, hidden, int(bool(swiglu)),
                 ptr(out), ptr(scales), s)
        else:
            call("tb_bf16_int8_convrot_quantize", ptr(input), rows, hidden, int(bool(swiglu)),
                 int(forced_threads), ptr(out), ptr(scales), s)
    return out, scales


def turing_bf16_int8_convrot_quantize(input, group_size=256, swiglu=False, forced_threads=0):
    """bindings.cpp:603-646."""
    if forced_threads not in (0, 512, 768, 1024):
        raise RuntimeError("forced_threads must be 0, 512, 768, or 1024")
    return _rowbuffer(input, group_size, swiglu, False, False, forced_threads)


def turing_bf16_int4_convrot_quantize(input, group_size=256, swiglu=False):
    """bindings.cpp:648-688."""
    return _rowbuffer(input, group_size, swiglu, True, False)


def turing_bf16_gelu_int8_convrot_quantize(input, group_size=256):
    return _rowbuffer(input, group_size, False, False, True)


def turing_bf16_gelu_int4_convrot_quantize(input, group_size=256):
    return _rowbuffer(input, group_size, False, True, True)


def _staged(input, group_size, act, int4):
    input = input.contiguous()
    _check_cuda_2d(input, "input")
    _check(input.dtype in (torch.float16, torch.bfloat16), "input must be float16 or bfloat16")
    label = "SwiGLU" if act == 1 else "GELU"
    _check(group_size == 256, f"{label} staged ConvRot only supports group_size=256")
    rows, cols = input.shape
    if act == 1:
        _check(cols % 2 == 0, "SwiGLU input width must be even")
    hidden = cols // 2 if act == 1 else cols
    _check(rows > 0, f"{label} staged ConvRot requires at least one row")
    _check(hidden > 0 and hidden % group_size == 0,
           f"activated {label} width must be positive and divisible by 256")
    with torch.cuda.device(input.device):
        _require_blackwell(input.device, f"{label} staged ConvRot")
        rotated = torch.empty((rows, hidden), dtype=input.dtype, device=input.device)
        partial = torch.empty((rows, hidden // group_size), dtype=torch.float32,
                              device=input.device)
        out = torch.empty((rows, hidden // 2 if int4 else hidden), dtype=torch.int8,
                          device=input.device)
        scales = torch.empty((rows, 1), dtype=torch.float32, device=input.device)
        name = {(1, False): "tb_swiglu_int8_convrot_quantize",
                (1, True): "tb_swiglu_int4_convrot_quantize",
                (2, False): "tb_gelu_int8_convrot_quantize",
                (2, True): "tb_gelu_int4_convrot_quantize"}[(act, bool(int4))]
        call(name, ptr(input), _lib.dtype_code(input), rows, hidden, ptr(rotated), ptr(partial),
             ptr(out), ptr(scales), stream_of(input))
    return out, scales


def turing_swiglu_int8_convrot_quantize(input, group_size=256):
    return _staged(input, group_size, 1, False)


def turing_swiglu_int4_convrot_quantize(input, group_size=256):
    return _staged(input, group_size, 1, True)


def turing_gelu_int8_convrot_quantize(input, group_size=256):
    return _staged(input, group_size, 2, False)


def turing_gelu_int4_convrot_quantize(input, group_size=256):
    return _staged(input, group_size, 2, True)


def _check_float_like(t: torch.Tensor, name: str) -> None:
    _check(t.dtype in (torch.float16, torch.bfloat16, torch.float32),
           f"{name} must be float16, bfloat16, or float32")


def turing_segmented_rms_adaln(input, weight, scale, shift, segments, epsilon):
    """bindings.cpp:734-801: affine RMSNorm + segmented AdaLN modulation."""
    input = input.contiguous()
    weight = weight.contiguous()
    segments = segments.contiguous()
    _check_cuda_2d(input, "input")
    _check_float_like(input, "input")
    _check(weight.is_cuda and weight.dim() == 1 and weight.is_contiguous(),
           "weight must be a contiguous 1D CUDA tensor")
    _check(scale.is_cuda and scale.dim() == 2 and scale.stride(1) == 1,
           "scale must be a CUDA matrix with contiguous rows")
    _check(shift.is_cuda and shift.dim() == 2 and shift.stride(1) == 1,
           "shift must be a CUDA matrix with contiguous rows")
    _check(segments.is_cuda and segments.dim() == 2 and segments.is_contiguous(),
           "segments must be a contiguous 2D CUDA tensor")
    _check(segments.dtype == torch.int32 and segments.size(1) == 3,
           "segments must be int32 [start, stop, modulation_row] triples")
    dev = input.device
    _check(weight.device == dev and scale.device == dev and shift.device == dev
           and segments.device == dev,
           "all segmented RMSNorm+AdaLN tensors must use the same CUDA device")
    _check(weight.dtype == input.dtype and scale.dtype == input.dtype
           and shift.dtype == input.dtype, "weight, scale, and shift dtypes must match input")
    rows, hidden = input.shape
    _check(rows > 0 and hidden > 0, "segmented RMSNorm+AdaLN input dimensions must be positive")
    _check(weight.numel() == hidden, "RMSNorm weight length must match the input hidden dimension")
    _check(scale.size(0) > 0 and scale.size(1) == hidden, "scale must be [modulation_rows, hidden]")
    _check(shift.shape == scale.shape, "shift shape must match scale shape")
    _check(segments.size(0) > 0, "segments must contain at least one row")
    _check(math.isfinite(epsilon) and epsilon > 0.0, "RMSNorm epsilon must be finite and positive")
    with torch.cuda.device(dev):
        _require_blackwell(dev, "segmented RMSNorm+AdaLN")
        out = torch.empty_like(input)
        call("tb_segmented_rms_adaln", ptr(input), ptr(weight), ptr(scale), ptr(shift),
             ptr(segments), ptr(out), rows, hidden, scale.size(0), scale.stride(0),
             shift.stride(0), segments.size(0), float_dtype_code(input), float(epsilon),
             stream_of(input))
    return out


def turing_layer_norm_adaln(input, scale, shift, epsilon):
    """bindings.cpp:803-849: FP32-statistics LayerNorm + Wan AdaLN modulation."""
    input = input.contiguous()
    scale = scale.contiguous()
    shift = shift.contiguous()
    _check(input.is_cuda and input.dim() == 3 and input.is_contiguous(),
           "input must be contiguous CUDA [batch, sequence, hidden]")
    _check_float_like(input, "input")
    _check(scale.is_cuda and scale.dim() == 3 and scale.is_contiguous(),
           "scale must be contiguous CUDA [batch, modulation_steps, hidden]")
    _check(shift.is_cuda and shift.dim() == 3 and shift.is_contiguous(),
           "shift must be contiguous CUDA [batch, modulation_steps, hidden]")
    _check(input.device == scale.device and input.device == shift.device,
           "LayerNorm+AdaLN tensors must use the same CUDA device")
    _check(input.dtype == scale.dtype and input.dtype == shift.dtype,
           "LayerNorm+AdaLN tensor dtypes must match")
    _check(scale.shape == shift.shape, "shift shape must match scale shape")
    _check(scale.size(0) == input.size(0) and scale.size(2) == input.size(2),
           "scale must match input batch and hidden dimensions")
    _check(input.size(0) > 0 and input.size(1) > 0 and input.size(2) > 0 and scale.size(1) > 0,
           "LayerNorm+AdaLN dimensions must be positive")
    _check(math.isfinite(epsilon) and epsilon > 0.0, "LayerNorm epsilon must be finite and positive")
    with torch.cuda.device(input.device):
        _require_blackwell(input.device, "LayerNorm+AdaLN")
        out = torch.empty_like(input)
        call("tb_layer_norm_adaln", ptr(input), ptr(scale), ptr(shift), ptr(out), input.size(0),
             input.size(1), input.size(2), scale.size(1), float_dtype_code(input), float(epsilon),
             stream_of(input))
    return out
