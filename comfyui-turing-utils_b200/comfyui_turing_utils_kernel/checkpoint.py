"""ConvRot checkpoint format reader: lets a ConvRot-quantized .safetensors
checkpoint drive this package's kernels without ComfyUI.

Restates the format rules of the plugin's loader
(comfyui_turing_utils/quantization/convrot.py:37-42 constants, :82-144
legacy normalization and layer classification, :147-232 .comfy_quant JSON
tensors and safetensors header checks, :235-263 model screening, :294-371
activation configuration) with the same results and error messages, and adds
what the loader gets from ComfyUI: a bounds-checked tensor reader for the
safetensors container (8-byte little-endian header length, JSON header of
dtype / shape / data_offsets relative to the end of the header) and the
kernel call plan of every quantized layer.

Per-layer quantization metadata comes from either
  * the header: __metadata__["_quantization_metadata"] = JSON
    {"layers": {name: config}}, or
  * a U8 tensor "<name>.comfy_quant" holding the config as UTF-8 JSON.
A config names a format (int8_tensorwise, legacy int8_rowwise,
convrot_w4a4, asym_w4a8_int8); its options live at the top level or under
"params" (the top level wins).
"""
from __future__ import annotations

import dataclasses
import json
import math
import struct
from pathlib import Path
from typing import Any, Iterator

import numpy as np
import torch

FORMAT_W4 = "convrot_w4a4"
FORMAT_CODEBOOK_W4 = "asym_w4a8_int8"
FORMAT_W8 = "int8_tensorwise"
FORMAT_W8_LEGACY = "int8_rowwise"
MODEL_EXTENSIONS = (".safetensors", ".sft")
MAX_HEADER_BYTES = 128 * 1024 * 1024
MAX_CONFIG_BYTES = 1024 * 1024
QUANT_SUFFIX = ".comfy_quant"
HEADER_KEY = "_quantization_metadata"


@dataclasses.dataclass(frozen=True)
class ConvRotSummary:
    """Layer counts by (weight, activation) kind (convrot.py:45-50)."""
    w4a4: int = 0
    w4a8: int = 0
    codebook_w4a8: int = 0
    w8a8: int = 0


# --------------------------------------------------------------- configs --

def _params_of(config: dict, layer: str) -> dict:
    params = config.get("params", {})
    if not isinstance(params, dict):
        raise ValueError(f"ConvRot layer {layer} has non-object params metadata")
    return params


def _option(config: dict, layer: str, name: str, default: Any) -> Any:
    if name in config:
        return config[name]
    return _params_of(config, layer).get(name, default)


def _is_int(value: Any) -> bool:
    return isinstance(value, int) and not isinstance(value, bool)


def _check_activation(layer: str, kind: str, dtype: Any, expected: str) -> None:
    if dtype not in ("int4", "int8"):
        raise ValueError(f"ConvRot {kind} layer {layer} declares unsupported "
                         f"linear_dtype={dtype!r}; expected {expected}")


def classify_config(config: Any, layer: str, force_int8_gemm: bool) -> tuple[str, str] | None:
    """(weight kind, activation dtype) of one layer's config, or None for a
    layer that is not ConvRot-quantized (convrot.py:82-144).  Weight kinds:
    "w8" (int8_tensorwise), "w4" (convrot_w4a4), "w4_codebook"
    (asym_w4a8_int8).  A legacy W8 config (format absent or int8_rowwise,
    convrot and per_row true) is rewritten in place to int8_tensorwise."""
    if not isinstance(config, dict):
        raise ValueError(f"Quantization metadata for layer {layer} must be an object")
    fmt = config.get("format")
    if (fmt in (None, FORMAT_W8_LEGACY) and _option(config, layer, "convrot", False) is True
            and _option(config, layer, "per_row", False) is True):
        config["format"] = fmt = FORMAT_W8
    _params_of(config, layer)

    if fmt == FORMAT_W4:
        dtype = _option(config, layer, "linear_dtype", "int4")
        _check_activation(layer, "W4", dtype, "'int4' or 'int8'")
        return ("w4", "int8" if force_int8_gemm else dtype)

    if fmt == FORMAT_CODEBOOK_W4:
        if _option(config, layer, "convrot", True) is not True:
            raise ValueError(f"Grouped-codebook W4A8 layer {layer} must declare convrot=true")
        group = _option(config, layer, "group_size", 16)
        if not _is_int(group) or group < 4:
            raise ValueError(f"Grouped-codebook W4A8 layer {layer} has invalid group_size={group!r}")
        if _option(config, layer, "convrot_groupsize", 256) != 256:
            raise ValueError(f"Grouped-codebook W4A8 layer {layer} requires convrot_groupsize=256")
        return ("w4_codebook", "int8")

    convrot = _option(config, layer, "convrot", False)
    if not isinstance(convrot, bool):
        raise ValueError(f"Quantized layer {layer} has non-boolean convrot={convrot!r}")
    if not convrot:
        return None
    if fmt != FORMAT_W8:
        raise ValueError(f"ConvRot layer {layer} uses unsupported weight format {fmt!r}")
    dtype = _option(config, layer, "linear_dtype", "int8")
    _check_activation(layer, "W8", dtype, "'int8'")
    if dtype != "int8" and not force_int8_gemm:
        raise ValueError(f"ConvRot W8 layer {layer} cannot use linear_dtype={dtype!r}; "
                         "W8 ConvRot supports INT8 activations only")
    return ("w8", "int8")


def decode_quant_tensor(value: torch.Tensor, key: str) -> dict:
    """The JSON object stored in a .comfy_quant U8 tensor (convrot.py:147-156)."""
    if not isinstance(value, torch.Tensor):
        raise TypeError(f"{key} must be a JSON byte tensor")
    return _json_object(value.detach().cpu().numpy().tobytes(), key)


def encode_quant_tensor(config: dict) -> torch.Tensor:
    """A config as a .comfy_quant U8 tensor (convrot.py:159-160)."""
    return torch.frombuffer(bytearray(json.dumps(config).encode("utf-8")), dtype=torch.uint8)


def _json_object(raw: bytes, key: str) -> dict:
    try:
        value = json.loads(raw)
    except (UnicodeDecodeError, json.JSONDecodeError) as exc:
        raise ValueError(f"{key} contains invalid quantization JSON") from exc
    if not isinstance(value, dict):
        raise ValueError(f"{key} quantization JSON must be an object")
    return value


# ------------------------------------------------------------ container --

def read_safetensors_header(path: str | Path) -> tuple[dict, int, int]:
    """(header dict, byte offset of the data, file size) with the loader's
    checks (convrot.py:163-185)."""
    path = Path(path)
    size = path.stat().st_size
    with path.open("rb") as f:
        head = f.read(8)
        if len(head) != 8:
            raise ValueError("file is too short to contain a safetensors header")
        (n,) = struct.unpack("<Q", head)
        if n == 0 or n > MAX_HEADER_BYTES:
            raise ValueError(f"invalid safetensors header size {n}")
        if 8 + n > size:
            raise ValueError(f"safetensors header ends at byte {8 + n}, beyond file size {size}")
        raw = f.read(n)
    try:
        header = json.loads(raw)
    except (UnicodeDecodeError, json.JSONDecodeError) as exc:
        raise ValueError("safetensors header contains invalid JSON") from exc
    if not isinstance(header, dict):
        raise ValueError("safetensors header must be an object")
    return header, 8 + n, size


def _byte_range(info: Any, key: str, data_start: int, size: int) -> tuple[list, int, int]:
    """Validated (shape, absolute start, absolute end) of a tensor descriptor."""
    if not isinstance(info, dict):
        raise ValueError(f"{key} has an invalid safetensors tensor descriptor")
    shape, offsets = info.get("shape"), info.get("data_offsets")
    if (not isinstance(shape, list) or not all(_is_int(d) and d >= 0 for d in shape)
            or not isinstance(offsets, list) or len(offsets) != 2
            or not all(_is_int(o) for o in offsets)):
        raise ValueError(f"{key} has invalid shape or data offsets")
    lo, hi = offsets
    return shape, data_start + lo, data_start + hi


def _check_inside(key: str, lo_rel: int, lo: int, hi: int, size: int) -> None:
    if lo_rel < 0 or hi < lo or hi > size:
        raise ValueError(f"{key} data offsets are outside the safetensors file")


def read_quant_config(handle, info: Any, key: str, data_start: int, size: int) -> dict:
    """The config held by a .comfy_quant tensor of an open file
    (convrot.py:188-232)."""
    if not isinstance(info, dict):
        raise ValueError(f"{key} has an invalid safetensors tensor descriptor")
    if info.get("dtype") != "U8":
        raise ValueError(f"{key} must use U8 storage")
    shape, lo, hi = _byte_range(info, key, data_start, size)
    nbytes = hi - lo
    if nbytes != math.prod(shape):
        raise ValueError(f"{key} byte length does not match its U8 shape")
    if nbytes > MAX_CONFIG_BYTES:
        raise ValueError(f"{key} is too large to be quantization JSON")
    _check_inside(key, lo - data_start, lo, hi, size)
    handle.seek(lo)
    raw = handle.read(nbytes)
    if len(raw) != nbytes:
        raise ValueError(f"{key} tensor data is truncated")
    return _json_object(raw, key)


def _header_layers(raw: Any) -> dict:
    parsed = json.loads(raw)
    if not isinstance(parsed, dict) or not isinstance(parsed.get("layers"), dict):
        raise ValueError("safetensors _quantization_metadata must contain a layers object")
    return parsed


def convrot_skip_reason(path: str | Path) -> str | None:
    """None when the file holds at least one supported ConvRot layer, else
    why it is not a ConvRot model (convrot.py:235-263)."""
    path = Path(path)
    if path.suffix.lower() not in MODEL_EXTENSIONS:
        return f"unsupported file extension {path.suffix!r}"
    try:
        header, data_start, size = read_safetensors_header(path)
        metadata = header.get("__metadata__", {})
        if not isinstance(metadata, dict):
            return "safetensors __metadata__ must be an object"
        raw = metadata.get(HEADER_KEY)
        if raw is not None:
            try:
                layers = _header_layers(raw)["layers"]
            except ValueError as exc:
                if isinstance(exc, json.JSONDecodeError):
                    raise
                return str(exc)
            if any(classify_config(cfg, name, True) is not None for name, cfg in layers.items()):
                return None
        with path.open("rb") as f:
            for key, info in header.items():
                if key == "__metadata__" or not key.endswith(QUANT_SUFFIX):
                    continue
                cfg = read_quant_config(f, info, key, data_start, size)
                if classify_config(cfg, key[: -len(QUANT_SUFFIX)], True) is not None:
                    return None
    except Exception as exc:  # the loader reports any read failure as a reason
        return f"could not read ConvRot metadata ({exc})"
    return "does not contain supported ConvRot quantization metadata"


# ------------------------------------------------------ activation config --

def configure_convrot_activation(state_dict: dict, metadata: dict | None, force_int8_gemm: bool,
                                 model_prefix: str | None = None
                                 ) -> tuple[dict, ConvRotSummary]:
    """Classify every ConvRot layer of a loaded checkpoint, check that a layer
    described twice is described alike, apply the force-INT8-GEMM override
    (linear_dtype = "int8" on every non-codebook layer) to the header and the
    .comfy_quant tensors, and count the layers (convrot.py:294-371).  Returns
    the updated metadata; the state dict's .comfy_quant tensors are
    re-encoded in place."""
    if not isinstance(force_int8_gemm, bool):
        raise ValueError(f"force_int8_gemm must be boolean, got {force_int8_gemm!r}")
    metadata = dict(metadata or {})
    keep = (lambda name: True) if model_prefix is None else (lambda name: name.startswith(model_prefix))

    described: list[tuple[str, dict]] = []
    header = None
    if metadata.get(HEADER_KEY) is not None:
        try:
            header = json.loads(metadata[HEADER_KEY])
        except (TypeError, json.JSONDecodeError) as exc:
            raise ValueError("Safetensors _quantization_metadata contains invalid JSON") from exc
        if not isinstance(header, dict) or not isinstance(header.get("layers"), dict):
            raise ValueError("Safetensors _quantization_metadata must contain a layers object")
        described += [(name, cfg) for name, cfg in header["layers"].items() if keep(name)]
    tensor_cfgs: dict[str, dict] = {}
    for key, value in state_dict.items():
        if key.endswith(QUANT_SUFFIX) and keep(key[: -len(QUANT_SUFFIX)]):
            tensor_cfgs[key] = decode_quant_tensor(value, key)
            described.append((key[: -len(QUANT_SUFFIX)], tensor_cfgs[key]))

    kinds: dict[str, tuple[str, str]] = {}
    quantized: list[tuple[dict, str]] = []
    for name, cfg in described:
        kind = classify_config(cfg, name, force_int8_gemm)
        if kind is None:
            continue
        seen = kinds.setdefault(name, kind)
        if seen != kind:
            raise ValueError(f"Conflicting ConvRot metadata for layer {name}: "
                             f"{seen[0]}/{seen[1]} versus {kind[0]}/{kind[1]}")
        quantized.append((cfg, kind[0]))
    if not quantized:
        raise ValueError("The selected model does not contain supported ConvRot quantization metadata")
    if force_int8_gemm:
        for cfg, weight in quantized:
            if weight != "w4_codebook":
                cfg["linear_dtype"] = "int8"

    if header is not None:
        metadata[HEADER_KEY] = json.dumps(header)
    for key, cfg in tensor_cfgs.items():
        state_dict[key] = encode_quant_tensor(cfg)
    counts = {("w4", "int4"): 0, ("w4", "int8"): 0, ("w4_codebook", "int8"): 0, ("w8", "int8"): 0}
    for kind in kinds.values():
        counts[kind] = counts.get(kind, 0) + 1
    return metadata, ConvRotSummary(counts[("w4", "int4")], counts[("w4", "int8")],
                                    counts[("w4_codebook", "int8")], counts[("w8", "int8")])


# --------------------------------------------------------- tensor reader --

# safetensors dtype tag -> (numpy storage dtype, torch dtype of the tensor)
_DTYPES = {
    "F64": (np.float64, torch.float64), "F32": (np.float32, torch.float32),
    "F16": (np.float16, torch.float16), "BF16": (np.int16, torch.bfloat16),
    "I64": (np.int64, torch.int64), "I32": (np.int32, torch.int32),
    "I16": (np.int16, torch.int16), "I8": (np.int8, torch.int8), "U8": (np.uint8, torch.uint8),
    "BOOL": (np.bool_, torch.bool),
    "F8_E4M3": (np.uint8, torch.float8_e4m3fn), "F8_E5M2": (np.uint8, torch.float8_e5m2),
}


class SafetensorsFile:
    """Read-only view of a .safetensors file: the header is checked once and
    each tensor is read (memory-mapped) only when asked for, with its byte
    range checked against its dtype, shape and the file."""

    def __init__(self, path: str | Path):
        self.path = Path(path)
        self.header, self.data_start, self.size = read_safetensors_header(self.path)
        meta = self.header.get("__metadata__", {})
        if not isinstance(meta, dict):
            raise ValueError("safetensors __metadata__ must be an object")
        self.metadata: dict = meta

    def keys(self) -> list[str]:
        return [k for k in self.header if k != "__metadata__"]

    def info(self, key: str) -> tuple[str, list, int, int]:
        """(dtype tag, shape, absolute byte start, end)."""
        desc = self.header[key]
        shape, lo, hi = _byte_range(desc, key, self.data_start, self.size)
        dtype = desc.get("dtype")
        if dtype not in _DTYPES:
            raise ValueError(f"{key} has unsupported dtype {dtype!r}")
        _check_inside(key, lo - self.data_start, lo, hi, self.size)
        itemsize = np.dtype(_DTYPES[dtype][0]).itemsize
        if hi - lo != math.prod(shape) * itemsize:
            raise ValueError(f"{key} byte length does not match its {dtype} shape {shape}")
        return dtype, shape, lo, hi

    def tensor(self, key: str) -> torch.Tensor:
        dtype, shape, lo, hi = self.info(key)
        np_dtype, t_dtype = _DTYPES[dtype]
        count = math.prod(shape)
        if count == 0:
            return torch.empty(shape, dtype=t_dtype)
        arr = np.memmap(self.path, dtype=np_dtype, mode="r", offset=lo, shape=(count,))
        t = torch.from_numpy(np.array(arr))  # own the bytes; the map closes here
        if t.dtype != t_dtype:
            t = t.view(t_dtype)
        return t.reshape(shape)

    def quant_configs(self) -> dict[str, dict]:
        """Every layer's quantization config: header entries first, then
        .comfy_quant tensors (same precedence as configure_convrot_activation)."""
        out: dict[str, dict] = {}
        raw = self.metadata.get(HEADER_KEY)
        if raw is not None:
            out.update(_header_layers(raw)["layers"])
        with self.path.open("rb") as f:
            for key, info in self.header.items():
                if key.endswith(QUANT_SUFFIX):
                    out.setdefault(key[: -len(QUANT_SUFFIX)],
                                   read_quant_config(f, info, key, self.data_start, self.size))
        return out


# ------------------------------------------------------- kernel call plan --

# (weight kind, activation dtype) -> (activation quantizer, linear op) of
# this package, as the plugin's dispatcher pairs them
# (quantization/dispatch.py:326-393, 538-615, 673-740, 780-804).
KERNEL_PLAN = {
    ("w8", "int8"): ("turing_bf16_int8_convrot_quantize", "turing_int8_linear"),
    ("w4", "int8"): ("turing_bf16_int8_convrot_quantize", "turing_w4a8_linear"),
    ("w4", "int4"): ("turing_bf16_int4_convrot_quantize", "turing_int4_linear"),
    ("w4_codebook", "int8"): ("turing_bf16_int8_convrot_quantize", "turing_codebook_w4a8_linear"),
}


@dataclasses.dataclass(frozen=True)
class LayerPlan:
    name: str
    weight: str          # "w8" | "w4" | "w4_codebook"
    activation: str      # "int8" | "int4"
    quantizer: str       # op of this package that quantizes the layer's input
    linear: str          # op of this package that runs the layer
    config: dict
    tensors: tuple[str, ...]   # the file's tensors of this layer ("<name>.*"), sorted


def layer_plans(path: str | Path, force_int8_gemm: bool = False,
                model_prefix: str | None = None) -> Iterator[LayerPlan]:
    """The ConvRot layers of a checkpoint and the kernels that run each."""
    st = SafetensorsFile(path)
    names = st.keys()
    for name, cfg in st.quant_configs().items():
        if model_prefix is not None and not name.startswith(model_prefix):
            continue
        kind = classify_config(dict(cfg), name, force_int8_gemm)
        if kind is None:
            continue
        quantizer, linear = KERNEL_PLAN[kind]
        own = tuple(sorted(k for k in names
                           if k.startswith(name + ".") and not k.endswith(QUANT_SUFFIX)))
        yield LayerPlan(name, kind[0], kind[1], quantizer, linear, cfg, own)
