"""Generate tests/golden/checkpoint_cases.json by running the REFERENCE's
ConvRot checkpoint-format code (comfyui_turing_utils/quantization/convrot.py:
37-42, 82-144, 147-232, 294-371) on seeded synthetic cases.

    python tests/golden/make_checkpoint_golden.py [/path/to/reference]

Test infrastructure only.  convrot.py imports ComfyUI modules that are not
installed; they are replaced by empty stand-ins (none of the functions called
here touches them).  Each case records its input (configs, a state dict of
small tensors, or the bytes of a .safetensors file) and the reference's
result or error message; tests/test_checkpoint.py replays them against
comfyui_turing_utils_kernel.checkpoint.
"""
from __future__ import annotations

import base64
import importlib.util
import json
import struct
import os
import sys
import tempfile
import types
from pathlib import Path

import torch
from safetensors.torch import save_file

OUT = Path(__file__).resolve().parent / "checkpoint_cases.json"


def load_reference(root: Path):
    pkg = root / "comfyui_turing_utils"
    stubs = {
        "folder_paths": {}, "comfy": {}, "comfy.model_detection": {}, "comfy.model_management": {},
        "comfy.sd": {}, "comfy.utils": {},
        "comfyui_turing_utils.attention": {"apply_attention_backend": None,
                                           "normalize_attention_backend": None},
        "comfyui_turing_utils.adapters": {},
        "comfyui_turing_utils.adapters.registry": {"apply_model_adapters": None},
        "comfyui_turing_utils.precision": {"normalize_turing_convrot_weight_dtypes": None,
                                           "prepare_turing_runtime": None,
                                           "select_compute_dtype": None},
    }
    for name, attrs in stubs.items():
        mod = types.ModuleType(name)
        mod.__dict__.update(attrs)
        sys.modules[name] = mod
    comfy = sys.modules["comfy"]
    for sub in ("model_detection", "model_management", "sd", "utils"):
        setattr(comfy, sub, sys.modules[f"comfy.{sub}"])
    # Default arguments evaluated at import time.
    comfy.sd.CLIPType = types.SimpleNamespace(STABLE_DIFFUSION="stable_diffusion")
    for name, path in (("comfyui_turing_utils", pkg), ("comfyui_turing_utils.quantization",
                                                       pkg / "quantization")):
        mod = types.ModuleType(name)
        mod.__path__ = [str(path)]
        sys.modules[name] = mod
    spec = importlib.util.spec_from_file_location("comfyui_turing_utils.quantization.convrot",
                                                  pkg / "quantization" / "convrot.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def qt(config) -> list:
    return list(json.dumps(config).encode("utf-8"))


def run(fn):
    try:
        return {"ok": fn()}
    except Exception as exc:  # the reference's error behaviour is part of the fixture
        return {"error": type(exc).__name__, "message": str(exc)}


CLASSIFY = [
    ({"format": "int8_tensorwise", "convrot": True}, False),
    ({"format": "int8_tensorwise", "params": {"convrot": True}}, False),
    ({"format": "int8_tensorwise", "convrot": True, "linear_dtype": "int4"}, False),
    ({"format": "int8_tensorwise", "convrot": True, "linear_dtype": "int4"}, True),
    ({"format": "int8_tensorwise", "convrot": True, "linear_dtype": "fp8"}, True),
    ({"format": "int8_tensorwise", "params": {"convrot": True, "linear_dtype": "int8"},
      "linear_dtype": "int4"}, False),
    ({"format": "convrot_w4a4"}, False),
    ({"format": "convrot_w4a4", "linear_dtype": "int8"}, False),
    ({"format": "convrot_w4a4", "params": {"linear_dtype": "int8"}}, False),
    ({"format": "convrot_w4a4"}, True),
    ({"format": "convrot_w4a4", "linear_dtype": "fp16"}, True),
    ({"format": "asym_w4a8_int8", "group_size": 16, "convrot": True, "convrot_groupsize": 256}, False),
    ({"format": "asym_w4a8_int8"}, True),
    ({"format": "asym_w4a8_int8", "convrot": False}, False),
    ({"format": "asym_w4a8_int8", "group_size": 3}, False),
    ({"format": "asym_w4a8_int8", "group_size": True}, False),
    ({"format": "asym_w4a8_int8", "group_size": 128.0}, False),
    ({"format": "asym_w4a8_int8", "params": {"group_size": 128}, "convrot_groupsize": 128}, False),
    ({"convrot": True, "per_row": True}, False),
    ({"convrot": True, "convrot_groupsize": 256, "per_row": True}, False),
    ({"format": "int8_rowwise", "convrot": True, "per_row": True}, False),
    ({"format": "int8_rowwise", "params": {"convrot": True, "per_row": True}}, False),
    ({"format": "int8_rowwise", "convrot": True}, False),
    ({"convrot": True}, False),
    ({"format": "float8_e4m3fn"}, False),
    ({"format": "int8_tensorwise"}, False),
    ({"format": "mxfp8", "convrot": True}, False),
    ({"format": "int8_tensorwise", "convrot": "yes"}, False),
    ({"format": "int8_tensorwise", "params": [1, 2]}, False),
    ([1, 2], False),
]

CONFIGURE = [
    # (state-dict comfy_quant configs by layer, header metadata layers or None, force, prefix)
    ({"blocks.0.mlp.fc1": {"format": "asym_w4a8_int8", "group_size": 16, "convrot": True,
                           "convrot_groupsize": 256}}, None, True, None),
    ({"blocks.0.mlp.fc1": {"format": "asym_w4a8_int8", "convrot": False}}, None, False, None),
    ({}, {"blocks.0.attn.q": {"format": "convrot_w4a4"}}, False, None),
    ({"blocks.0.attn.q": {"format": "convrot_w4a4", "linear_dtype": "int4"}},
     {"blocks.0.attn.q": {"format": "convrot_w4a4", "linear_dtype": "int4"}}, True, None),
    ({"model.diffusion_model.blocks.0.q": {"format": "convrot_w4a4"},
      "text_encoders.t5.layer.0.q": {"format": "int8_tensorwise", "convrot": True,
                                     "linear_dtype": "int4"}}, None, False, "model.diffusion_model."),
    ({"a": {"format": "int8_tensorwise", "convrot": True, "linear_dtype": "int4"}}, None, False, None),
    ({"a": {"format": "convrot_w4a4"}, "b": {"format": "int8_tensorwise", "params": {"convrot": True}}},
     None, True, None),
    ({"a": {"convrot": True, "convrot_groupsize": 256, "per_row": True}}, None, False, None),
    ({}, {"a": {"format": "int8_rowwise", "convrot": True, "per_row": True}}, False, None),
    ({"a": {"convrot": True}}, None, False, None),
    ({"a": {"format": "convrot_w4a4", "linear_dtype": "int8"}}, None, False, None),
    ({"a": {"format": "int8_tensorwise", "convrot": True, "linear_dtype": "int4"}}, None, True, None),
    ({"a": {"format": "float8_e4m3fn"}}, None, False, None),
    ({"a": {"format": "nvfp4", "convrot": True}}, None, False, None),
    ({"a": {"format": "convrot_w4a4", "linear_dtype": "int4"}},
     {"a": {"format": "convrot_w4a4", "linear_dtype": "int8"}}, False, None),
    ({"a": {"format": "convrot_w4a4"}, "b": {"format": "asym_w4a8_int8"},
      "c": {"format": "int8_tensorwise", "convrot": True}, "d": {"format": "float8_e4m3fn"}},
     {"e": {"format": "convrot_w4a4", "linear_dtype": "int8"}}, False, None),
]


def configure_case(mod, layers, header, force, prefix):
    sd = {f"{k}.comfy_quant": torch.tensor(qt(v), dtype=torch.uint8) for k, v in layers.items()}
    sd["blocks.0.attn.q.weight"] = torch.zeros(2, dtype=torch.int8)
    md = {"format": "pt"}
    if header is not None:
        md["_quantization_metadata"] = json.dumps({"layers": header})

    def go():
        meta, summary = mod.configure_convrot_activation(sd, md, force, prefix)
        configs = {k: json.loads(bytes(v.tolist())) for k, v in sd.items() if k.endswith(".comfy_quant")}
        return {"metadata": meta, "summary": [summary.w4a4, summary.w4a8, summary.codebook_w4a8,
                                              summary.w8a8], "configs": configs}
    return {"layers": layers, "header": header, "force": force, "prefix": prefix, "result": run(go)}


def st_file(tensors: dict, metadata: dict | None) -> bytes:
    with tempfile.TemporaryDirectory() as d:
        p = Path(d) / "m.safetensors"
        save_file(tensors, str(p), metadata=metadata)
        return p.read_bytes()


def raw_file(header: dict, payload: bytes = b"", size_override: int | None = None) -> bytes:
    h = json.dumps(header).encode()
    n = len(h) if size_override is None else size_override
    return struct.pack("<Q", n) + h + payload


def skip_cases():
    q = lambda c: torch.tensor(qt(c), dtype=torch.uint8)  # noqa: E731
    w = torch.zeros((4, 4), dtype=torch.int8)
    good_cfg = json.dumps({"format": "int8_tensorwise", "convrot": True}).encode()
    cases = [
        ("w8_tensor.safetensors", st_file({"l.weight": w, "l.comfy_quant": q({"format": "int8_tensorwise", "convrot": True})}, None)),
        ("w4_header.safetensors", st_file({"l.weight": w}, {"_quantization_metadata": json.dumps({"layers": {"l": {"format": "convrot_w4a4"}}})})),
        ("legacy.sft", st_file({"l.weight": w, "l.comfy_quant": q({"convrot": True, "per_row": True})}, None)),
        ("dense.safetensors", st_file({"l.weight": w.float()}, None)),
        ("fp8.safetensors", st_file({"l.weight": w, "l.comfy_quant": q({"format": "float8_e4m3fn"})}, None)),
        ("bad_format.safetensors", st_file({"l.weight": w, "l.comfy_quant": q({"format": "mxfp8", "convrot": True})}, None)),
        ("model.ckpt", st_file({"l.weight": w}, None)),
        ("short.safetensors", b"\x01\x02"),
        ("zero_header.safetensors", struct.pack("<Q", 0) + b"{}"),
        ("huge_header.safetensors", struct.pack("<Q", 1 << 40) + b"{}"),
        ("header_past_end.safetensors", raw_file({"a": 1}, size_override=4096)),
        ("bad_json.safetensors", struct.pack("<Q", 5) + b"{bad!"),
        ("list_header.safetensors", raw_file([1, 2])),
        ("meta_not_dict.safetensors", raw_file({"__metadata__": [1]})),
        ("layers_missing.safetensors", raw_file({"__metadata__": {"_quantization_metadata": json.dumps({"x": 1})}})),
        ("cq_wrong_dtype.safetensors", raw_file({"l.comfy_quant": {"dtype": "I8", "shape": [len(good_cfg)], "data_offsets": [0, len(good_cfg)]}}, good_cfg)),
        ("cq_bad_shape.safetensors", raw_file({"l.comfy_quant": {"dtype": "U8", "shape": [len(good_cfg) + 1], "data_offsets": [0, len(good_cfg)]}}, good_cfg)),
        ("cq_bool_shape.safetensors", raw_file({"l.comfy_quant": {"dtype": "U8", "shape": [True], "data_offsets": [0, 1]}}, good_cfg)),
        ("cq_past_end.safetensors", raw_file({"l.comfy_quant": {"dtype": "U8", "shape": [len(good_cfg)], "data_offsets": [8, 8 + len(good_cfg)]}}, good_cfg)),
        ("cq_negative.safetensors", raw_file({"l.comfy_quant": {"dtype": "U8", "shape": [4], "data_offsets": [-4, 0]}}, good_cfg)),
        ("cq_not_json.safetensors", raw_file({"l.comfy_quant": {"dtype": "U8", "shape": [5], "data_offsets": [0, 5]}}, b"{bad!")),
        ("cq_list_json.safetensors", raw_file({"l.comfy_quant": {"dtype": "U8", "shape": [6], "data_offsets": [0, 6]}}, b"[1, 2]")),
        ("cq_descriptor_list.safetensors", raw_file({"l.comfy_quant": [1]}, good_cfg)),
        ("cq_too_large.safetensors", raw_file({"l.comfy_quant": {"dtype": "U8", "shape": [2 << 20], "data_offsets": [0, 2 << 20]}}, good_cfg)),
        ("cq_ok_raw.safetensors", raw_file({"__metadata__": {"format": "pt"}, "l.comfy_quant": {"dtype": "U8", "shape": [len(good_cfg)], "data_offsets": [0, len(good_cfg)]}}, good_cfg)),
        ("header_w8_rowwise_bad.safetensors", st_file({"l.weight": w}, {"_quantization_metadata": json.dumps({"layers": {"l": {"format": "int8_rowwise", "convrot": True}}})})),
        ("header_invalid_json.safetensors", st_file({"l.weight": w}, {"_quantization_metadata": "{nope"})),
    ]
    return cases


def main(root: Path) -> None:
    mod = load_reference(root)
    out = {"classify": [], "configure": [], "skip": []}
    for cfg, force in CLASSIFY:
        res = run(lambda: (lambda r: list(r) if r is not None else None)(
            mod._classify_config(json.loads(json.dumps(cfg)), "blocks.0.x", force)))
        out["classify"].append({"config": cfg, "force": force, "result": res})
    for layers, header, force, prefix in CONFIGURE:
        out["configure"].append(configure_case(mod, layers, header, force, prefix))
    out["configure"].append({"layers": None, "header": None, "force": "yes", "prefix": None,
                             "result": run(lambda: mod.configure_convrot_activation({}, None, "yes"))})
    with tempfile.TemporaryDirectory() as d:
        for name, data in skip_cases():
            p = Path(d) / name
            p.write_bytes(data)
            out["skip"].append({"name": name, "bytes": base64.b64encode(data).decode(),
                                "reason": mod._convrot_skip_reason(p)})
    OUT.write_text(json.dumps(out, indent=1) + "\n")
    print(f"wrote {OUT} ({len(out['classify'])} classify, {len(out['configure'])} configure, "
          f"{len(out['skip'])} file cases)")


if __name__ == "__main__":
    # The reference checkout: argv[1], else TB_REFERENCE_ROOT, else a
    # `reference` directory beside this repository.
    default = os.environ.get("TB_REFERENCE_ROOT", Path(__file__).resolve().parents[3] / "reference")
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else Path(default))
