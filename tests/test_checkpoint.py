"""ConvRot checkpoint format reader (comfyui_turing_utils_kernel.checkpoint)
against the reference loader's own results: tests/golden/checkpoint_cases.json
was produced by running comfyui_turing_utils/quantization/convrot.py on the
same inputs (tests/golden/make_checkpoint_golden.py).  Results and error
messages must be identical.  The tensor reader is checked against the
safetensors library on files it wrote."""
from __future__ import annotations

import base64
import copy
import json
from pathlib import Path

import pytest
import torch
from safetensors import safe_open
from safetensors.torch import save_file

from comfyui_turing_utils_kernel import checkpoint as ck

CASES = json.loads((Path(__file__).resolve().parent / "golden" / "checkpoint_cases.json").read_text())


def _run(fn):
    try:
        return {"ok": fn()}
    except Exception as exc:
        return {"error": type(exc).__name__, "message": str(exc)}


@pytest.mark.parametrize("case", CASES["classify"], ids=lambda c: json.dumps(c["config"])[:60])
def test_classify_matches_reference(case):
    got = _run(lambda: (lambda r: None if r is None else list(r))(
        ck.classify_config(copy.deepcopy(case["config"]), "blocks.0.x", case["force"])))
    assert got == case["result"]


def _quant_tensor(cfg) -> torch.Tensor:
    return torch.tensor(list(json.dumps(cfg).encode("utf-8")), dtype=torch.uint8)


@pytest.mark.parametrize("case", CASES["configure"], ids=lambda c: json.dumps(c["layers"])[:60])
def test_configure_matches_reference(case):
    if case["layers"] is None:
        got = _run(lambda: ck.configure_convrot_activation({}, None, case["force"]))
        assert got == case["result"]
        return
    sd = {f"{k}.comfy_quant": _quant_tensor(v) for k, v in case["layers"].items()}
    sd["blocks.0.attn.q.weight"] = torch.zeros(2, dtype=torch.int8)
    md = {"format": "pt"}
    if case["header"] is not None:
        md["_quantization_metadata"] = json.dumps({"layers": case["header"]})

    def go():
        meta, s = ck.configure_convrot_activation(sd, md, case["force"], case["prefix"])
        configs = {k: json.loads(bytes(v.tolist())) for k, v in sd.items() if k.endswith(".comfy_quant")}
        return {"metadata": meta, "summary": [s.w4a4, s.w4a8, s.codebook_w4a8, s.w8a8],
                "configs": configs}
    assert _run(go) == case["result"]


@pytest.mark.parametrize("case", CASES["skip"], ids=lambda c: c["name"])
def test_skip_reason_matches_reference(tmp_path, case):
    p = tmp_path / case["name"]
    p.write_bytes(base64.b64decode(case["bytes"]))
    assert ck.convrot_skip_reason(p) == case["reason"]


def test_tensor_reader_matches_safetensors(tmp_path):
    g = torch.Generator().manual_seed(3)
    tensors = {
        "a.weight": torch.randint(-127, 128, (13824 // 64, 5120 // 64), generator=g, dtype=torch.int8),
        "a.weight_scale": torch.rand(216, generator=g),
        "a.bias": torch.randn(216, generator=g).to(torch.bfloat16),
        "b.weight": torch.randint(0, 256, (64, 32), generator=g, dtype=torch.uint8),
        "b.scale": torch.rand(64, 2, generator=g).to(torch.float16),
        "c.f8": torch.randn(5, 7, generator=g).to(torch.float8_e4m3fn),
        "c.i64": torch.arange(11, dtype=torch.int64),
        "c.i32": torch.arange(3, dtype=torch.int32),
        "c.f64": torch.randn(2, 2, generator=g, dtype=torch.float64),
        "c.empty": torch.empty((0, 4), dtype=torch.float32),
        "c.flag": torch.tensor([True, False]),
    }
    p = tmp_path / "m.safetensors"
    save_file(tensors, str(p), metadata={"format": "pt"})
    st = ck.SafetensorsFile(p)
    assert sorted(st.keys()) == sorted(tensors)
    with safe_open(str(p), framework="pt") as ref:
        for k in tensors:
            a, b = st.tensor(k), ref.get_tensor(k)
            assert a.dtype == b.dtype and a.shape == b.shape
            assert torch.equal(a.view(torch.uint8) if a.dtype.is_floating_point and a.element_size() == 1 else a,
                               b.view(torch.uint8) if b.dtype.is_floating_point and b.element_size() == 1 else b)


def test_tensor_reader_rejects_bad_ranges(tmp_path):
    p = tmp_path / "m.safetensors"
    save_file({"x": torch.zeros(8, dtype=torch.float32)}, str(p))
    raw = p.read_bytes()
    n = int.from_bytes(raw[:8], "little")
    header = json.loads(raw[8:8 + n])
    header["x"]["shape"] = [9]
    body = json.dumps(header).encode()
    p.write_bytes(len(body).to_bytes(8, "little") + body + raw[8 + n:])
    with pytest.raises(ValueError, match="byte length does not match"):
        ck.SafetensorsFile(p).tensor("x")
    header["x"]["shape"] = [8]
    header["x"]["data_offsets"] = [4, 36]
    body = json.dumps(header).encode()
    p.write_bytes(len(body).to_bytes(8, "little") + body + raw[8 + n:])
    with pytest.raises(ValueError, match="outside the safetensors file"):
        ck.SafetensorsFile(p).tensor("x")


def test_layer_plans(tmp_path):
    w = torch.zeros((4, 4), dtype=torch.int8)
    layers = {
        "blocks.0.attn.q": {"format": "int8_tensorwise", "convrot": True},
        "blocks.0.ffn.up": {"format": "convrot_w4a4"},
        "blocks.0.ffn.down": {"format": "convrot_w4a4", "linear_dtype": "int8"},
        "blocks.0.attn.o": {"format": "asym_w4a8_int8", "group_size": 128},
        "blocks.0.norm": {"format": "float8_e4m3fn"},
    }
    tensors = {f"{k}.weight": w.clone() for k in layers}
    tensors["blocks.0.attn.q.weight_scale"] = torch.ones(4)
    tensors["blocks.0.ffn.up.comfy_quant"] = _quant_tensor(layers.pop("blocks.0.ffn.up"))
    p = tmp_path / "m.safetensors"
    save_file(tensors, str(p), metadata={"_quantization_metadata": json.dumps({"layers": layers})})
    plans = {pl.name: pl for pl in ck.layer_plans(p)}
    assert set(plans) == {"blocks.0.attn.q", "blocks.0.ffn.up", "blocks.0.ffn.down", "blocks.0.attn.o"}
    assert (plans["blocks.0.attn.q"].linear, plans["blocks.0.attn.q"].activation) == ("turing_int8_linear", "int8")
    assert plans["blocks.0.attn.q"].tensors == ("blocks.0.attn.q.weight", "blocks.0.attn.q.weight_scale")
    assert (plans["blocks.0.ffn.up"].quantizer, plans["blocks.0.ffn.up"].linear) == \
        ("turing_bf16_int4_convrot_quantize", "turing_int4_linear")
    assert plans["blocks.0.ffn.down"].linear == "turing_w4a8_linear"
    assert plans["blocks.0.attn.o"].linear == "turing_codebook_w4a8_linear"
    forced = {pl.name: pl for pl in ck.layer_plans(p, force_int8_gemm=True)}
    assert forced["blocks.0.ffn.up"].linear == "turing_w4a8_linear"
    import comfyui_turing_utils_kernel as k
    for pl in plans.values():  # every planned op exists in this package
        assert hasattr(k, pl.quantizer) and hasattr(k, pl.linear), pl
