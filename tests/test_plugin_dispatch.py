"""The plugin's own dispatcher, patched as INTEGRATION.md shows, reaches this
package's ops (the drop-in boundary of comfyui_turing_utils/hardware.py:24-42
and quantization/dispatch.py:326-393, 538-670, 673-740, 746-806).

The test copies the reference plugin's `hardware.py`, `kernel_api.py` and
`quantization/dispatch.py` into a temporary package, applies the diff hunks
printed in INTEGRATION.md to them (so the documented edits are the tested
ones), stubs ComfyUI's comfy-kitchen, and calls `int8_linear`,
`codebook_w4a8_linear` and `convrot_w4a4_linear` with fake CUDA tensors on a
simulated capability-(10, 0) device.  Spies on this package's ops record what
the dispatcher passes; the ops run their registered fake implementations, so
the shapes and dtypes the dispatcher reshapes are the real contract.  Needs
the reference checkout (TB_REFERENCE_ROOT, else a `reference` directory
beside this repository); skipped without it.
"""
from __future__ import annotations

import importlib
import os
import re
import sys
import types
from pathlib import Path

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from conftest import ROOT

REF = Path(os.environ.get("TB_REFERENCE_ROOT", ROOT.parent / "reference"))
PLUGIN = REF / "comfyui_turing_utils"
pytestmark = pytest.mark.skipif(not (PLUGIN / "quantization" / "dispatch.py").exists(),
                                reason="reference plugin checkout not present")


def _integration_hunks() -> dict[str, list[tuple[str, str]]]:
    """(old, new) text pairs per file from INTEGRATION.md's ```diff blocks."""
    text = (ROOT / "INTEGRATION.md").read_text()
    edits: dict[str, list[tuple[str, str]]] = {}
    for block in re.findall(r"```diff\n(.*?)```", text, flags=re.S):
        lines = block.split("\n")
        path = next(l[6:] for l in lines if l.startswith("+++ b/"))
        hunks, cur = [], None
        for line in lines:
            if line.startswith(("--- a/", "+++ b/")):
                continue
            if line.startswith("@@"):
                cur = ([], [])
                hunks.append(cur)
            elif cur is not None and line:
                tag, body = line[0], line[1:]
                if tag in " -":
                    cur[0].append(body)
                if tag in " +":
                    cur[1].append(body)
        edits[path] = [("\n".join(o), "\n".join(n)) for o, n in hunks]
    return edits


def _apply(source: str, hunks: list[tuple[str, str]], name: str) -> str:
    for old, new in hunks:
        assert source.count(old) == 1, f"hunk does not apply exactly once to {name}:\n{old}"
        source = source.replace(old, new)
    return source


class KitchenCalled(Exception):
    pass


def _kitchen_stub() -> dict[str, types.ModuleType]:
    """comfy_kitchen with the names dispatch.py imports; every Kitchen
    compute call raises KitchenCalled so a route that leaves this package
    is visible."""
    root = types.ModuleType("comfy_kitchen")
    backends = types.ModuleType("comfy_kitchen.backends")
    cuda = types.ModuleType("comfy_kitchen.backends.cuda")
    acts = types.ModuleType("comfy_kitchen.backends._activations")
    for name in ("int8_linear", "convrot_w4a4_linear", "w4a8_int8_linear", "int4_linear",
                 "quantize_int8_rowwise_convrot64", "quantize_int4_rowwise_convrot64",
                 "quantize_int8_convrot_staged", "rotate_int8_convrot_weight",
                 "quantize_int4_rowwise"):
        def call(*args, _name=name, **kwargs):
            raise KitchenCalled(_name)
        setattr(cuda, name, call)

    def apply_input_act(x, act):
        if act in (None, "none"):
            return x
        raise KitchenCalled(f"apply_input_act({act})")

    acts.apply_input_act = apply_input_act
    root.backends, backends.cuda, backends._activations = backends, cuda, acts
    root.list_backends = lambda: {}
    return {"comfy_kitchen": root, "comfy_kitchen.backends": backends,
            "comfy_kitchen.backends.cuda": cuda, "comfy_kitchen.backends._activations": acts}


@pytest.fixture
def plugin(tmp_path, monkeypatch):
    """The patched plugin modules, imported from a temporary package."""
    edits = _integration_hunks()
    pkg = tmp_path / "comfyui_turing_utils"
    (pkg / "quantization").mkdir(parents=True)
    (pkg / "__init__.py").write_text("")
    (pkg / "quantization" / "__init__.py").write_text("")
    for rel in ("hardware.py", "kernel_api.py", "quantization/dispatch.py"):
        src = (PLUGIN / rel).read_text()
        key = f"comfyui_turing_utils/{rel}"
        if key in edits:
            src = _apply(src, edits[key], key)
        (pkg / rel).write_text(src)
    for name, mod in _kitchen_stub().items():
        monkeypatch.setitem(sys.modules, name, mod)
    for name in [m for m in sys.modules if m.startswith("comfyui_turing_utils.")
                 or m == "comfyui_turing_utils"]:
        monkeypatch.delitem(sys.modules, name)
    monkeypatch.syspath_prepend(str(tmp_path))
    # A simulated B200 at cuda:0 (the fake tensors below live there).  Only
    # the plugin's hardware module sees torch.cuda.is_available() == True:
    # fake tensors would touch the real CUDA runtime if torch itself saw it.
    import torch._subclasses.fake_tensor as fake_tensor

    monkeypatch.setattr(fake_tensor, "init_gpu_context", lambda device: None)
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    monkeypatch.setattr(torch.cuda, "get_device_capability", lambda index=None: (10, 0))
    monkeypatch.setattr(torch.cuda, "get_device_name", lambda index=None: "NVIDIA B200")
    hardware = importlib.import_module("comfyui_turing_utils.hardware")
    hardware.torch = types.SimpleNamespace(
        device=torch.device,
        cuda=types.SimpleNamespace(
            is_available=lambda: True,
            current_device=lambda: torch.cuda.current_device(),
            get_device_capability=lambda index=None: torch.cuda.get_device_capability(index),
            get_device_name=lambda index=None: torch.cuda.get_device_name(index)))
    dispatch = importlib.import_module("comfyui_turing_utils.quantization.dispatch")
    yield types.SimpleNamespace(hardware=hardware, dispatch=dispatch)
    for name in [m for m in sys.modules if m.startswith("comfyui_turing_utils.")
                 or m == "comfyui_turing_utils"]:
        sys.modules.pop(name, None)


@pytest.fixture
def spies(monkeypatch):
    """Wraps this package's linear-path ops; records (name, args, kwargs)."""
    import comfyui_turing_utils_kernel as kernel

    calls = []
    for name in kernel.__all__:
        fn = getattr(kernel, name)
        if not callable(fn):
            continue

        def spy(*args, _name=name, _fn=fn, **kwargs):
            calls.append((_name, args, kwargs))
            return _fn(*args, **kwargs)

        monkeypatch.setattr(kernel, name, spy)
    return calls


def _cuda(shape, dtype):
    return torch.empty(shape, dtype=dtype, device="cuda")


def test_widened_predicate(plugin, monkeypatch):
    hw = plugin.hardware
    dev = torch.device("cuda", 0)
    assert hw.is_supported_turing_device(dev)
    assert hw.is_supported_attention_device(dev)
    for cap, name, want in (((9, 0), "NVIDIA H100", False), ((7, 5), "Tesla T4", True),
                            ((7, 5), "NVIDIA GeForce GTX 1650", False), ((8, 9), "L40S", False)):
        monkeypatch.setattr(torch.cuda, "get_device_capability", lambda index=None, c=cap: c)
        monkeypatch.setattr(torch.cuda, "get_device_name", lambda index=None, n=name: n)
        assert hw.is_supported_turing_device(dev) is want, (cap, name)
    assert not hw.is_supported_turing_device(torch.device("cpu"))


def test_int8_linear_reaches_quantizer_and_gemm(plugin, spies):
    """dispatch.py:618-670 with the ConvRot W8A8 layout (configs[0]'s widths)."""
    with FakeTensorMode(allow_non_fake_inputs=True):
        x = _cuda((2, 8, 5120), torch.bfloat16)
        w, ws, b = _cuda((64, 5120), torch.int8), _cuda((), torch.float32), _cuda((64,), torch.bfloat16)
        out = plugin.dispatch.int8_linear(x, w, ws, bias=b, convrot=True, convrot_groupsize=256)
        assert out.shape == (2, 8, 64) and out.dtype == torch.bfloat16
    names = [c[0] for c in spies]
    assert names == ["turing_bf16_int8_convrot_quantize", "turing_int8_linear"]
    (_, qargs, qkw), (_, largs, _) = spies
    assert qargs[0].shape == (16, 5120) and qargs[1] == 256 and qkw == {"swiglu": False}
    qa, wq, a_s, w_s, bias = largs
    assert qa.shape == (16, 5120) and qa.dtype == torch.int8
    assert a_s.shape == (16,) and a_s.dtype == torch.float32
    assert w_s.shape == (64,) and w_s.dtype == torch.float32  # scalar scale expanded
    assert bias is b


@pytest.mark.parametrize("act,width,want", [
    ("gelu_tanh", 13824, ("turing_bf16_gelu_int8_convrot_quantize", (256,), {})),
    ("swiglu", 2 * 5120, ("turing_bf16_int8_convrot_quantize", (256,), {"swiglu": True})),
])
def test_int8_linear_fused_activation_quantizers(plugin, spies, act, width, want):
    with FakeTensorMode(allow_non_fake_inputs=True):
        x = _cuda((16, width), torch.bfloat16)
        k = width // 2 if act == "swiglu" else width
        out = plugin.dispatch.int8_linear(x, _cuda((64, k), torch.int8), _cuda((64,), torch.float32),
                                          convrot=True, input_act=act)
        assert out.shape == (16, 64)
    name, args, kwargs = spies[0]
    assert (name, args[1:], kwargs) == want
    assert spies[1][0] == "turing_int8_linear"


def test_narrow_rows_also_stay_in_this_package(plugin, spies):
    """Widths below Kitchen's 48 KiB launch (dispatch.py:356-363) go to the
    bundled quantizer on sm_100 after the INT8-quantizer hunk."""
    with FakeTensorMode(allow_non_fake_inputs=True):
        out = plugin.dispatch.int8_linear(_cuda((4, 256), torch.bfloat16),
                                          _cuda((32, 256), torch.int8),
                                          _cuda((32,), torch.float32), convrot=True)
        assert out.shape == (4, 32)
    assert [c[0] for c in spies] == ["turing_bf16_int8_convrot_quantize", "turing_int8_linear"]


def test_unpatched_predicate_leaves_for_kitchen(plugin, spies, monkeypatch):
    """The gate is the predicate: reporting a non-Turing, non-B200 device sends
    the call to comfy-kitchen without touching this package."""
    monkeypatch.setattr(torch.cuda, "get_device_capability", lambda index=None: (9, 0))
    with FakeTensorMode(allow_non_fake_inputs=True):
        with pytest.raises(KitchenCalled, match="int8_linear"):
            plugin.dispatch.int8_linear(_cuda((16, 5120), torch.bfloat16),
                                        _cuda((64, 5120), torch.int8), _cuda((64,), torch.float32),
                                        convrot=True)
    assert spies == []


def test_codebook_w4a8_linear_route(plugin, spies):
    """dispatch.py:673-740 (configs[2]: grouped-codebook W4A8, group 16)."""
    n, k, g = 64, 5120, 16
    with FakeTensorMode(allow_non_fake_inputs=True):
        x = _cuda((16, k), torch.bfloat16)
        qdata = _cuda((n, k // 2), torch.int8)
        s_rel = _cuda((n, k // g), torch.float8_e4m3fn)
        s_ch, cb, b = _cuda((n,), torch.float32), _cuda((16,), torch.float32), _cuda((n,), torch.bfloat16)
        out = plugin.dispatch.codebook_w4a8_linear(x, qdata, s_rel, s_ch, codebook=cb, bias=b,
                                                   group_size=g)
        assert out.shape == (16, n) and out.dtype == torch.bfloat16
    assert [c[0] for c in spies] == ["turing_bf16_int8_convrot_quantize",
                                     "turing_codebook_w4a8_linear"]
    args = spies[1][1]
    assert args[1] is qdata and args[3] is s_rel and args[4] is s_ch and args[5] is cb
    assert args[6] is b and args[7] == g


def test_convrot_w4a4_linear_int8_activation_route(plugin, spies):
    """dispatch.py:780-789: signed-nibble W4 weights with INT8 activations."""
    with FakeTensorMode(allow_non_fake_inputs=True):
        out = plugin.dispatch.convrot_w4a4_linear(_cuda((16, 5120), torch.bfloat16),
                                                  _cuda((64, 2560), torch.int8),
                                                  _cuda((64,), torch.float32),
                                                  linear_dtype="int8")
        assert out.shape == (16, 64)
    assert [c[0] for c in spies] == ["turing_bf16_int8_convrot_quantize", "turing_w4a8_linear"]


@pytest.mark.parametrize("act,width,quantizer", [
    (None, 5120, "turing_bf16_int4_convrot_quantize"),
    ("gelu_tanh", 13824, "turing_bf16_gelu_int4_convrot_quantize"),
])
def test_convrot_w4a4_linear_int4_route(plugin, spies, act, width, quantizer):
    """dispatch.py:791-804 (configs[3]: W4A4 up- and GELU-fused down-projection)."""
    with FakeTensorMode(allow_non_fake_inputs=True):
        b = _cuda((64,), torch.bfloat16)
        out = plugin.dispatch.convrot_w4a4_linear(_cuda((16, width), torch.bfloat16),
                                                  _cuda((64, width // 2), torch.int8),
                                                  _cuda((64,), torch.float32), bias=b,
                                                  linear_dtype="int4", input_act=act)
        assert out.shape == (16, 64) and out.dtype == torch.bfloat16
    assert [c[0] for c in spies] == [quantizer, "turing_int4_linear"]
    qa, wq, a_s, w_s, bias = spies[1][1]
    assert qa.shape == (16, width // 2) and qa.dtype == torch.int8  # packed INT4 codes
    assert a_s.shape == (16,) and bias is b
