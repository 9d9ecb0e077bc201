"""The C-ABI library loads, exports every symbol include/*.h declares, and
rejects invalid arguments with the reference's messages before touching the
GPU (these calls never launch anything, so they run on the CPU)."""
from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from conftest import LIB, ROOT


def declared_symbols():
    names = []
    for header in (ROOT / "include").glob("*.h"):
        text = header.read_text()
        names += re.findall(r"TB_API\s+(?:const\s+char\s*\*|int)\s*(tb_\w+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_the_path():
    names = declared_symbols()
    for required in ("tb_int8_linear", "tb_bf16_int8_convrot_quantize",
                     "tb_codebook_w4a8_linear", "tb_dequantize_int8_bf16",
                     "tb_w4a8_linear", "tb_int4_linear",
                     "tb_quant_per_warp_int8", "tb_quant_per_block_int8"):
        assert required in names


def test_library_exports_every_declared_symbol():
    assert LIB.exists(), "libturing_b200.so was not built"
    lib = ctypes.CDLL(str(LIB))
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r" T (tb_\w+)", out))
    assert set(declared_symbols()) <= exported


def test_binding_table_matches_header():
    from comfyui_turing_utils_kernel import _lib

    assert set(_lib.SIGNATURES) | {"tb_last_error"} == set(declared_symbols())


def _lib():
    from comfyui_turing_utils_kernel import _lib as L

    return L


def test_invalid_arguments_are_rejected_with_messages():
    L = _lib()
    lib = L.load()
    fake = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    st = lib.tb_int8_linear(fake, fake, fake, fake, None, fake, 4, 8, 24, 8, 0, None)
    assert st == L.TB_ERR_INVALID
    assert L.last_error() == "Turing INT8 linear requires K%16=0 and N%8=0"
    st = lib.tb_bf16_int8_convrot_quantize(fake, 3, 300, 0, 0, fake, fake, None)
    assert st == L.TB_ERR_INVALID
    assert "divisible by 256" in L.last_error()
    st = lib.tb_bf16_int8_convrot_quantize(fake, 3, 256, 0, 640, fake, fake, None)
    assert L.last_error() == "forced_threads must be 0, 512, 768, or 1024"
    st = lib.tb_codebook_w4a8_linear(fake, fake, fake, fake, fake, fake, None, fake, 8, fake,
                                     4, 16, 32, 12, 0, 0, None)
    assert st == L.TB_ERR_INVALID
    assert L.last_error() == "unsupported Turing codebook W4A8 group size"
    st = lib.tb_w4a8_linear(fake, fake, fake, fake, None, fake, 8, fake, 4, 8, 24, 8, 0, None)
    assert st == L.TB_ERR_INVALID
    assert L.last_error() == "Turing W4A8 linear requires K%16=0 and N%8=0"
    st = lib.tb_w4a8_linear(fake, fake, fake, fake, None, None, 8, fake, 4, 8, 32, 8, 0, None)
    assert L.last_error() == "Turing W4A8 linear needs an 8-row-aligned int8 weight workspace"
    st = lib.tb_int4_linear(fake, fake, fake, fake, None, None, fake, 8, fake, 4, 8, 32, 8, None)
    assert st == L.TB_ERR_INVALID
    assert L.last_error() == "Turing W4A4 linear needs an int8 [M, K] activation workspace"
    st = lib.tb_quant_per_warp_int8(fake, 0, fake, fake, 1, 1, 64, 128, 0, 0, 128, 64, 48, 1,
                                    None)
    assert st == L.TB_ERR_INVALID
    st = lib.tb_dequantize_int8_bf16(fake, 4, fake, fake, 3, fake, 2, 8, None)
    assert L.last_error() == "output_columns must be positive and no larger than the accumulator width"


def test_convrot_entries_reject_misaligned_pointers():
    """A C host that sub-allocates its own VRAM may pass pointers off the
    16-byte boundary the ConvRot kernels' vector loads and stores need; every
    ConvRot entry rejects them before launching anything."""
    L = _lib()
    lib = L.load()
    good = ctypes.c_void_p(4096)   # never dereferenced: validation fails first
    odd = ctypes.c_void_p(4096 + 8)
    st = lib.tb_bf16_int8_convrot_quantize(odd, 4, 256, 0, 0, good, good, None)
    assert st == L.TB_ERR_INVALID
    assert L.last_error() == "ConvRot input and output must be 16-byte aligned"
    st = lib.tb_bf16_gelu_int4_convrot_quantize(good, 4, 256, odd, good, None)
    assert st == L.TB_ERR_INVALID
    assert L.last_error() == "ConvRot input and output must be 16-byte aligned"
    st = lib.tb_bf16_int4_convrot_quantize(good, 4, 256, 0, good, ctypes.c_void_p(4098), None)
    assert st == L.TB_ERR_INVALID
    assert L.last_error() == "ConvRot scales must be 4-byte aligned"
    st = lib.tb_swiglu_int8_convrot_quantize(good, L.TB_DTYPE_BF16, 4, 256, odd, good, good,
                                             good, None)
    assert st == L.TB_ERR_INVALID
    assert "scratch must be 16-byte" in L.last_error()
    st = lib.tb_swiglu_int8_convrot_quantize_noalloc(odd, L.TB_DTYPE_F16, 4, 256, good, good,
                                                     None)
    assert st == L.TB_ERR_INVALID
    assert L.last_error() == "ConvRot input and output must be 16-byte aligned"


def test_python_binding_raises_runtime_error():
    import torch

    from comfyui_turing_utils_kernel import _C

    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        _C.turing_int8_linear(torch.zeros((4, 16), dtype=torch.int8),
                              torch.zeros((8, 16), dtype=torch.int8),
                              torch.ones(4), torch.ones(8))
