"""TEST INFRASTRUCTURE ONLY: loaders for the reference's own CUDA kernels built
by oracle/ref/build_ref.py into oracle/_ref (the unmodified reference sources
compiled for sm_100a).  Used by tests/golden/make_golden.py and the GPU tests
that compare this repository's kernels with the reference's on the same
inputs.  Nothing in the product imports this module."""
from __future__ import annotations

import ctypes
import importlib.machinery
import importlib.util
from pathlib import Path

import torch

REF_DIR = Path(__file__).resolve().parent / "_ref"
_p, _i = ctypes.c_void_p, ctypes.c_int


def available() -> bool:
    return (REF_DIR / "libref_linear.so").exists() and any(REF_DIR.glob("ref_sage*.so"))


def linear():
    lib = ctypes.CDLL(str(REF_DIR / "libref_linear.so"))
    lib.ref_bf16_convrot.argtypes = [_p, _i, _i, _i, _i, _i, _p, _p, _p]
    lib.ref_staged_convrot.argtypes = [_p, _i, _i, _i, _i, _i, _p, _p, _p, _p, _p]
    lib.ref_int8_linear.argtypes = [_p, _p, _p, _p, _p, _p, _i, _i, _i, _p]
    lib.ref_w4a8_linear.argtypes = [_p, _p, _p, _p, _p, _p, _i, _i, _i, _p]
    lib.ref_codebook_linear.argtypes = [_p, _p, _p, _p, _p, _p, _p, _p, _i, _p, _i, _i, _i, _i, _p]
    lib.ref_dequant.argtypes = [_p, _p, _p, _i, _p, _i, _i, _p]
    lib.ref_segmented_rms_adaln.argtypes = [_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i,
                                            ctypes.c_float, _p]
    lib.ref_layer_norm_adaln.argtypes = [_p, _p, _p, _p, _i, _i, _i, _i, _i, ctypes.c_float, _p]
    return lib


def sage():
    torch.ops.load_library  # torch must be imported before the extension
    so = next(REF_DIR.glob("ref_sage*.so"))
    loader = importlib.machinery.ExtensionFileLoader("ref_sage", str(so))
    spec = importlib.util.spec_from_file_location("ref_sage", str(so), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"reference kernel {what} failed")
