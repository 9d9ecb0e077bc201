"""Test configuration: import paths, the `gpu` marker, and shared helpers.

CPU tests (-m "not gpu") check the oracle against the reference's known
answers and golden fixtures, the host logic, and that the C-ABI library loads
and exports every declared symbol.  GPU tests (-m gpu) are the parity tests
proper: the sm_100a kernels, called through the C ABI, against the oracle.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "comfyui-turing-utils_b200"
for p in (str(ROOT), str(PKG_DIR)):
    if p not in sys.path:
        sys.path.insert(0, p)

LIB = PKG_DIR / "comfyui_turing_utils_kernel" / "libturing_b200.so"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
    if not LIB.exists():
        # Cross-compiles for sm_100a; needs nvcc (present in the build image).
        subprocess.run(["make", "-C", str(PKG_DIR / "csrc"), "-j8"], check=False,
                       stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    """bf16/fp16 torch tensor -> uint16 numpy bits (on CPU)."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(bits: np.ndarray, dtype=torch.bfloat16) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(dtype)


def make_activation(rows: int, cols: int, seed: int, outlier_frac: float = 0.005,
                    outlier_gain: float = 20.0) -> torch.Tensor:
    """Seeded bf16 activations ~N(0,1) with a fraction of outlier channels scaled
    (the BASELINE config 1/4 distribution), generated on the CPU."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((rows, cols), generator=g, dtype=torch.float32)
    n_out = int(round(cols * outlier_frac))
    if n_out:
        idx = torch.randperm(cols, generator=g)[:n_out]
        x[:, idx] *= outlier_gain
    return x.to(torch.bfloat16)


@pytest.fixture(scope="session")
def oracle():
    import oracle as o

    o.build()
    return o
