"""The CPU restatement of the norm + AdaLN fusions (oracle.rms_adaln,
oracle.layer_norm_adaln) against the reference kernel's own outputs
(tests/golden/{rms,ln}_adaln_*.npz, made by tests/golden/make_golden.py from
kernel/csrc/turing/segmented_rms_adaln.cu).  The kernels reduce in fp32, the
oracle in float64, so outputs agree to the output dtype's last-bit rounding:
the tolerances below are two units in the last place of that dtype."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
DTYPES = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}
TOL = {"bf16": (2.0 ** -7, 2.0 ** -8), "f16": (2.0 ** -9, 2.0 ** -10), "f32": (1e-5, 2e-6)}


def values(a: np.ndarray, dtype) -> np.ndarray:
    if dtype == torch.float32:
        return a.astype(np.float64)
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(dtype).double().numpy()


@pytest.mark.parametrize("tag", sorted(DTYPES))
def test_rms_adaln_oracle_matches_reference_kernel(oracle, tag):
    dt = DTYPES[tag]
    d = np.load(GOLDEN / f"rms_adaln_{tag}.npz")
    got = oracle.rms_adaln(values(d["x"], dt), values(d["w"], dt), values(d["scale"], dt),
                           values(d["shift"], dt), d["segments"], 1e-6, dt)
    rtol, atol = TOL[tag]
    torch.testing.assert_close(torch.from_numpy(got), torch.from_numpy(values(d["out"], dt)),
                               rtol=rtol, atol=atol)


@pytest.mark.parametrize("tag", sorted(DTYPES))
def test_layer_norm_adaln_oracle_matches_reference_kernel(oracle, tag):
    dt = DTYPES[tag]
    d = np.load(GOLDEN / f"ln_adaln_{tag}.npz")
    got = oracle.layer_norm_adaln(values(d["x"], dt), values(d["scale"], dt),
                                  values(d["shift"], dt), 1e-6, dt)
    rtol, atol = TOL[tag]
    torch.testing.assert_close(torch.from_numpy(got), torch.from_numpy(values(d["out"], dt)),
                               rtol=rtol, atol=atol)


def test_segment_lookup_rules(oracle):
    seg = np.array([[0, 4, 2], [4, 9, 0], [9, 11, 1], [12, 13, 7]], np.int32)
    rows = oracle.segment_rows(seg, 14, 3)
    assert rows.tolist() == [2] * 4 + [0] * 5 + [1] * 2 + [0, 0, 0]
