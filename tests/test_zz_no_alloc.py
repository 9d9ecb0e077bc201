"""The allocation-free SwiGLU INT8 ConvRot quantizer.

tb_swiglu_int8_convrot_quantize_noalloc serves callers that cannot allocate
device memory when they quantize (a host whose memory manager owns all VRAM,
or a path that must not take cudaMalloc's implicit synchronisation): its
scratch is a fixed 16 MiB array in the library's device image.  These tests
call it through the C ABI and compare it with the allocating entry point
tb_swiglu_int8_convrot_quantize (caller-owned scratch), bit for bit, on two
calls in a row so a stale scratch array would show.  This file is collected
last so a run that stops at the first failure has run everything else.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from comfyui_turing_utils_kernel import _lib


def _noalloc(x: torch.Tensor, hidden: int):
    out = torch.empty((x.size(0), hidden), dtype=torch.int8, device=x.device)
    scales = torch.empty((x.size(0), 1), dtype=torch.float32, device=x.device)
    _lib.call("tb_swiglu_int8_convrot_quantize_noalloc", _lib.ptr(x), _lib.dtype_code(x),
              x.size(0), hidden, _lib.ptr(out), _lib.ptr(scales), _lib.stream_of(x))
    return out, scales


def _allocating(x: torch.Tensor, hidden: int):
    rows = x.size(0)
    rotated = torch.empty((rows, hidden), dtype=x.dtype, device=x.device)
    partial = torch.empty((rows, hidden // 256), dtype=torch.float32, device=x.device)
    out = torch.empty((rows, hidden), dtype=torch.int8, device=x.device)
    scales = torch.empty((rows, 1), dtype=torch.float32, device=x.device)
    _lib.call("tb_swiglu_int8_convrot_quantize", _lib.ptr(x), _lib.dtype_code(x), rows, hidden,
              _lib.ptr(rotated), _lib.ptr(partial), _lib.ptr(out), _lib.ptr(scales),
              _lib.stream_of(x))
    return out, scales


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_noalloc_matches_allocating_entry_point_twice(dtype):
    hidden = 5120
    for call, (rows, seed) in enumerate([(257, 11), (64, 12)]):
        g = torch.Generator().manual_seed(seed)
        x = (torch.randn((rows, 2 * hidden), generator=g) * (1 + call)).to(dtype).cuda()
        got_q, got_s = _noalloc(x, hidden)
        want_q, want_s = _allocating(x, hidden)
        torch.cuda.synchronize()
        assert torch.equal(got_q, want_q), f"codes differ on call {call}"
        assert torch.equal(got_s, want_s), f"scales differ on call {call}"
    assert _lib.device_error() == 0


# The largest problem at hidden 5120 that fits the 16 MiB scratch:
# rows * 5120 * 2 rotated bytes (already a multiple of 256) + rows * 80 bytes
# of partial absmax = 10320 * rows <= 16 * 2**20, so 1625 rows (16,770,000
# bytes); 1626 rows need 16,780,320 bytes.
FULL_ROWS = 1625


@pytest.mark.gpu
def test_noalloc_fills_its_scratch_exactly():
    """At the size limit the partial absmax ends within 7 KB of the array's
    end: an off-by-one in where it starts would overflow the array or
    overlap the rotated rows, and the codes would differ."""
    hidden = 5120
    assert FULL_ROWS * hidden * 2 + FULL_ROWS * hidden // 64 <= 16 << 20
    assert (FULL_ROWS + 1) * hidden * 2 + (FULL_ROWS + 1) * hidden // 64 > 16 << 20
    for seed in (21, 22):
        g = torch.Generator().manual_seed(seed)
        x = torch.randn((FULL_ROWS, 2 * hidden), generator=g).to(torch.bfloat16).cuda()
        got_q, got_s = _noalloc(x, hidden)
        want_q, want_s = _allocating(x, hidden)
        torch.cuda.synchronize()
        assert torch.equal(got_q, want_q)
        assert torch.equal(got_s, want_s)
    assert _lib.device_error() == 0


def test_noalloc_rejects_problems_larger_than_its_scratch():
    fake = ctypes.c_void_p(16)  # never dereferenced: the size check fails first
    status = _lib.load().tb_swiglu_int8_convrot_quantize_noalloc(
        fake, _lib.TB_DTYPE_BF16, 4096, 5120, fake, fake, None)
    assert status == _lib.TB_ERR_INVALID
    assert "16 MiB" in _lib.last_error()
    # One row more than the largest problem that fits.
    status = _lib.load().tb_swiglu_int8_convrot_quantize_noalloc(
        fake, _lib.TB_DTYPE_BF16, FULL_ROWS + 1, 5120, fake, fake, None)
    assert status == _lib.TB_ERR_INVALID
    assert "16 MiB" in _lib.last_error()
