"""GPU parity: Sage Q/K INT8 quantizers vs the CPU oracle (codes and scales
bit-exact under the IEEE-divide definition both use)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_bits

pytestmark = pytest.mark.gpu

from comfyui_turing_utils_kernel.turing_sage import quant  # noqa: E402


@pytest.mark.parametrize("layout", ["HND", "NHD"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("L,D", [(1, 64), (63, 128), (65, 64), (129, 128), (151, 128),
                                 (4096, 128)])
def test_per_warp_and_per_block(oracle, layout, dtype, L, D):
    g = torch.Generator().manual_seed(L * 3 + D)
    q = (torch.randn((2, 3, L, D), generator=g) * 0.7).to(dtype)
    k = (torch.randn((2, 3, L, D), generator=g) + torch.randn((2, 3, 1, D), generator=g) * 2).to(dtype)
    if layout == "NHD":
        q, k = q.transpose(1, 2).contiguous(), k.transpose(1, 2).contiguous()
    fp16 = dtype == torch.float16
    q8, qs, k8, ks = quant.per_warp_int8(q.cuda(), k.cuda(), tensor_layout=layout)
    wq, wqs = oracle.sage_quant(bf16_bits(q), 16, layout=layout, fp16=fp16, block=64)
    wk, wks = oracle.sage_quant(bf16_bits(k), 64, layout=layout, fp16=fp16)
    assert np.array_equal(q8.cpu().numpy(), wq) and np.array_equal(qs.cpu().numpy(), wqs)
    assert np.array_equal(k8.cpu().numpy(), wk) and np.array_equal(ks.cpu().numpy(), wks)
    k8s, kss = quant.quantize_key_per_block(k.cuda(), tensor_layout=layout, smooth_k=True)
    mean = oracle.token_mean(bf16_bits(k), layout=layout, fp16=fp16)
    wk2, wks2 = oracle.sage_quant(bf16_bits(k), 64, layout=layout, fp16=fp16, mean_bits=mean)
    assert np.array_equal(k8s.cpu().numpy(), wk2) and np.array_equal(kss.cpu().numpy(), wks2)


def test_strided_input():
    """Last-dim-contiguous views (a slice of a fused QKV buffer) quantize like
    their contiguous copy."""
    base = torch.randn((1, 128, 3, 4, 64), device="cuda").to(torch.bfloat16)
    q = base[:, :, 0]  # NHD view with non-contiguous strides
    q8a, qsa = quant.quantize_query_per_warp(q, tensor_layout="NHD")
    q8b, qsb = quant.quantize_query_per_warp(q.contiguous(), tensor_layout="NHD")
    assert torch.equal(q8a, q8b) and torch.equal(qsa, qsb)
