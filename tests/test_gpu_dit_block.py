"""The DiT block on the sm_100a kernels against the fp32 torch reference
block with the same dequantized weights (the reference's dequantize-then-
compute path composed), and its tensor-parallel form on two GPUs (NCCL)
against one GPU.  The block's output is x plus three residual branches, so
the comparison is on the branches' sum (out - x).  Bound: relative L2 of the
branch sum <= 3e-2 and cosine >= 0.999 — the INT8 activations of seven
linears and two attentions each add ~1e-2 relative noise, bf16 storage of
every intermediate the rest."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

from comfyui_turing_utils_kernel import _lib  # noqa: E402
from comfyui_turing_utils_kernel import dit_block as db  # noqa: E402

ROOT = Path(__file__).resolve().parent.parent
SMALL = db.BlockConfig(dim=1024, heads=8, head_dim=128, ffn=2560)


def _inputs(cfg, L, Lc, seed=9, device="cuda"):
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn((L, cfg.dim), generator=g, device=device).to(torch.bfloat16)
    ctx = torch.randn((Lc, cfg.dim), generator=g, device=device).to(torch.bfloat16)
    return x, ctx, db.rope_freqs(L, cfg.head_dim, seed=4, device=device)


def _compare(out, ref, x):
    d_out = out.float() - x.float()
    d_ref = ref.float() - x.float()
    rel = ((d_out - d_ref).norm() / d_ref.norm()).item()
    cos = torch.nn.functional.cosine_similarity(d_out.flatten(), d_ref.flatten(), dim=0).item()
    return rel, cos


@pytest.mark.parametrize("cfg,L,Lc,split", [(SMALL, 300, 40, None), (db.BlockConfig(), 640, 64, None),
                                            (SMALL, 600, 40, 256)])
def test_block_matches_fp32_reference(cfg, L, Lc, split):
    """split: self-attention in two launches (rows [0, split) and
    [split, L)), the O projection of finished rows between them."""
    plan = db.shard_plan(cfg, 1, 0)
    w = db.make_weights(cfg, plan, seed=3, device="cuda")
    x, ctx, freqs = _inputs(cfg, L, Lc)
    out = db.DiTBlock(cfg, w, plan, db.KernelOps(), attn_split=split).forward(x, ctx, freqs)
    assert out.dtype == torch.bfloat16 and out.shape == x.shape
    ref = db.DiTBlock(cfg, w, plan, db.TorchOps()).forward(x.float(), ctx, freqs.float())
    rel, cos = _compare(out, ref, x)
    assert rel <= 3e-2 and cos >= 0.999, (rel, cos)
    assert _lib.device_error() == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_rank(rank: int, world: int, port: int, out_dir: str) -> None:
    import datetime

    sys.path.insert(0, str(ROOT / "comfyui-turing-utils_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=120),
                                         device_id=torch.device("cuda", rank))
    try:
        plan = db.shard_plan(SMALL, world, rank)
        w = db.make_weights(SMALL, plan, seed=3, device="cuda")
        x, ctx, freqs = _inputs(SMALL, 300, 40)
        rows = db.local_rows(300, world, rank, db.token_chunks(300, world))
        out = db.DiTBlock(SMALL, w, plan, db.KernelOps(),
                          group=torch.distributed.group.WORLD).forward(x[rows.cuda()], ctx, freqs)
        torch.cuda.synchronize()
        torch.save((rows, out.cpu()), Path(out_dir) / f"out{rank}.pt")
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.timeout(600)
def test_tensor_parallel_two_gpus(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_tp_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    plan = db.shard_plan(SMALL, 1, 0)
    w = db.make_weights(SMALL, plan, seed=3, device="cuda")
    x, ctx, freqs = _inputs(SMALL, 300, 40)
    full = torch.full_like(x, float("nan"))
    for r in range(2):
        rows, out = torch.load(tmp_path / f"out{r}.pt")
        full[rows.cuda()] = out.cuda()
    assert not torch.isnan(full).any()
    ref = db.DiTBlock(SMALL, w, plan, db.TorchOps()).forward(x.float(), ctx, freqs.float())
    rel, cos = _compare(full, ref, x)
    assert rel <= 3e-2 and cos >= 0.999, (rel, cos)
