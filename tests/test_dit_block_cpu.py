"""DiT block host logic on the CPU: the tensor-parallel shard plan (whole
256-channel ConvRot groups per rank), the weight quantization round trip, and
the tensor-parallel block on world-size-2 gloo ranks with the fp32 torch
backend against the same block on one rank."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch

from comfyui_turing_utils_kernel import dit_block as db

ROOT = Path(__file__).resolve().parent.parent
SMALL = db.BlockConfig(dim=1024, heads=8, head_dim=128, ffn=2560)


def test_shard_plan_matches_convrot_groups():
    cfg = db.BlockConfig()
    p8 = db.shard_plan(cfg, 8, 0)
    assert p8.heads == (6, 4, 6, 4, 6, 4, 6, 4) and p8.attn == (5,) * 8
    # Each 6-head O shard takes one head of attention output from its neighbour.
    assert p8.head_moves() == [(1, 0, 5, 1), (3, 2, 15, 1), (5, 4, 25, 1), (7, 6, 35, 1)]
    assert db.shard_plan(cfg, 8, 0).ffn == tuple([7 * 256] * 6 + [6 * 256] * 2)
    assert db.shard_plan(cfg, 4, 0).heads == (10, 10, 10, 10)
    assert db.shard_plan(cfg, 2, 1).head0 == 20 and db.shard_plan(cfg, 2, 1).ffn0 == 27 * 256
    assert db.shard_plan(cfg, 4, 0).head_moves() == []
    for world in (1, 2, 4, 8):
        p = db.shard_plan(cfg, world, 0)
        assert sum(p.heads) == 40 and sum(p.ffn) == 13824
        assert all(h * 128 % 256 == 0 for h in p.heads) and all(f % 256 == 0 for f in p.ffn)
    with pytest.raises(ValueError):
        db.shard_plan(cfg, 32, 0)


def test_sequence_parallel_layout():
    assert db.token_chunks(75600, 8) == 3 and db.token_chunks(75600, 1) == 1
    rows = [db.local_rows(96, 2, r, 4) for r in range(2)]
    assert sorted(torch.cat(rows).tolist()) == list(range(96))
    assert rows[0][:12].tolist() == list(range(12)) and rows[1][:12].tolist() == list(range(12, 24))
    with pytest.raises(ValueError):
        db.token_chunks(75601, 2)


def test_ops_count_matches_config():
    assert abs(db.block_ops(db.BlockConfig(), 75600, 512) / 1e12 - 163.08) < 0.01


def test_quantized_weight_round_trip():
    w = torch.randn(64, 512) * 0.02
    ql = db.QuantLinear.from_float(w, None)
    h = db.hadamard256()
    assert torch.allclose(h @ h, torch.eye(256), atol=1e-6) and torch.equal(h, h.t())
    err = (ql.dequantized() - w).norm() / w.norm()
    assert err < 0.02, err


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


MOVES = db.BlockConfig(dim=2560, heads=20, head_dim=128, ffn=6912)  # 4 ranks: heads 6/4/6/4


def _block_out(world: int, rank: int, cfg=SMALL, L=96):
    """(full x, this rank's token indices, this rank's output tokens)."""
    torch.manual_seed(0)
    plan = db.shard_plan(cfg, world, rank)
    w = db.make_weights(cfg, plan, seed=3)
    g = torch.Generator().manual_seed(9)
    x = torch.randn((L, cfg.dim), generator=g)
    ctx = torch.randn((16, cfg.dim), generator=g)
    freqs = db.rope_freqs(L, cfg.head_dim, seed=4, dtype=torch.float32)
    rows = db.local_rows(L, world, rank, db.token_chunks(L, world))
    block = db.DiTBlock(cfg, w, plan, db.TorchOps(), group=None)
    return x, rows, block.forward(x[rows], ctx, freqs, L=L)


def _rank_main(rank: int, world: int, port: int, out_dir: str, moves: bool) -> None:
    sys.path.insert(0, str(ROOT / "comfyui-turing-utils_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _, rows, out = _block_out(world, rank, *((MOVES, 64) if moves else (SMALL, 96)))
        torch.save((rows, out), Path(out_dir) / f"out{rank}.pt")
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world,moves", [(2, False), (4, True)])
def test_tensor_parallel_block_equals_one_rank(tmp_path, world, moves):
    """World 4 on the 20-head config moves one head of attention output from
    each 4-head O shard's rank to its 6-head neighbour."""
    import torch.multiprocessing as mp

    x, _, single = _block_out(1, 0, *((MOVES, 64) if moves else (SMALL, 96)))
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), moves),
                       nprocs=world, start_method="spawn", join=True)
    full = torch.full_like(x, float("nan"))
    for r in range(world):
        rows, out = torch.load(tmp_path / f"out{r}.pt")
        full[rows] = out
    assert not torch.isnan(full).any()            # the ranks' tokens cover the sequence once
    delta_tp, delta_1 = full - x, single - x
    rel = (delta_tp - delta_1).norm() / delta_1.norm()
    # Row-parallel weights are quantized per shard (their own per-channel
    # scales over the shard's columns), so the two runs differ by weight
    # rounding only.
    assert rel < 0.02, rel
