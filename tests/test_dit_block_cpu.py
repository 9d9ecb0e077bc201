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


def test_token_shards_are_whole_quantizer_blocks():
    b = db.token_shards(75600, 8)
    assert [t1 - t0 for t0, t1 in b] == [9472] * 6 + [9408, 9360]
    assert b[0][0] == 0 and b[-1][1] == 75600
    assert all(t0 % 64 == 0 for t0, _ in b) and all(b[i][1] == b[i + 1][0] for i in range(7))
    assert db.token_shards(96, 2) == [(0, 64), (64, 96)]
    assert db.token_shards(75600, 1) == [(0, 75600)]
    with pytest.raises(ValueError):
        db.token_shards(100, 4)


def _a2a_out(world: int, rank: int, L: int, group=None, split=None):
    """All-to-all sequence-parallel block (fp32 backend): this rank's tokens;
    `split` makes self-attention two launches, each returning its rows in its
    own all-to-all."""
    cfg = SMALL
    w = db.make_weights(cfg, db.shard_plan(cfg, 1, 0), seed=3)
    g = torch.Generator().manual_seed(9)
    x = torch.randn((L, cfg.dim), generator=g)
    ctx = torch.randn((16, cfg.dim), generator=g)
    freqs = db.rope_freqs(L, cfg.head_dim, seed=4, dtype=torch.float32)
    seq = db.SeqShards.make(L, world, rank, group)
    t0, t1 = seq.bounds[rank]
    block = db.DiTBlock(cfg, w, db.shard_plan(cfg, 1, 0), db.TorchOps(), seq=seq,
                        attn_split=split)
    return x, (t0, t1), block.forward(x[t0:t1], ctx, freqs)


def _a2a_rank_main(rank: int, world: int, port: int, out_dir: str, L: int, split) -> None:
    sys.path.insert(0, str(ROOT / "comfyui-turing-utils_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _, bounds, out = _a2a_out(world, rank, L, split=split)
        torch.save((bounds, out), Path(out_dir) / f"a2a{rank}.pt")
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world,L,split", [(2, 96, None), (4, 200, None), (4, 200, 100),
                                           (2, 96, 80)])
def test_all_to_all_block_equals_one_rank(tmp_path, world, L, split):
    """Token shards for the linears, head shards for self-attention, the
    all-to-alls around it: the same weights and arithmetic as one rank, so the
    rows agree to fp32 summation order (uneven shards at L = 200: 64,64,64,8;
    with `split` the attention output returns in two all-to-alls whose row
    ranges cut through shards)."""
    import torch.multiprocessing as mp

    x, _, single = _block_out(1, 0, SMALL, L)
    mp.start_processes(_a2a_rank_main, args=(world, _free_port(), str(tmp_path), L, split),
                       nprocs=world, start_method="spawn", join=True)
    full = torch.full_like(x, float("nan"))
    for r in range(world):
        (t0, t1), out = torch.load(tmp_path / f"a2a{r}.pt")
        full[t0:t1] = out
    assert not torch.isnan(full).any()
    rel = ((full - x) - (single - x)).norm() / (single - x).norm()
    assert rel < 1e-5, rel


def test_branches_and_trace_one_rank():
    """With one branch enabled only that residual is added; the trace holds
    every branch output before its add."""
    cfg = SMALL
    plan = db.shard_plan(cfg, 1, 0)
    w = db.make_weights(cfg, plan, seed=3)
    g = torch.Generator().manual_seed(9)
    x = torch.randn((64, cfg.dim), generator=g)
    ctx = torch.randn((16, cfg.dim), generator=g)
    freqs = db.rope_freqs(64, cfg.head_dim, seed=4, dtype=torch.float32)
    block = db.DiTBlock(cfg, w, plan, db.TorchOps())
    trace = []
    out = block.forward(x, ctx, freqs, branches=("ffn",), trace=trace)
    assert [t[0] for t in trace] == ["self", "cross", "ffn"]
    y = trace[2][2]
    assert torch.allclose(out, x + y * w.modulation[5].float(), atol=1e-5)


def test_reference_rows_equal_fp32_block_rows():
    cfg = SMALL
    plan = db.shard_plan(cfg, 1, 0)
    w = db.make_weights(cfg, plan, seed=3)
    g = torch.Generator().manual_seed(9)
    x = torch.randn((96, cfg.dim), generator=g)
    ctx = torch.randn((16, cfg.dim), generator=g)
    freqs = db.rope_freqs(96, cfg.head_dim, seed=4, dtype=torch.float32)
    full = db.DiTBlock(cfg, w, plan, db.TorchOps()).forward(x, ctx, freqs)
    idx = torch.tensor([0, 5, 17, 63, 64, 95])
    rows = db.reference_rows(cfg, w, x, ctx, freqs, idx)
    assert torch.allclose(rows, full[idx], rtol=1e-4, atol=1e-4), (rows - full[idx]).abs().max()


def test_phase_profiler_window(monkeypatch, caplog):
    """COMFYUI_TURING_UTILS_PROFILE_CALLS semantics (the plugin's
    profiling.py:28-95): events per phase over the first N calls, one report,
    then off; off by default."""
    from comfyui_turing_utils_kernel import profiling

    class FakeEvent:
        clock = [0.0]

        def record(self):
            FakeEvent.clock[0] += 1.5
            self.t = FakeEvent.clock[0]

        def synchronize(self):
            pass

        def elapsed_time(self, other):
            return other.t - self.t

    assert not profiling.CudaPhaseProfiler(0).enabled
    monkeypatch.setenv("COMFYUI_TURING_UTILS_PROFILE_CALLS", "2")
    prof = profiling.CudaPhaseProfiler(profiling._profile_call_limit(), FakeEvent, nvtx=False)
    monkeypatch.setattr(db, "PROFILER", prof)
    cfg = SMALL
    plan = db.shard_plan(cfg, 1, 0)
    w = db.make_weights(cfg, plan, seed=3)
    g = torch.Generator().manual_seed(9)
    x = torch.randn((64, cfg.dim), generator=g)
    ctx = torch.randn((16, cfg.dim), generator=g)
    freqs = db.rope_freqs(64, cfg.head_dim, seed=4, dtype=torch.float32)
    block = db.DiTBlock(cfg, w, plan, db.TorchOps())
    with caplog.at_level("WARNING", logger="comfyui-turing-utils"):
        for _ in range(3):
            block.forward(x, ctx, freqs)
    assert not prof.enabled and prof.calls == 2
    assert set(prof.last_report) == {"dit.norm_qkv", "dit.qk_prologue", "dit.self_attention_o",
                                     "dit.cross_attention", "dit.ffn"}
    assert all(n == 2 for n, _ in prof.last_report.values())
    assert sum("[Turing profile] attention_calls=2" in r.message for r in caplog.records) == 1
