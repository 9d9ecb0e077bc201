"""Host logic of the multi-GPU bench path, run as world-size-2 ``gloo`` ranks on
the CPU: process-group set-up from the torchrun environment, the barrier, the
max-over-ranks timing reduction, the reference arm's rank-0-only rule, and a
rank that fails before its collective (the survivor's collective ends with an
error instead of waiting forever)."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path
from types import SimpleNamespace

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str, fail_rank: int) -> None:
    import datetime

    sys.path.insert(0, str(ROOT))
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    import bench

    if fail_rank >= 0:
        # Short process-group timeout: a survivor must not wait for long.
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=5))
        world_, rank_ = dist.get_world_size(), dist.get_rank()
    else:
        world_, rank_, _ = bench.dist_setup(SimpleNamespace(impl="ours"))
    result = {"world": world_, "rank": rank_}
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        bench.barrier(world_)
        result["max"] = bench.max_over_ranks(1.5 + rank, world_)
        bench.barrier(world_)
    except Exception as exc:  # recorded for the parent; the rank exits normally
        result["error"] = type(exc).__name__
    Path(out_dir, f"rank{rank}.json").write_text(json.dumps(result))
    if fail_rank < 0:
        dist.destroy_process_group()


def _spawn(tmp_path, fail_rank=-1):
    import torch.multiprocessing as mp

    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path), fail_rank), nprocs=2,
                       start_method="spawn", join=True)
    return [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(2)]


def test_setup_barrier_and_max_over_ranks(tmp_path):
    res = _spawn(tmp_path)
    assert [r["world"] for r in res] == [2, 2]
    assert [r["rank"] for r in res] == [0, 1]
    assert [r["max"] for r in res] == [2.5, 2.5]


def test_failed_rank_ends_the_survivors_collective_with_an_error(tmp_path):
    res = _spawn(tmp_path, fail_rank=1)
    assert res[1]["error"] == "RuntimeError"
    assert "error" in res[0] and "max" not in res[0]


@pytest.mark.timeout(600)
def test_reference_arm_prints_one_line_from_rank_zero():
    port = _free_port()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), str(ROOT / "bench.py"),
           "--gpus", "2", "--impl", "reference", "--workload", "linear", "--steps", "1",
           "--warmup", "0", "--cpu-rows", "4"]
    env = dict(os.environ, OMP_NUM_THREADS="2")
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=540, env=env, cwd=ROOT)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [line for line in proc.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference" and rec["n_gpus"] == 2
    assert rec["cpu_baseline"]["kind"] == "port"
    assert rec["e2e"]["h2d_bytes_per_step"] == 0
