"""CPU (gloo, world_size 2) tests of the multi-rank plumbing of bench.py: one process per
rank, barriers, max-over-ranks timing, per-rank data shards, and the reference arm under
torchrun (rank 0 alone works, the other rank exits cleanly)."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import REPO


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out) -> None:
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    sys.path.insert(0, str(REPO))
    import bench
    d = bench.Dist(world, backend="gloo")
    d.barrier()
    worst = d.max(10.0 + rank)  # each rank's "elapsed ms"
    p = bench.prompts_for(d.rank, 4, 8, 100)
    out.put((rank, worst, p.tolist()))
    d.barrier()
    d.close()


def test_two_rank_gloo_timing_and_shards():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[1] for r in res] == [11.0, 11.0]          # max over ranks on every rank
    assert res[0][2] != res[1][2]                        # each rank holds its own sequences
    assert np.array(res[0][2]).shape == (4, 8)


def test_reference_arm_under_torchrun_two_ranks(tmp_path):
    env = dict(os.environ, LLX_ARTEFACTS=str(tmp_path / "art"), CUDA_VISIBLE_DEVICES="")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(REPO / "bench.py"),
           "--impl", "reference", "--gpus", "2", "--config", "c1", "--steps", "1", "--warmup", "1",
           "--cpu-decode", "2"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=str(tmp_path))
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1  # rank 0 alone prints
    import json
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference" and rec["value"] > 0 and rec["e2e"]["h2d_bytes_per_step"] == 0
    assert rec["cpu_baseline"]["kind"] == "port"
