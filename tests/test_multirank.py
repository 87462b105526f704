"""Multi-process host logic on CPU (gloo, world size 2): the bench's
max-over-ranks timing and its rank-0-only reference arm under torchrun."""
import json
import os
import socket
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_max(rank, world, port, out_q):
    import datetime
    import torch.distributed as dist
    sys.path.insert(0, REPO)
    import bench
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        out_q.put((rank, bench.max_over_ranks(10.0 + 5.0 * rank, dist, "cpu")))
    finally:
        dist.destroy_process_group()


def test_time_is_the_slowest_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_max, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = dict(q.get(timeout=60) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert got == {0: 15.0, 1: 15.0}


def test_single_process_max_is_identity():
    sys.path.insert(0, REPO)
    import bench
    assert bench.max_over_ranks(3.25) == 3.25


def test_reference_arm_prints_once_under_torchrun():
    env = dict(os.environ, OMP_NUM_THREADS="1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), "bench.py", "--impl", "reference",
           "--gpus", "2", "--steps", "3", "--warmup", "3", "--cpu-budget", "1"]
    res = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, res.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    assert d["cpu_baseline"]["cores"] >= 1 and d["e2e"]["h2d_bytes_per_step"] == 0
