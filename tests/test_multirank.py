"""The bench's multi-GPU host logic on CPU ranks (gloo, world size 2): every rank its own independent sequences,
the job's time the slowest rank's, the reference arm's work on rank 0 only."""
import json
import multiprocessing as mp
import os
import socket
import subprocess
import sys
from datetime import timedelta

import numpy as np

from conftest import ROOT

sys.path.insert(0, str(ROOT))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import torch.distributed as dist

    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        prompts = bench.rank_prompts(4, 16, 1000, rank)
        slowest = bench.max_over_ranks(10.0 + 5.0 * rank, world, "cpu")
        out.put((rank, prompts.tolist(), slowest))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_ranks_shard_sequences_and_take_the_slowest():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict((r, (np.array(pr), sl)) for r, pr, sl in (out.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert not np.array_equal(got[0][0], got[1][0])  # independent sequences, not a split of one
    assert (got[0][0][:, 0] == 1).all() and (got[1][0][:, 0] == 1).all()  # each starts with BOS
    assert got[0][1] == got[1][1] == 15.0  # both ranks report the slowest rank's time


def test_reference_arm_works_on_rank_zero_only():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2")
    run = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--model", "stories15m",
                          "--steps", "1", "--warmup", "1"], env=env, capture_output=True, text=True, timeout=300)
    assert run.returncode == 0 and run.stdout.strip() == ""
    env = dict(os.environ, RANK="0", WORLD_SIZE="1")
    run = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--model", "stories15m",
                          "--steps", "1", "--warmup", "1"], env=env, capture_output=True, text=True, timeout=300)
    assert run.returncode == 0
    line = json.loads(run.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["cpu_baseline"]["kind"] == "port"
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["config"]["model"] == "stories15m"
