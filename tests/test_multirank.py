"""The bench's multi-GPU host logic on CPU ranks (gloo, world size 2): the workload's sequences split evenly over the
ranks, every sequence's generated ids all-gathered in rank order, the job's time the slowest rank's, the reference
arm's work on rank 0 only."""
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
        mine = bench.shard(8, world, rank)
        prompts = bench.workload_prompts(8, 16, 1000)[mine]
        # each rank's "generated ids": its sequences' prompt heads, so the gathered table is known in advance
        ids = prompts[:, :5] + 7
        gathered = bench.gather_ids(ids, world, "cpu").numpy()
        slowest = bench.max_over_ranks(10.0 + 5.0 * rank, world, "cpu")
        out.put((rank, prompts.tolist(), gathered.tolist(), slowest))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_ranks_split_the_sequences_gather_the_ids_and_take_the_slowest():
    import bench

    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict((r, (np.array(pr), np.array(ga), sl)) for r, pr, ga, sl in (out.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    every = bench.workload_prompts(8, 16, 1000)
    # rank r holds sequences 4r .. 4r + 3 of the one workload: together all of them, once
    assert np.array_equal(np.concatenate([got[0][0], got[1][0]]), every)
    assert (every[:, 0] == 1).all()  # each starts with BOS
    # both ranks end with every sequence's ids, in sequence order
    for r in (0, 1):
        assert np.array_equal(got[r][1], every[:, :5] + 7)
    assert got[0][2] == got[1][2] == 15.0  # both ranks report the slowest rank's time


def test_the_split_is_even_or_refused():
    import bench

    assert [bench.shard(64, 8, r) for r in (0, 7)] == [slice(0, 8), slice(56, 64)]
    assert bench.shard(64, 1, 0) == slice(0, 64)
    try:
        bench.shard(64, 3, 0)
    except SystemExit as e:
        assert "evenly" in str(e)
    else:
        raise AssertionError("an uneven split was accepted")


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
