"""The multi-GPU plumbing of bench.py (weak-scaling batch shards,
strong-scaling head shards, max-over-ranks timing, whole-job tokens/s) on two
CPU ranks with the gloo backend."""

import os
import pathlib
import socket
import sys

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = pathlib.Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out, cfg):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        w = bench.workload(cfg)
        plan = bench.shard(world, rank, w)
        ms = 10.0 + 5.0 * rank  # rank 1 is the slow one
        ms_max = bench.max_over_ranks(ms, world)
        value = bench.job_tokens_per_s(w, world, ms_max)
        part = plan["rows"] if w["shard"] == "batch" else plan["heads"]
        out[rank] = (plan["seed"], part, plan["global_batch"], plan["H_local"], ms_max, value)
    finally:
        dist.destroy_process_group()


def _run(cfg, world=2):
    port = _free_port()
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(world, port, out, cfg), nprocs=world, join=True)
    return out[0], out[1]


def test_two_rank_weak_scaling_plumbing():
    (s0, r0, g0, h0, m0, v0), (s1, r1, g1, h1, m1, v1) = _run("config1")
    assert s0 != s1 and r0 == (0, 8) and r1 == (8, 16) and g0 == g1 == 16
    assert h0 == h1 == 16
    assert m0 == m1 == pytest.approx(15.0)
    assert v0 == v1 == pytest.approx(2 * 8 * 8192 / 15e-3)


def test_two_rank_head_sharded_strong_scaling_plumbing():
    # config 3: one sequence of 32 heads, 16 per rank; the job's tokens are
    # the one sequence's, over the slowest rank's time.
    (s0, p0, g0, h0, m0, v0), (s1, p1, g1, h1, m1, v1) = _run("config3")
    assert s0 != s1 and p0 == (0, 16) and p1 == (16, 32) and g0 == g1 == 1
    assert h0 == h1 == 16
    assert m0 == m1 == pytest.approx(15.0)
    assert v0 == v1 == pytest.approx(65536 / 15e-3)
