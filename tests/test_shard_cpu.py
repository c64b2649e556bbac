"""Env sharding host logic on CPU ranks (gloo, world size 2)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lewm_flash_b200.shard import env_range, gather_plans, plan_shard, shard_inputs


@pytest.mark.parametrize("n,world", [(0, 3), (1, 2), (7, 2), (1024, 8), (256, 8), (5, 8)])
def test_env_ranges_partition_contiguously(n, world):
    ranges = [env_range(n, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (s0, e0), (s1, e1) in zip(ranges, ranges[1:]):
        assert e0 == s1
    sizes = [e - s for s, e in ranges]
    assert max(sizes) - min(sizes) <= 1


def test_env_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        env_range(10, 2, 2)


def _fake_plan(emb, goal):
    """Stand-in for a device plan: per-env outputs that depend only on that env."""
    return (emb.sum(-1, keepdim=True) * 2.0, goal[:, :3] + 1.0)


def _worker(rank, world, port, n_envs, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        emb = torch.randn(n_envs, 4, generator=g)
        goal = torch.randn(n_envs, 6, generator=g)
        local = plan_shard(_fake_plan, {"emb": emb, "goal": goal}, rank, world)
        out = gather_plans(local, n_envs, [(1,), (3,)])
        if rank == 0:
            want = _fake_plan(emb, goal)
            q.put([bool(torch.equal(o, w)) for o, w in zip(out, want)])
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n_envs", [5, 1])
def test_two_rank_gather_reassembles_env_order(n_envs):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_envs, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=10) == [True, True]


def test_shard_inputs_requires_common_env_dim():
    with pytest.raises(ValueError):
        shard_inputs({"a": torch.zeros(3, 2), "b": torch.zeros(4, 2)}, 0, 2)
