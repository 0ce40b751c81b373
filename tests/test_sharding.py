"""Length-balanced request sharding (LPT) and the optional output gather.

The partitioner is pure host logic; the gather runs as two ``gloo`` ranks on
the CPU (the same code path that uses NCCL on GPUs, minus the transport)."""

from __future__ import annotations

import itertools
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from flashdec_b200.sharding import gather_outputs, lpt_partition, shard_loads


def _log_uniform(seed, n=64):
    rng = np.random.default_rng(seed)
    return [int(x) for x in np.exp(rng.uniform(np.log(512), np.log(131072), size=n))]


@pytest.mark.parametrize("ranks", [1, 2, 3, 4, 8])
def test_lpt_is_a_partition_and_balanced(ranks):
    lens = _log_uniform(4)
    shards = lpt_partition(lens, ranks)
    flat = sorted(itertools.chain.from_iterable(shards))
    assert flat == list(range(len(lens)))
    for s in shards:
        assert s == sorted(s)
    loads = shard_loads(lens, shards)
    # Graham's bound for LPT: makespan <= 4/3 OPT, and OPT >= max(mean, longest)
    opt_lb = max(sum(lens) / ranks, max(lens))
    assert max(loads) <= 4 / 3 * opt_lb + 1e-9


def test_lpt_is_deterministic_with_ties_to_lower_rank():
    assert lpt_partition([5, 5, 5, 5], 2) == [[0, 2], [1, 3]]
    assert lpt_partition([1, 9, 3], 2) == [[1], [0, 2]]
    assert lpt_partition([], 3) == [[], [], []]
    with pytest.raises(ValueError):
        lpt_partition([1], 0)


def test_lpt_matches_exhaustive_optimum_on_small_cases():
    rng = np.random.default_rng(0)
    for _ in range(30):
        lens = [int(x) for x in rng.integers(1, 100, size=7)]
        best = min(max(sum(lens[i] for i in range(7) if assign[i] == r) for r in range(3))
                   for assign in itertools.product(range(3), repeat=7))
        got = max(shard_loads(lens, lpt_partition(lens, 3)))
        assert got <= 4 / 3 * best + 1e-9


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, lens, dst, result_q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shards = lpt_partition(lens, world)
        hq, d = 4, 8
        full = torch.arange(len(lens) * hq * d, dtype=torch.float32).view(len(lens), hq, d)
        local = full[shards[rank]] if shards[rank] else full[:0]
        out = gather_outputs(local, shards, rank, dst=dst)
        ok = (out is None and dst is not None and rank != dst) or (
            out is not None and torch.equal(out, full))
        result_q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dst", [None, 0])
def test_gather_outputs_two_gloo_ranks(dst):
    lens = [700, 90000, 512, 30000, 1200]  # uneven shards (3 + 2 rows)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, lens, dst, q))
             for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == {0: True, 1: True}


def _c4_worker(rank, world, port, result_q):
    """LPT shards of BASELINE c4's 64 requests, each rank holding only its
    rows, reassembled on every rank by the gather."""
    import torch.distributed as dist

    from tests.golden.cases import c4_lengths

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lens = c4_lengths()
        shards = lpt_partition(lens, world)
        hq, d = 32, 4
        # row r carries the request's own index and length: the gather must
        # put every row back at its request's position
        full = torch.zeros(len(lens), hq, d)
        for r, n in enumerate(lens):
            full[r, :, 0] = r
            full[r, :, 1] = n
        out = gather_outputs(full[shards[rank]], shards, rank)
        loads = shard_loads(lens, shards)
        ok = torch.equal(out, full) and max(loads) <= 4 / 3 * max(sum(lens) / world, max(lens))
        result_q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_c4_shards_and_gather_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_c4_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == {0: True, 1: True}
