"""Sequence sharding host logic, with world-size-2 gloo ranks on the CPU."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from inferd_b200.sharded import OutputGather, assign_by_tokens, gather_outputs, shard_range


@pytest.mark.parametrize("n,world", [(0, 1), (5, 1), (64, 2), (7, 2), (3, 4), (256, 8), (10, 3)])
def test_shard_range_covers_in_order(n, world):
    spans = [shard_range(n, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (lo0, hi0), (lo1, hi1) in zip(spans, spans[1:]):
        assert hi0 == lo1
    sizes = [hi - lo for lo, hi in spans]
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("workload", ["decode", "long", "verify"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_bench_shards_balance_tokens(workload, world):
    # the benchmark's ranks own every sequence once, the same number each, and within
    # 0.1 % of the mean token count (a contiguous split of the same lengths is 8.7 % off
    # at four ranks for decode)
    import bench

    lens, owners = bench.rank_shards(workload, world)
    assert sorted(i for o in owners for i in o) == list(range(lens.size))
    assert len({len(o) for o in owners}) == 1
    tokens = np.array([lens[o].sum() for o in owners])
    assert tokens.max() / tokens.mean() < 1.001
    if world == 1:
        assert owners[0] == list(range(lens.size))  # the single-GPU order is unchanged


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)
    with pytest.raises(ValueError):
        shard_range(-1, 2, 0)


def test_assign_by_tokens_balances_kv_bytes():
    rng = np.random.default_rng(0)
    lens = rng.integers(16384, 32769, size=256)  # long-context workload, 8 GPUs
    owners = assign_by_tokens(lens, 8)
    flat = sorted(i for o in owners for i in o)
    assert flat == list(range(256))
    loads = [int(lens[o].sum()) for o in owners]
    # greedy longest-first is within one sequence of the mean
    assert max(loads) - min(loads) <= int(lens.max())
    assert all(o == sorted(o) for o in owners)


def test_assign_by_tokens_more_ranks_than_sequences():
    owners = assign_by_tokens([5, 1], 4)
    assert sorted(len(o) for o in owners) == [0, 0, 1, 1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        results = {}
        # equal shards, as bench.py runs them: 3 sequences per rank of [4, 2] outputs
        local = torch.arange(12, dtype=torch.float32).view(3, 4) + 100 * rank
        results["equal"] = gather_outputs(local).tolist()
        # ragged shards from the token-balanced assignment
        counts = [2, 1]
        ragged = torch.full((counts[rank], 3), float(rank + 1))
        out = torch.empty(3, 3)
        results["ragged"] = gather_outputs(ragged, counts, out=out).tolist()
        # the decode loop's double-buffered gather: every step's result is that step's rows,
        # also when the steps' collectives are in flight together
        for counts in ([3, 3], [2, 1], [0, 4]):
            g = OutputGather((2,), torch.float32, torch.device("cpu"), counts)
            steps = []
            for step in range(5):
                buf = g.local()
                assert buf.shape == (counts[rank], 2)
                buf.copy_(torch.full((counts[rank], 2), float(1000 * step + 10 * rank)))
                buf[:, 1] += torch.arange(counts[rank], dtype=torch.float32)
                g.start()
                if step % 2:  # read every other step, as a loop that overlaps steps would
                    steps.append(g.result().tolist())
            g.wait_all()
            results[f"loop_{counts}"] = steps
        q.put((rank, results))
    finally:
        dist.destroy_process_group()


def test_gather_outputs_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect_equal = torch.cat([torch.arange(12, dtype=torch.float32).view(3, 4) + 100 * r
                              for r in range(2)]).tolist()
    expect_ragged = [[1.0] * 3, [1.0] * 3, [2.0] * 3]
    for r in range(2):
        assert got[r]["equal"] == expect_equal
        assert got[r]["ragged"] == expect_ragged
        for counts in ([3, 3], [2, 1], [0, 4]):
            want = [[[1000.0 * step + 10 * rr, 1000.0 * step + 10 * rr + i]
                     for rr in range(2) for i in range(counts[rr])] for step in (1, 3)]
            assert got[r][f"loop_{counts}"] == want, counts
