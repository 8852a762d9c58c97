"""Sharding of independent sequences across GPUs (CPU; the N > 1 path with
world_size-2 gloo process groups)."""
import os
import socket

import pytest

from zynfer_b200 import shard, workload


def test_assignment_covers_every_sequence_once():
    lens = workload.prompt_lengths(64, 20250601)
    for world in (1, 2, 4, 8):
        parts = shard.assign_sequences(lens, world, 136)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(64))
        sizes = [len(p) for p in parts]
        assert max(sizes) - min(sizes) <= 1
        loads = [sum(lens[i] for i in p) for p in parts]
        assert max(loads) / (sum(loads) / world) < 1.05  # length-balanced within 5%


def test_prompt_lengths_in_range_and_seeded():
    a = workload.prompt_lengths(64, 1)
    assert a == workload.prompt_lengths(64, 1)
    assert all(512 <= x <= 4096 for x in a)
    assert workload.prompt(3, 10, 1).tolist() == workload.prompt(3, 10, 1).tolist()
    assert max(workload.prompt(0, 1000, 1)) < 151936


def test_workload_tokens_match_oracle_generator():
    from oracle import oracle as O
    assert workload.tokens(500, 7, 1003).tolist() == O.synth_tokens(500, 7, 1003, 151936).tolist()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lens = workload.prompt_lengths(64, 20250601)
    mine = shard.assign_sequences(lens, world, 136)[rank]
    t = shard.max_over_ranks(10.0 + rank)
    s = shard.sum_over_ranks(float(len(mine)))
    rows = shard.gather_over_ranks([float(rank), float(len(mine)), 0.5])
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, mine, t, s, rows))


def test_two_rank_gloo_max_over_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][2] == res[1][2] == 11.0       # slowest rank sets the time
    assert res[0][3] == res[1][3] == 64.0       # every sequence is somewhere
    assert sorted(res[0][1] + res[1][1]) == list(range(64))
    for r in res:                                # per-rank rows reach every rank in rank order
        assert r[4] == [[0.0, 32.0, 0.5], [1.0, 32.0, 0.5]]
