"""Sharding independent sequences across GPUs (one process per GPU, no collective
on the hot path). Sequences are independent in the reference (one Session per
sequence, src/model/qwen_forward.zig:21-31), so a batch shards by sequence:
each rank holds a full weight replica and its own sequences' KV cache.
"""
from __future__ import annotations


def assign_sequences(lengths: list[int], world: int, extra_tokens: int = 0) -> list[list[int]]:
    """Length-balanced assignment: sequences in decreasing final length go to
    the rank with the least KV so far (ties: fewer sequences, then lower rank).
    Every rank gets len(lengths) // world or one more sequence."""
    n = len(lengths)
    if world <= 0:
        raise ValueError("world must be positive")
    cap = [n // world + (1 if r < n % world else 0) for r in range(world)]
    load = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(n), key=lambda j: (-(lengths[j] + extra_tokens), j)):
        r = min((r for r in range(world) if len(out[r]) < cap[r]), key=lambda r: (load[r], len(out[r]), r))
        out[r].append(i)
        load[r] += lengths[i] + extra_tokens
    for o in out:
        o.sort()
    return out


def max_over_ranks(value: float, device=None) -> float:
    """MAX all-reduce of one float (timing: the slowest rank sets the time)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device=None) -> float:
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_over_ranks(values: list[float], device=None) -> list[list[float]]:
    """All-gather one row of floats per rank (rank order); off the hot path."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [list(map(float, values))]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [o.tolist() for o in out]
