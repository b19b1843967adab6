"""KV-head sharding across the GPUs of one node.

The cache operation shards the way SGLang tensor parallelism shards the KV
pool: each rank holds ``tp_k_head_num`` of the KV heads of every layer
(akv/system/sglang.patch:2100) and replicates the request metadata (the
scheduler state is identical on every TP rank, srt/context_system/ir.py:129).
Drop metadata is therefore computed on every rank, reposition and decode
attention touch only the rank's heads, and no data crosses GPUs: the only
communication is a barrier around timed regions and a MAX reduction of the
timings.
"""

from __future__ import annotations

import torch


def kv_head_range(rank: int, world: int, kv_heads: int) -> tuple[int, int]:
    """Heads [start, end) of ``rank``; the heads must split evenly."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank outside the world")
    if kv_heads % world:
        raise ValueError(f"{kv_heads} KV heads do not split over {world} ranks")
    per = kv_heads // world
    return rank * per, (rank + 1) * per


def shard_heads(pool: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """The rank's [slots, heads_local, dim] slice of a full [slots, heads, dim] pool."""
    a, b = kv_head_range(rank, world, pool.shape[1])
    return pool[:, a:b]


def max_over_ranks(value: float, group=None) -> float:
    """MAX all-reduce of a scalar (a timing) over the ranks of ``group``."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return value
    device = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
