"""KV-head-group sharding of the attention path across the GPUs of one node.

Matches the reference's tensor-parallel head split (nanovllm/engine/model_runner.py:111,
nanovllm/models/qwen3.py:56-59): rank r of g holds kv heads [r*KVH/g, (r+1)*KVH/g) and the q heads
of those groups, with its own cache; block tables, lengths and slot mappings are the same on every
rank.  Attention never crosses a kv-head group, so the path needs no collective: the heads meet
again in the engine's all-reduce after o_proj.
"""
from __future__ import annotations

import torch


def kv_head_range(num_kv_heads: int, rank: int, world: int) -> tuple[int, int]:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} kv heads do not split over {world} ranks")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def q_head_range(num_heads: int, num_kv_heads: int, rank: int, world: int) -> tuple[int, int]:
    if num_heads % num_kv_heads:
        raise ValueError(f"{num_heads} q heads are not a multiple of {num_kv_heads} kv heads")
    lo, hi = kv_head_range(num_kv_heads, rank, world)
    group = num_heads // num_kv_heads
    return lo * group, hi * group


def shard_q(q: torch.Tensor, num_kv_heads: int, rank: int, world: int) -> torch.Tensor:
    """q (or out) rows [tokens, Hq, D] -> this rank's heads (a view)."""
    lo, hi = q_head_range(q.shape[1], num_kv_heads, rank, world)
    return q[:, lo:hi]


def shard_cache(cache: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Paged cache [num_blocks, block_size, KVH, D] (or rows [T, KVH, D] with dim=-2) -> this
    rank's own contiguous cache."""
    lo, hi = kv_head_range(cache.shape[-2], rank, world)
    return cache[..., lo:hi, :].contiguous()
