"""KV-head sharding across tensor-parallel ranks.

The engine divides heads by the world size at backend creation
(nanovllm/engine/model_runner.py:99-105) and gives every rank a cache of
Hkv / tp heads (model_runner.py:334-346): rank r owns KV heads
[r * Hkv/tp, (r+1) * Hkv/tp) and the q heads that read them. The KV append
and attention then run locally on each rank; no collective touches them.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    q_heads: slice
    kv_heads: slice

    @property
    def num_q_heads(self) -> int:
        return self.q_heads.stop - self.q_heads.start

    @property
    def num_kv_heads(self) -> int:
        return self.kv_heads.stop - self.kv_heads.start


def kv_head_shard(num_q_heads: int, num_kv_heads: int, rank: int, world: int) -> HeadShard:
    """Head ranges owned by `rank` of `world` tensor-parallel ranks."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    if num_kv_heads % world or num_q_heads % world:
        raise ValueError("the world size must divide both head counts")
    kv = num_kv_heads // world
    q = num_q_heads // world
    return HeadShard(rank, world, slice(rank * q, (rank + 1) * q),
                     slice(rank * kv, (rank + 1) * kv))


def shard_tensors(shard: HeadShard, q: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                  k_cache: torch.Tensor, v_cache: torch.Tensor):
    """This rank's views of q [T, Hq, D], new K/V [T, Hkv, D] and the NHD
    caches [N, bs, Hkv, D] (contiguous copies of the cache shard, as the
    engine allocates a separate cache per rank)."""
    return (q[:, shard.q_heads], key[:, shard.kv_heads], value[:, shard.kv_heads],
            k_cache[:, :, shard.kv_heads].contiguous(), v_cache[:, :, shard.kv_heads].contiguous())
