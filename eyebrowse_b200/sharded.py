"""Head-sharded attention across GPUs: one process per GPU, torch.distributed
(NCCL) for the single exchange at the head-concat boundary.

Attention is independent per KV-head group, so rank g of G owns KV heads
[g*Hkv/G, (g+1)*Hkv/G) and their query heads, keeps its own cache slice
[max_seq, Hkv/G, hd] and runs the fused call on its slice with no traffic to
other ranks. The per-rank outputs [rows, H/G, hd] are all-gathered into
[G, rows, H/G, hd] and eb_head_concat restores [rows, H, hd].
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    h0: int   # first query head of this rank
    h1: int   # one past the last query head
    kv0: int  # first KV head
    kv1: int

    @property
    def n_heads(self) -> int:
        return self.h1 - self.h0

    @property
    def n_kv_heads(self) -> int:
        return self.kv1 - self.kv0


def head_shard(n_heads: int, n_kv_heads: int, world: int, rank: int) -> HeadShard:
    """The query/KV head range rank `rank` of `world` owns. KV heads split
    evenly and each rank takes the query heads that read its KV heads
    (query head h reads KV head h // (n_heads // n_kv_heads))."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if n_heads % n_kv_heads:
        raise ValueError(f"n_heads {n_heads} not a multiple of n_kv_heads {n_kv_heads}")
    if n_kv_heads % world:
        raise ValueError(f"{world} ranks do not divide {n_kv_heads} KV heads")
    kv_per = n_kv_heads // world
    group = n_heads // n_kv_heads
    kv0 = rank * kv_per
    return HeadShard(rank, world, kv0 * group, (kv0 + kv_per) * group, kv0, kv0 + kv_per)


def gather_heads(o_local, gath, full, world: int, rows: int, heads_per: int, head_dim: int,
                 dtype_code: int, group=None):
    """All-gather per-rank outputs [rows, heads_per, hd] over NCCL into `gath`
    [world, rows, heads_per, hd], then concatenate heads on the device into
    `full` [rows, world*heads_per, hd] with eb_head_concat."""
    import torch.distributed as dist

    import eyebrowse_b200 as eb
    dist.all_gather_into_tensor(gath, o_local, group=group)
    eb.head_concat(gath, full, world, rows, heads_per, head_dim, dtype_code)


def concat_heads_host(shards):
    """Host-side equivalent of eb_head_concat for CPU tests: a list of G numpy
    arrays [rows, heads_per, hd] -> [rows, G*heads_per, hd]."""
    import numpy as np
    return np.concatenate(shards, axis=1)
