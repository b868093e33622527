"""Sharded attention across GPUs: one process per GPU, torch.distributed
for the plumbing, and a single exchange at the head-concat boundary.

Attention is independent per KV-head group and per sequence:
  - prefill (head_shard): rank g of G owns KV heads [g*Hkv/G, (g+1)*Hkv/G)
    and their query heads, keeps its own cache slice [max_seq, Hkv/G, hd]
    and runs the fused call on its slice with no traffic to other ranks;
  - batched decode (decode_shard): the ranks form a grid of KV-head groups x
    sequence buckets -- the head split first (as many groups as divide both
    the world and Hkv), the sequences of a decode batch spread over the rest
    and balanced by context length -- so a model with fewer KV heads than
    GPUs still uses every GPU.
The per-rank outputs meet at the head-concat boundary in one of two ways:
  - GatheredOutput: the attention kernel itself stores every finished output
    tile or row into every rank's gathered buffer over NVLink (TMA stores for
    prefill, eb_attention_prefill_gather; plain stores for decode,
    eb_attention_decode_batched_gather) while the rest of the kernel runs.
    No library collective runs; one device barrier per step.
  - gather_heads: NCCL all-gather into [G, rows, H/G, hd], then
    eb_head_concat restores [rows, H, hd] (the library-collective baseline,
    head split only).
GatheredOutput also keeps a multicast mode for prefill (one store through
the NVLink multicast address, eb_head_broadcast): bit-identical, but slower
on this B200 pool at 8 GPUs (its docstring has the figures); "auto" picks
the peer stores.
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


@dataclass(frozen=True)
class DecodeShard:
    """A rank's part of a batched decode: query/KV heads [h0, h1) / [kv0, kv1)
    of the sequences `seqs` (global indices, ascending)."""
    rank: int
    world: int
    head_groups: int
    h0: int
    h1: int
    kv0: int
    kv1: int
    seqs: tuple

    @property
    def n_heads(self) -> int:
        return self.h1 - self.h0

    @property
    def n_kv_heads(self) -> int:
        return self.kv1 - self.kv0


def balance_sequences(ctx, buckets: int):
    """Sequences (indices into ctx) per bucket: longest first, each to the
    least-loaded bucket (ties to the lowest index), so the K/V rows each
    bucket reads are balanced. Deterministic: every rank computes the same."""
    import heapq
    order = sorted(range(len(ctx)), key=lambda i: (-int(ctx[i]), i))
    heap = [(0, b) for b in range(buckets)]
    out = [[] for _ in range(buckets)]
    for i in order:
        load, b = heapq.heappop(heap)
        out[b].append(i)
        heapq.heappush(heap, (load + int(ctx[i]), b))
    return [tuple(sorted(x)) for x in out]


def decode_shard(n_heads: int, n_kv_heads: int, world: int, rank: int, ctx,
                 head_groups: int | None = None) -> DecodeShard:
    """Rank `rank`'s part of a batched decode over sequences with context
    lengths `ctx`: head group rank % G_h (G_h = head_groups, by default the
    largest count dividing both world and n_kv_heads) of the sequences in
    bucket rank // G_h of the world / G_h context-balanced buckets."""
    import math
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    gh = head_groups or math.gcd(world, n_kv_heads)
    if world % gh or n_kv_heads % gh:
        raise ValueError(f"{gh} head groups for {world} ranks and {n_kv_heads} KV heads")
    hs = head_shard(n_heads, n_kv_heads, gh, rank % gh)
    buckets = balance_sequences(ctx, world // gh)
    return DecodeShard(rank, world, gh, hs.h0, hs.h1, hs.kv0, hs.kv1, buckets[rank // gh])


def gather_heads(o_local, gath, full, world: int, rows: int, heads_per: int, head_dim: int,
                 dtype_code: int, group=None):
    """All-gather per-rank outputs [rows, heads_per, hd] over NCCL into `gath`
    [world, rows, heads_per, hd], then concatenate heads on the device into
    `full` [rows, world*heads_per, hd] with eb_head_concat."""
    import torch.distributed as dist

    import eyebrowse_b200 as eb
    dist.all_gather_into_tensor(gath, o_local, group=group)
    eb.head_concat(gath, full, world, rows, heads_per, head_dim, dtype_code)


class GatheredOutput:
    """The gathered [rows, n_heads, head_dim] output of a head-sharded prefill,
    double-buffered in torch symmetric memory (every rank's buffers mapped
    into every process; torch allocates, maps and provides the device
    barrier, the stores are this library's). Two ways to fill it:

      mode "peer":      the attention kernel TMA-stores each finished output
                        tile into all ranks' buffers over NVLink, overlapped
                        with the rest of the kernel (each word leaves the GPU
                        world - 1 times);
      mode "multicast": the attention kernel writes this rank's heads into
                        its own buffer, then eb_head_broadcast sends them once
                        through the buffers' NVLink multicast address and the
                        switch writes every rank's copy (each word leaves once);
      mode "auto":      peer. Measured on B200 (config 3, S=8192): at 2 GPUs
                        peer stores add ~5 us to the kernel; at 8 GPUs the
                        peer step takes 0.167-0.177 ms and the multicast step
                        0.201 ms. A streaming multimem.st kernel reaches ~330
                        GB/s per sender with 2 GPUs in the multicast group but
                        ~80 GB/s with 8, so the single copy does not win.

    Step i writes buffer i % 2:

        gather = g.next()                  # eb_head_gather for this step
        eyebrowse_b200.attention_prefill_gather(..., gather, ...)
        g.finish()                         # broadcast (multicast mode), barrier
        use(g.full)                        # this step's gathered output

    One barrier per step is enough: a rank writes a buffer again only two
    steps later, after every rank has passed the barrier of the step in
    between, and so after every rank has finished reading it (reads are
    stream-ordered before that next step's call)."""

    def __init__(self, rows: int, n_heads: int, head_dim: int, dtype, shard: HeadShard,
                 group=None, mode: str = "auto"):
        import ctypes

        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        from torch._C._distributed_c10d import _SymmetricMemory

        import eyebrowse_b200 as eb
        grp = group or dist.group.WORLD
        self.eb, self.shard, self.rows, self.n_heads, self.hd = eb, shard, rows, n_heads, head_dim
        self.dtype_code = {torch.float32: eb.EB_F32, torch.float16: eb.EB_F16,
                           torch.bfloat16: eb.EB_BF16}[dtype]
        self.bufs = symm_mem.empty(2, rows, n_heads, head_dim, dtype=dtype, device="cuda")
        self.handle = symm_mem.rendezvous(self.bufs, grp.group_name)
        world, rank = self.handle.world_size, self.handle.rank
        base = self.bufs.data_ptr() - self.handle.buffer_ptrs[rank]
        self.stride = self.bufs[1].data_ptr() - self.bufs[0].data_ptr()
        has_mc = bool(_SymmetricMemory.has_multicast_support(
            torch._C._autograd.DeviceType.CUDA, torch.cuda.current_device())
            and self.handle.multicast_ptr)
        if mode == "auto":
            mode = "peer"
        if mode == "multicast" and not has_mc:
            raise RuntimeError("NVLink multicast is not supported on these GPUs")
        self.mode = mode
        self.mc = self.handle.multicast_ptr + base if mode == "multicast" else 0
        if mode == "multicast":
            addrs = [[self.bufs[i].data_ptr()] for i in range(2)]
        else:
            addrs = [[p + base + i * self.stride for p in self.handle.buffer_ptrs]
                     for i in range(2)]
        self._dst = [(ctypes.c_uint64 * len(a))(*a) for a in addrs]
        self.gathers = [eb.HeadGather(n_dst=len(a), head_offset=shard.h0, n_heads_total=n_heads,
                                      dst=ctypes.cast(d, ctypes.POINTER(ctypes.c_uint64)))
                        for a, d in zip(addrs, self._dst)]
        self.step = -1

    def next(self):
        """The eb_head_gather of the next step (alternating buffers)."""
        self.step += 1
        return self.gathers[self.step % 2]

    @property
    def full(self):
        """The gathered output of the current step."""
        return self.bufs[max(self.step, 0) % 2]

    def finish(self):
        """After this rank's attention call: in multicast mode, send this
        rank's heads to every rank; then the cross-GPU barrier."""
        if self.mode == "multicast":
            i = max(self.step, 0) % 2
            self.eb.head_broadcast(self.bufs[i], self.mc + i * self.stride, self.rows,
                                   self.n_heads, self.shard.h0, self.shard.n_heads, self.hd,
                                   self.dtype_code)
        self.barrier()

    def barrier(self):
        """Device-side barrier across the group's GPUs on the current stream."""
        self.handle.barrier(channel=0)


def concat_heads_host(shards):
    """Host-side equivalent of eb_head_concat for CPU tests: a list of G numpy
    arrays [rows, heads_per, hd] -> [rows, G*heads_per, hd]."""
    import numpy as np
    return np.concatenate(shards, axis=1)
