"""The head-sharded multi-GPU path's host logic, run as two gloo ranks on CPU:
each rank computes its KV-head group's attention with the oracle, the ranks
all-gather their outputs, and the concatenated heads must equal the
unsharded attention exactly (attention is independent per head, so the
per-head arithmetic is identical)."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_head_shard_bounds():
    from eyebrowse_b200.sharded import head_shard
    shards = [head_shard(32, 8, 4, r) for r in range(4)]
    assert [(s.h0, s.h1, s.kv0, s.kv1) for s in shards] == [
        (0, 8, 0, 2), (8, 16, 2, 4), (16, 24, 4, 6), (24, 32, 6, 8)]
    # every query head's KV head lies in its rank's KV range (h // group)
    for s in shards:
        assert all(s.kv0 <= h // 4 < s.kv1 for h in range(s.h0, s.h1))
    with pytest.raises(ValueError):
        head_shard(32, 8, 3, 0)
    with pytest.raises(ValueError):
        head_shard(30, 8, 2, 0)


def _rank_main(rank, world, port, out_path):
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    from eyebrowse_b200.sharded import concat_heads_host, head_shard
    from oracle import oracle as orc
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    S, H, Hkv, hd = 24, 8, 4, 16
    rng = np.random.default_rng(0)  # same full inputs on every rank
    q = rng.standard_normal((S, H, hd)).astype(np.float32)
    k = rng.standard_normal((S, Hkv, hd)).astype(np.float32)
    v = rng.standard_normal((S, Hkv, hd)).astype(np.float32)
    sh = head_shard(H, Hkv, world, rank)
    ql = np.ascontiguousarray(q[:, sh.h0:sh.h1])
    kl = np.ascontiguousarray(k[:, sh.kv0:sh.kv1])
    vl = np.ascontiguousarray(v[:, sh.kv0:sh.kv1])
    ol = orc.attn_prefill(ql, kl, vl, sh.n_heads, sh.n_kv_heads, S, hd, 0.25).reshape(
        S, sh.n_heads, hd)
    parts = [torch.empty(S, sh.n_heads, hd) for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(ol))
    full = concat_heads_host([p.numpy() for p in parts])
    if rank == 0:
        want = orc.attn_prefill(q, k, v, H, Hkv, S, hd, 0.25).reshape(S, H, hd)
        np.save(out_path, np.stack([full, want]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_head_sharding_gloo(tmp_path):
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = str(tmp_path / "res.npy")
    mp.start_processes(_rank_main, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
    full, want = np.load(out)
    assert np.array_equal(full, want)


def test_decode_shard_covers_every_row_once():
    """Every (sequence, query head) of a batched decode belongs to exactly one
    rank, for head-only, mixed and batch-only splits; sequence buckets are
    balanced by context length."""
    from eyebrowse_b200.sharded import decode_shard
    ctx = np.random.default_rng(5).integers(512, 32769, size=64)
    for H, Hkv, world, gh in ((32, 8, 8, None), (8, 4, 8, None), (32, 8, 4, 1), (16, 2, 4, None)):
        seen = np.zeros((64, H), np.int32)
        loads = {}
        for r in range(world):
            s = decode_shard(H, Hkv, world, r, ctx, head_groups=gh)
            seen[np.ix_(list(s.seqs), range(s.h0, s.h1))] += 1
            assert all(s.kv0 <= h // (H // Hkv) < s.kv1 for h in range(s.h0, s.h1))
            loads.setdefault(r // s.head_groups, int(ctx[list(s.seqs)].sum()))
        assert (seen == 1).all(), (H, Hkv, world, gh)
        assert max(loads.values()) <= 1.01 * min(loads.values())
    with pytest.raises(ValueError):
        decode_shard(32, 8, 8, 0, ctx, head_groups=3)


def _decode_rank_main(rank, world, port, out_path):
    """One gloo rank of a 2 x 2 decode shard: its (sequences, heads) through
    the oracle, all-gathered and placed by global sequence and head."""
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    from eyebrowse_b200.sharded import decode_shard
    from oracle import oracle as orc
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    B, H, Hkv, hd, ms = 6, 8, 4, 16, 40
    rng = np.random.default_rng(1)
    pos = rng.integers(3, ms, size=B).astype(np.int32)
    kc = rng.standard_normal((B, ms, Hkv, hd)).astype(np.float32)
    vc = rng.standard_normal((B, ms, Hkv, hd)).astype(np.float32)
    q = rng.standard_normal((B, H, hd)).astype(np.float32)
    s = decode_shard(H, Hkv, world, rank, pos + 1, head_groups=2)
    seqs = list(s.seqs)
    lo = orc.attn_decode_batched(np.ascontiguousarray(q[seqs][:, s.h0:s.h1]),
                                 np.ascontiguousarray(kc[seqs][:, :, s.kv0:s.kv1]),
                                 np.ascontiguousarray(vc[seqs][:, :, s.kv0:s.kv1]), pos[seqs],
                                 s.n_heads, s.n_kv_heads, hd, ms, ms * s.n_kv_heads * hd, 0.25)
    parts = [None] * world
    dist.all_gather_object(parts, (seqs, s.h0, s.h1, lo.reshape(len(seqs), s.n_heads, hd)))
    if rank == 0:
        full = np.full((B, H, hd), np.nan, np.float32)
        for sq, h0, h1, o in parts:
            full[np.ix_(sq, range(h0, h1))] = o
        want = orc.attn_decode_batched(q, kc, vc, pos, H, Hkv, hd, ms, ms * Hkv * hd,
                                       0.25).reshape(B, H, hd)
        np.save(out_path, np.stack([full, want]))
    dist.barrier()
    dist.destroy_process_group()


def test_four_rank_decode_sharding_gloo(tmp_path):
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = str(tmp_path / "dec.npy")
    mp.start_processes(_decode_rank_main, args=(4, port, out), nprocs=4, join=True,
                       start_method="spawn")
    full, want = np.load(out)
    assert np.array_equal(full, want)
