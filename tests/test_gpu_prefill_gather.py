"""GPU parity of the prefill with the head gather fused into the attention
kernel (eb_attention_prefill_gather), on one GPU: the shards of a head-sharded
run (eyebrowse_b200.sharded.head_shard) run one after another, each storing
its finished output tiles into two destination buffers at its head offset,
as it would into two ranks' gathered buffers. Both buffers must hold the
whole [S, H, hd] output, equal to each other bit for bit and to the oracle
at the north-star tolerance on the checked rows.

Covers the one-tile kernel (a shard with few heads: the longest item
decides the grid) and the two-tile GQA-pair kernel, 16-bit q with the q prep
and its RoPE table rows fused into the kernel, a ragged last tile, and the
shard shapes of config 3 on 4 and 8 GPUs at full length."""
import os

import numpy as np
import pytest

from _util import assert_close, randn, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("S,H,Hkv,world,dt", [
    (700, 8, 4, 4, "f16"),     # 2 heads per shard: one-tile kernel
    (4608, 32, 8, 2, "f16"),   # 16 heads per shard: GQA-pair kernel
    (1100, 16, 8, 2, "bf16"),  # 8 heads per shard, bf16
    (8192, 32, 8, 8, "f16"),   # config 3 over 8 GPUs: 4 heads, 1 KV head per shard
    (8192, 32, 8, 4, "f16"),   # config 3 over 4 GPUs: 8 heads, 2 KV heads per shard
])
def test_prefill_gather_assembles_the_full_output(eb, orc, S, H, Hkv, world, dt):
    import torch

    from eyebrowse_b200.sharded import head_shard
    hd = 128
    code = eb.EB_F16 if dt == "f16" else eb.EB_BF16
    tdt = torch.float16 if dt == "f16" else torch.bfloat16
    rnd = orc.round_f16 if dt == "f16" else orc.round_bf16
    seed = S + H
    q = rnd(randn((S, H, hd), seed, 0.5)).reshape(S, H, hd)
    k = rnd(randn((S, Hkv, hd), seed + 1, 0.5)).reshape(S, Hkv, hd)
    v = rnd(randn((S, Hkv, hd), seed + 2, 0.5)).reshape(S, Hkv, hd)
    cos, sin = eb.rope_tables(S, hd, 5e5)
    layer = eb.make_layer(rope_cos=to_dev(cos), rope_sin=to_dev(sin))
    bufs = [torch.full((S, H, hd), float("nan"), device="cuda", dtype=tdt) for _ in range(2)]
    addrs = (eb.ctypes.c_uint64 * 2)(*[b.data_ptr() for b in bufs])
    for rank in range(world):
        sh = head_shard(H, Hkv, world, rank)
        desc = eb.make_desc(sh.n_heads, sh.n_kv_heads, hd, S, dtype_qkv=code, dtype_cache=code,
                            dtype_out=code)
        kc = torch.empty(S, sh.n_kv_heads, hd, device="cuda", dtype=tdt)
        vc = torch.empty_like(kc)
        nb = eb.attention_prefill_workspace_bytes(desc, S)
        ws = eb.alloc_workspace(nb) if nb else None
        g = eb.HeadGather(n_dst=2, head_offset=sh.h0, n_heads_total=H,
                          dst=eb.ctypes.cast(addrs, eb.ctypes.POINTER(eb.ctypes.c_uint64)))
        eb.attention_prefill_gather(desc, layer, S, to_dev(q[:, sh.h0:sh.h1], tdt),
                                    to_dev(k[:, sh.kv0:sh.kv1], tdt),
                                    to_dev(v[:, sh.kv0:sh.kv1], tdt), kc, vc, g, ws)
    torch.cuda.synchronize()
    got = [to_np(b) for b in bufs]
    assert np.array_equal(got[0], got[1])
    # oracle on the last 96 rows of every head (the longest causal rows) and
    # the first 32 (the shortest): q and k rotated in f32, only k rounded (as
    # the 16-bit cache stores it)
    qr = orc.rope(q, cos, sin, S, H, hd).reshape(S, H, hd)
    kr = rnd(orc.rope(k, cos, sin, S, Hkv, hd)).reshape(S, Hkv, hd)
    threads = max(1, min(32, os.cpu_count() or 1))
    tol = dict(max_abs=8e-3, rel_l2=4e-3) if dt == "bf16" else {}
    for r0, r1 in ((S - 96, S), (0, 32)):
        want = orc.attn_prefill_part(qr, kr, v, H, Hkv, S, hd, hd ** -0.5, (r0, r1), (0, H),
                                     nthreads=threads).reshape(S, H, hd)[r0:r1]
        assert_close(orc, got[0][r0:r1], want, what=f"gathered prefill rows [{r0},{r1}) {dt}",
                     **tol)
    assert eb.device_error() == 0
