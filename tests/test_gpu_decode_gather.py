"""GPU parity of the batched decode with the head gather fused into the
kernel (eb_attention_decode_batched_gather), on one GPU: the shards of a
4-rank decode (2 KV-head groups x 2 context-balanced sequence buckets,
eyebrowse_b200.sharded.decode_shard) run one after another, each storing
its rows into two destination buffers (as it would into two ranks' gathered
buffers) at the sequences' global rows and its head offset. Both buffers
must hold the whole [B, H, hd] output: equal to each other, to the oracle
at the north-star tolerance, and to the unsharded call. Covers the
tensor-core kernel (f16), the vector kernel (bf16) and the cluster-combined
kernel (f32, few sequences)."""
import numpy as np
import pytest

from _util import assert_close, randn, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cache,B", [("f16", 10), ("bf16", 10), ("f32", 3)])
def test_decode_gather_assembles_the_full_output(eb, orc, cache, B):
    import torch

    from eyebrowse_b200.sharded import decode_shard
    H, Hkv, hd, max_seq, world = 16, 8, 128, 2048, 4
    code = {"f16": eb.EB_F16, "bf16": eb.EB_BF16, "f32": eb.EB_F32}[cache]
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[cache]
    rnd = {"f16": orc.round_f16, "bf16": orc.round_bf16, "f32": lambda x: x}[cache]
    rng = np.random.default_rng(11 + B)
    pos = rng.integers(100, max_seq, size=B).astype(np.int32)
    kc = rnd(randn((B, max_seq, Hkv, hd), 900)).reshape(B, max_seq, Hkv, hd)
    vc = rnd(randn((B, max_seq, Hkv, hd), 901)).reshape(B, max_seq, Hkv, hd)
    q = rnd(randn((B, H, hd), 902)).reshape(B, H, hd)
    k = rnd(randn((B, Hkv, hd), 903)).reshape(B, Hkv, hd)
    v = rnd(randn((B, Hkv, hd), 904)).reshape(B, Hkv, hd)
    cos, sin = eb.rope_tables(max_seq, hd, 1e6)
    layer = eb.make_layer(rope_cos=to_dev(cos), rope_sin=to_dev(sin))
    bufs = [torch.full((B, H, hd), float("nan"), device="cuda", dtype=tdt) for _ in range(2)]
    addrs = (eb.ctypes.c_uint64 * 2)(*[b.data_ptr() for b in bufs])
    for rank in range(world):
        sh = decode_shard(H, Hkv, world, rank, pos + 1, head_groups=2)
        seqs = list(sh.seqs)
        nb = len(seqs)
        desc = eb.make_desc(sh.n_heads, sh.n_kv_heads, hd, max_seq, dtype_qkv=code,
                            dtype_cache=code, dtype_out=code)
        lk = to_dev(np.ascontiguousarray(kc[seqs][:, :, sh.kv0:sh.kv1]), tdt)
        lv = to_dev(np.ascontiguousarray(vc[seqs][:, :, sh.kv0:sh.kv1]), tdt)
        lq = to_dev(np.ascontiguousarray(q[seqs][:, sh.h0:sh.h1]), tdt)
        lkn = to_dev(np.ascontiguousarray(k[seqs][:, sh.kv0:sh.kv1]), tdt)
        lvn = to_dev(np.ascontiguousarray(v[seqs][:, sh.kv0:sh.kv1]), tdt)
        lpos = to_dev(pos[seqs])
        mp = int(pos[seqs].max())
        nbytes = eb.attention_decode_workspace_bytes(desc, nb, mp)
        ws = eb.alloc_workspace(nbytes) if nbytes else None
        g = eb.HeadGather(n_dst=2, head_offset=sh.h0, n_heads_total=H,
                          dst=eb.ctypes.cast(addrs, eb.ctypes.POINTER(eb.ctypes.c_uint64)))
        eb.attention_decode_batched_gather(desc, layer, nb, lpos, mp, lq, lkn, lvn, lk, lv,
                                           max_seq * sh.n_kv_heads * hd, g,
                                           to_dev(np.array(seqs, np.int32)), ws)
    torch.cuda.synchronize()
    got = [to_np(b) for b in bufs]
    assert np.array_equal(got[0], got[1])
    # oracle: the new rows (RoPE'd k, v) stored in each cache, then decode
    for b in range(B):
        kc[b, pos[b]] = rnd(orc.rope(k[b], cos, sin, 1, Hkv, hd, int(pos[b]))).reshape(Hkv, hd)
        vc[b, pos[b]] = v[b]
    qr = np.stack([orc.rope(q[b], cos, sin, 1, H, hd, int(pos[b])) for b in range(B)])
    want = orc.attn_decode_batched(qr, kc, vc, pos, H, Hkv, hd, max_seq, max_seq * Hkv * hd,
                                   hd ** -0.5, nthreads=8)
    tol = dict(max_abs=8e-3, rel_l2=4e-3) if cache == "bf16" else {}
    assert_close(orc, got[0], want, what=f"gathered decode {cache} vs oracle", **tol)
    assert eb.device_error() == 0


def test_decode_gather_rejects_bad_destinations(eb):
    import torch
    desc = eb.make_desc(16, 8, 128, 256, dtype_qkv=eb.EB_F16, dtype_cache=eb.EB_F16,
                        dtype_out=eb.EB_F16)
    layer = eb.make_layer()
    x = torch.zeros(1 << 20, device="cuda", dtype=torch.float16)
    pos = torch.zeros(1, device="cuda", dtype=torch.int32)
    bad = [(0, 0, 16, [x.data_ptr()]),            # no destination
           (1, 4, 16, [x.data_ptr()]),            # heads 4..19 past 16 heads
           (1, 0, 16, [x.data_ptr() + 2]),        # destination not 16-byte aligned
           (9, 0, 16, [x.data_ptr()] * 9)]        # more than 8 destinations
    for n, off, tot, ptrs in bad:
        arr = (eb.ctypes.c_uint64 * len(ptrs))(*ptrs)
        g = eb.HeadGather(n_dst=n, head_offset=off, n_heads_total=tot,
                          dst=eb.ctypes.cast(arr, eb.ctypes.POINTER(eb.ctypes.c_uint64)))
        with pytest.raises(eb.EbError) as e:
            eb.attention_decode_batched_gather(desc, layer, 1, pos, 0, x, x, x, x, x,
                                               256 * 8 * 128, g)
        assert e.value.status == 1
