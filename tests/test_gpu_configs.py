"""GPU parity of the fused attention primitive on the BASELINE.json configs.

Each test builds the config's seeded synthetic inputs, runs the C-ABI call
and the oracle (the reference's CPU attention, restated) on the same inputs,
and checks max-abs <= 2e-3 and rel-L2 <= 1e-3 against it. Configs whose
full oracle run would take minutes are checked on a stated subset of rows
(the oracle's row/head-restricted form computes exactly those outputs).
"""
import os

import numpy as np
import pytest

from _util import assert_close, randn, to_dev, to_np

pytestmark = pytest.mark.gpu


def _tables(eb, max_seq, hd, theta, rope_angles=None):
    cos, sin = eb.rope_tables(max_seq, hd, theta, rope_angles)
    return cos, sin


def test_config1_prefill_qwen3_geometry(eb, orc):
    """cfg1: S128 H16 Hkv8 hd128, f32 N(0,1), scale 1/sqrt(128), RoPE 1e6, no norm."""
    import torch
    S, H, Hkv, hd, max_seq = 128, 16, 8, 128, 4096
    q, k, v = randn((S, H, hd), 100), randn((S, Hkv, hd), 101), randn((S, Hkv, hd), 102)
    cos, sin = _tables(eb, max_seq, hd, 1e6)
    desc = eb.make_desc(H, Hkv, hd, max_seq, scale=1 / np.sqrt(128))
    cd, sd = to_dev(cos), to_dev(sin)
    layer = eb.make_layer(rope_cos=cd, rope_sin=sd)
    kc = torch.zeros(max_seq * Hkv * hd, device="cuda")
    vc = torch.zeros_like(kc)
    o = torch.empty(S * H * hd, device="cuda")
    ws = eb.alloc_workspace(eb.attention_prefill_workspace_bytes(desc, S))
    eb.attention_prefill(desc, layer, S, to_dev(q), to_dev(k), to_dev(v), kc, vc, o, ws)
    want, wkc, wvc = orc.attention_prefill(q, k, v, seq=S, h=H, hkv=Hkv, hd=hd, max_seq=max_seq,
                                           scale=1 / np.sqrt(128), cos=cos, sin=sin)
    assert_close(orc, to_np(o), want, what="cfg1 o")
    # cache rows: same f32 ops as the oracle -> exact
    assert np.array_equal(to_np(kc), wkc) and np.array_equal(to_np(vc), wvc)


def test_config2_decode_qwen3_geometry(eb, orc):
    """cfg2: cache [4096,8,128] f32, rows 0..2046 N(0,1); new token at 2047 with
    QK-RMSNorm (unit weights, eps 1e-6), RoPE 1e6, fused cache write."""
    import torch
    H, Hkv, hd, max_seq, pos = 16, 8, 128, 4096, 2047
    kc = randn((max_seq, Hkv, hd), 200)
    vc = randn((max_seq, Hkv, hd), 201)
    kc[pos:] = np.nan  # row pos is written by the call; rows past it are never read
    vc[pos:] = np.nan
    q, k, v = randn((H, hd), 202), randn((Hkv, hd), 203), randn((Hkv, hd), 204)
    ones = np.ones(hd, np.float32)
    cos, sin = _tables(eb, max_seq, hd, 1e6)
    desc = eb.make_desc(H, Hkv, hd, max_seq, eps=1e-6)
    layer = eb.make_layer(q_norm_w=to_dev(ones), k_norm_w=to_dev(ones), rope_cos=to_dev(cos),
                          rope_sin=to_dev(sin))
    want, wkc, wvc = orc.attention_decode(q, k, v, pos=pos, h=H, hkv=Hkv, hd=hd, max_seq=max_seq,
                                          scale=1 / np.sqrt(hd), kcache=kc, vcache=vc, eps=1e-6,
                                          q_norm_w=ones, k_norm_w=ones, cos=cos, sin=sin)
    ws = eb.alloc_workspace(eb.attention_decode_workspace_bytes(desc, 1, pos))
    for _ in range(2):
        kcd, vcd = to_dev(kc), to_dev(vc)
        o = torch.empty(H * hd, device="cuda")
        eb.attention_decode(desc, layer, pos, to_dev(q), to_dev(k), to_dev(v), kcd, vcd, o, ws)
        assert_close(orc, to_np(o), want, what="cfg2 o")
        row = slice(pos * Hkv * hd, (pos + 1) * Hkv * hd)
        assert_close(orc, to_np(kcd)[row], wkc[row], max_abs=1e-5, rel_l2=1e-6, what="cfg2 k row")
        assert np.array_equal(to_np(vcd)[row], wvc[row])


@pytest.mark.parametrize("S", [1024, 8192])
def test_config3_prefill_llama3_f16(eb, orc, S):
    """cfg3: S8192 H32 Hkv8 hd128, Q/K/V = 0.5*N(0,1) in f16, RoPE 5e5, f16 cache,
    f32 accumulate. The oracle gets the f16 inputs with RoPE applied in f32;
    only the K rows are rounded to f16 after RoPE, because the cache stores
    them so (the kernel's own rounding of q to its f16 MMA operand is part of
    the measured error). S=1024 is checked in full. S=8192 (the benchmarked
    shape) is checked on every 8th 128-row query tile -- tiles 0, 8, ..., 56,
    which the kernel schedules early, in the middle and late -- in full, for
    all 32 heads (both heads of every GQA pair), plus the last tile."""
    import torch
    H, Hkv, hd = 32, 8, 128
    max_seq = S
    q = orc.round_f16(randn((S, H, hd), 300, 0.5))
    k = orc.round_f16(randn((S, Hkv, hd), 301, 0.5))
    v = orc.round_f16(randn((S, Hkv, hd), 302, 0.5))
    cos, sin = _tables(eb, max_seq, hd, 5e5)
    desc = eb.make_desc(H, Hkv, hd, max_seq, dtype_qkv=eb.EB_F16, dtype_cache=eb.EB_F16,
                        dtype_out=eb.EB_F16)
    layer = eb.make_layer(rope_cos=to_dev(cos), rope_sin=to_dev(sin))
    kc = torch.zeros(max_seq * Hkv * hd, device="cuda", dtype=torch.float16)
    vc = torch.zeros_like(kc)
    o = torch.empty(S * H * hd, device="cuda", dtype=torch.float16)
    ws = eb.alloc_workspace(eb.attention_prefill_workspace_bytes(desc, S))
    eb.attention_prefill(desc, layer, S, to_dev(q, torch.float16), to_dev(k, torch.float16),
                         to_dev(v, torch.float16), kc, vc, o, ws)
    qr = orc.rope(q, cos, sin, S, H, hd)                   # f32 RoPE, not rounded
    kr = orc.round_f16(orc.rope(k, cos, sin, S, Hkv, hd))  # as the f16 cache stores it
    assert np.array_equal(to_np(kc), kr)           # the cache write is exact
    assert np.array_equal(to_np(vc), v.ravel())
    got = to_np(o).reshape(S, H, hd)
    scale = 1 / np.sqrt(hd)
    if S <= 1024:
        want = orc.attn_prefill(qr, kr, v, H, Hkv, S, hd, scale).reshape(S, H, hd)
        assert_close(orc, got, want, what="cfg3 S1024")
        return
    n_qt = S // 128
    tiles = sorted(set(range(0, n_qt, 8)) | {n_qt - 1})
    threads = max(1, min(32, os.cpu_count() or 1))
    for t in tiles:
        rows = (128 * t, 128 * (t + 1))
        part = orc.attn_prefill_part(qr, kr, v, H, Hkv, S, hd, scale, rows, (0, H),
                                     nthreads=threads).reshape(S, H, hd)
        assert_close(orc, got[rows[0]:rows[1]], part[rows[0]:rows[1]],
                     what=f"cfg3 S8192 query tile {t}")


def test_config4_gemma_prefill_then_decode(eb, orc):
    """cfg4 as specified: prefill S4096, then 256 decode steps; H8 Hkv4 hd256,
    scale 1.0, QK-norm weights N(1,0.1), weightless V-norm, partial rotary 32
    of 128 pairs (1e6), f32. The prefill is checked on every 8th 128-row
    query tile plus the last, all heads; all 256 decode steps run on the
    cache the prefill wrote, and every 16th step and the last are compared
    (the cache rows of the others are checked as they accumulate)."""
    import torch
    S, H, Hkv, hd, steps = 4096, 8, 4, 256, 256
    max_seq = S + steps
    q, k, v = randn((S, H, hd), 400), randn((S, Hkv, hd), 401), randn((S, Hkv, hd), 402)
    qw = (1 + 0.1 * randn((hd,), 403)).astype(np.float32)
    kw = (1 + 0.1 * randn((hd,), 404)).astype(np.float32)
    vw = np.ones(hd, np.float32)
    cos, sin = _tables(eb, max_seq, hd, 1e6, rope_angles=32)
    desc = eb.make_desc(H, Hkv, hd, max_seq, scale=1.0, eps=1e-6)
    layer = eb.make_layer(q_norm_w=to_dev(qw), k_norm_w=to_dev(kw), v_norm_w=to_dev(vw),
                          rope_cos=to_dev(cos), rope_sin=to_dev(sin))
    kcd = torch.zeros(max_seq * Hkv * hd, device="cuda")
    vcd = torch.zeros_like(kcd)
    o = torch.empty(S * H * hd, device="cuda")
    ws = eb.alloc_workspace(eb.attention_prefill_workspace_bytes(desc, S))
    eb.attention_prefill(desc, layer, S, to_dev(q), to_dev(k), to_dev(v), kcd, vcd, o, ws)
    # oracle: transform q/k/v as Attention::prefill does, then whole query tiles
    qn = orc.rope(orc.rmsnorm(q, qw, S * H, hd, 1e-6), cos, sin, S, H, hd)
    kn = orc.rope(orc.rmsnorm(k, kw, S * Hkv, hd, 1e-6), cos, sin, S, Hkv, hd)
    vn = orc.rmsnorm(v, vw, S * Hkv, hd, 1e-6)
    got = to_np(o).reshape(S, H, hd)
    threads = max(1, min(32, os.cpu_count() or 1))
    n_qt = S // 128
    for t in sorted(set(range(0, n_qt, 8)) | {n_qt - 1}):
        rows = (128 * t, 128 * (t + 1))
        part = orc.attn_prefill_part(qn, kn, vn, H, Hkv, S, hd, 1.0, rows, (0, H),
                                     nthreads=threads).reshape(S, H, hd)
        assert_close(orc, got[rows[0]:rows[1]], part[rows[0]:rows[1]],
                     what=f"cfg4 prefill query tile {t}")
    kc = np.zeros((max_seq, Hkv, hd), np.float32)
    vc = np.zeros_like(kc)
    kc[:S] = kn.reshape(S, Hkv, hd)
    vc[:S] = vn.reshape(S, Hkv, hd)
    assert_close(orc, to_np(kcd)[: S * Hkv * hd], kc[:S], max_abs=1e-5, rel_l2=1e-6,
                 what="cfg4 k cache")
    dws = eb.alloc_workspace(eb.attention_decode_workspace_bytes(desc, 1, max_seq - 1))
    od = torch.empty(H * hd, device="cuda")
    checked = 0
    for i in range(steps):
        pos = S + i
        qs, ks, vs = randn((H, hd), 500 + i), randn((Hkv, hd), 600 + i), randn((Hkv, hd), 700 + i)
        eb.attention_decode(desc, layer, pos, to_dev(qs), to_dev(ks), to_dev(vs), kcd, vcd, od, dws)
        if i % 16 == 0 or i == steps - 1:
            want, kcf, vcf = orc.attention_decode(qs, ks, vs, pos=pos, h=H, hkv=Hkv, hd=hd,
                                                  max_seq=max_seq, scale=1.0, kcache=kc.ravel(),
                                                  vcache=vc.ravel(), eps=1e-6, q_norm_w=qw,
                                                  k_norm_w=kw, v_norm_w=vw, cos=cos, sin=sin)
            kc, vc = kcf.reshape(kc.shape), vcf.reshape(vc.shape)
            assert_close(orc, to_np(od), want, what=f"cfg4 decode step {i} pos={pos}")
            checked += 1
        else:
            # the new row as Attention::decode writes it (norm, RoPE at pos)
            kc[pos] = orc.rope(orc.rmsnorm(ks, kw, Hkv, hd, 1e-6), cos, sin, 1, Hkv, hd,
                               pos).reshape(Hkv, hd)
            vc[pos] = orc.rmsnorm(vs, vw, Hkv, hd, 1e-6).reshape(Hkv, hd)
    assert checked == 17
    assert_close(orc, to_np(kcd), kc.ravel(), max_abs=1e-5, rel_l2=1e-6,
                 what="cfg4 cache after 256 decode steps")
    assert_close(orc, to_np(vcd), vc.ravel(), max_abs=1e-5, rel_l2=1e-6,
                 what="cfg4 v cache after 256 decode steps")


def test_config5_batched_decode_f16(eb, orc):
    """cfg5 geometry (H32 Hkv8 hd128, f16 caches, one new token per sequence)
    on 12 sequences with contexts U[512, 8192); every output checked."""
    import torch
    B, H, Hkv, hd, max_seq = 12, 32, 8, 128, 8192
    rng = np.random.default_rng(500)
    pos = rng.integers(512, 8192, size=B).astype(np.int32) - 1
    kc = orc.round_f16(randn((B, max_seq, Hkv, hd), 501)).reshape(B, max_seq, Hkv, hd)
    vc = orc.round_f16(randn((B, max_seq, Hkv, hd), 502)).reshape(B, max_seq, Hkv, hd)
    q = orc.round_f16(randn((B, H, hd), 503))
    k = orc.round_f16(randn((B, Hkv, hd), 504))
    v = orc.round_f16(randn((B, Hkv, hd), 505))
    cos, sin = _tables(eb, max_seq, hd, 5e5)
    desc = eb.make_desc(H, Hkv, hd, max_seq, dtype_qkv=eb.EB_F16, dtype_cache=eb.EB_F16,
                        dtype_out=eb.EB_F32)
    layer = eb.make_layer(rope_cos=to_dev(cos), rope_sin=to_dev(sin))
    kcd, vcd = to_dev(kc, torch.float16), to_dev(vc, torch.float16)
    o = torch.empty(B * H * hd, device="cuda")
    max_pos = int(pos.max())
    ws = eb.alloc_workspace(eb.attention_decode_workspace_bytes(desc, B, max_pos))
    eb.attention_decode_batched(desc, layer, B, to_dev(pos), max_pos, to_dev(q, torch.float16),
                                to_dev(k, torch.float16), to_dev(v, torch.float16), kcd, vcd,
                                max_seq * Hkv * hd, o, ws)
    # oracle: new rows (RoPE'd k, v) rounded to f16 into each cache, then decode
    for b in range(B):
        kr = orc.round_f16(orc.rope(k[b], cos, sin, 1, Hkv, hd, int(pos[b])))
        kc[b, pos[b]] = kr.reshape(Hkv, hd)
        vc[b, pos[b]] = v[b]
    qr = np.stack([orc.rope(q[b], cos, sin, 1, H, hd, int(pos[b])) for b in range(B)])
    want = orc.attn_decode_batched(qr, kc, vc, pos, H, Hkv, hd, max_seq, max_seq * Hkv * hd,
                                   1 / np.sqrt(hd), nthreads=8)
    assert_close(orc, to_np(o), want, what="cfg5")
    got_k = to_np(kcd).reshape(B, max_seq, Hkv, hd)
    for b in range(B):
        assert np.array_equal(got_k[b, pos[b]], kc[b, pos[b]])


def test_config5_bench_geometry(eb, orc):
    """cfg5 exactly as bench.py runs it: 64 sequences with bench.py's context
    draw (U[512, 32768], seed 5), H32 Hkv8 hd128, f16 caches of max_seq 32768,
    f16 q/k/v/o, RoPE 5e5. The caches are filled on the device; the 4 longest
    and the 4 shortest sequences (the most and the fewest split-K partials)
    are compared in full against the oracle, with their new cache rows."""
    import torch

    from bench import BatchedDecodeWork
    w = BatchedDecodeWork()
    B, H, Hkv, hd, max_seq = w.B, w.H, w.Hkv, w.hd, w.max_seq
    pos = w.pos.astype(np.int32)
    g = torch.Generator(device="cuda").manual_seed(55)
    kcd = torch.randn(B, max_seq, Hkv, hd, device="cuda", generator=g).half()
    vcd = torch.randn(B, max_seq, Hkv, hd, device="cuda", generator=g).half()
    q = orc.round_f16(randn((B, H, hd), 510))
    k = orc.round_f16(randn((B, Hkv, hd), 511))
    v = orc.round_f16(randn((B, Hkv, hd), 512))
    cos, sin = _tables(eb, max_seq, hd, w.theta)
    desc = eb.make_desc(H, Hkv, hd, max_seq, dtype_qkv=eb.EB_F16, dtype_cache=eb.EB_F16,
                        dtype_out=eb.EB_F16)
    layer = eb.make_layer(rope_cos=to_dev(cos), rope_sin=to_dev(sin))
    o = torch.full((B, H, hd), float("nan"), device="cuda", dtype=torch.float16)
    max_pos = int(pos.max())
    ws = eb.alloc_workspace(eb.attention_decode_workspace_bytes(desc, B, max_pos))
    eb.attention_decode_batched(desc, layer, B, to_dev(pos), max_pos, to_dev(q, torch.float16),
                                to_dev(k, torch.float16), to_dev(v, torch.float16), kcd, vcd,
                                max_seq * Hkv * hd, o, ws)
    got = to_np(o)
    order = np.argsort(pos, kind="stable")
    threads = max(1, min(32, os.cpu_count() or 1))
    for b in list(order[:4]) + list(order[-4:]):
        p = int(pos[b])
        kc = to_np(kcd[b, :p + 1])  # rows 0..p as the device holds them (row p written)
        vc = to_np(vcd[b, :p + 1])
        kr = orc.round_f16(orc.rope(k[b], cos, sin, 1, Hkv, hd, p)).reshape(Hkv, hd)
        assert np.array_equal(kc[p], kr), f"cfg5 seq {b}: new k row"
        assert np.array_equal(vc[p], v[b]), f"cfg5 seq {b}: new v row"
        qr = orc.rope(q[b], cos, sin, 1, H, hd, p)
        want = orc.attn_decode_batched(qr.reshape(1, H, hd), kc.reshape(1, p + 1, Hkv, hd),
                                       vc.reshape(1, p + 1, Hkv, hd), np.array([p], np.int32),
                                       H, Hkv, hd, p + 1, (p + 1) * Hkv * hd, hd ** -0.5,
                                       nthreads=threads)
        assert_close(orc, got[b], want, what=f"cfg5 seq {b} ctx {p + 1}")
    assert eb.device_error() == 0


def test_prefill_decode_consistency(eb, orc):
    """crates/eyebrowse-nn/src/tests.rs:181-244 pattern on the fused path: the
    last prefill row equals token-by-token decode through a fresh cache."""
    import torch
    S, H, Hkv, hd, max_seq = 40, 4, 2, 128, 64
    q, k, v = randn((S, H, hd), 800), randn((S, Hkv, hd), 801), randn((S, Hkv, hd), 802)
    qw = (1 + 0.1 * randn((hd,), 803)).astype(np.float32)
    kw = (1 + 0.1 * randn((hd,), 804)).astype(np.float32)
    cos, sin = _tables(eb, max_seq, hd, 1e4)
    desc = eb.make_desc(H, Hkv, hd, max_seq)
    layer = eb.make_layer(q_norm_w=to_dev(qw), k_norm_w=to_dev(kw), rope_cos=to_dev(cos),
                          rope_sin=to_dev(sin))
    kc = torch.zeros(max_seq * Hkv * hd, device="cuda")
    vc = torch.zeros_like(kc)
    o = torch.empty(S * H * hd, device="cuda")
    ws = eb.alloc_workspace(eb.attention_prefill_workspace_bytes(desc, S))
    eb.attention_prefill(desc, layer, S, to_dev(q), to_dev(k), to_dev(v), kc, vc, o, ws)
    pre_last = to_np(o).reshape(S, -1)[-1]
    kc2 = torch.full_like(kc, float("nan"))
    vc2 = torch.full_like(vc, float("nan"))
    dws = eb.alloc_workspace(eb.attention_decode_workspace_bytes(desc, 1, max_seq - 1))
    od = torch.empty(H * hd, device="cuda")
    for pos in range(S):
        eb.attention_decode(desc, layer, pos, to_dev(q[pos]), to_dev(k[pos]), to_dev(v[pos]),
                            kc2, vc2, od, dws)
    assert orc.rel_l2(to_np(od), pre_last) < 2e-3
    assert_close(orc, to_np(kc2)[: S * Hkv * hd], to_np(kc)[: S * Hkv * hd], max_abs=1e-5,
                 rel_l2=1e-6, what="decode-built cache vs prefill-built cache")
