"""Pins the CPU oracle before it is trusted as the checker.

Pins, in order of authority:
  * the reference's own known-answer assertions (kv_write placement,
    RoPE table rows, build_partial pass-through), re-run on the same inputs;
  * the reference's kernel unit-test inputs (ramps), checked against an
    independent float64 evaluation of the same formula;
  * HF transformers attention fixtures (tests/golden, made by
    gen_hf_golden.py), the library the reference's own golden scripts use.
"""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _attn_f64(q, k, v, h, hkv, s, hd, scale, n_q=None, pos0=0):
    """Independent float64 softmax attention (causal, GQA, seq-major)."""
    q = q.reshape(-1, h, hd).astype(np.float64)
    k = k.reshape(-1, hkv, hd).astype(np.float64)
    v = v.reshape(-1, hkv, hd).astype(np.float64)
    g = h // hkv
    rows = q.shape[0]
    o = np.zeros((rows, h, hd))
    for i in range(rows):
        last = pos0 + i
        for hh in range(h):
            sc = k[: last + 1, hh // g] @ q[i, hh] * scale
            w = np.exp(sc - sc.max())
            w /= w.sum()
            o[i, hh] = w @ v[: last + 1, hh // g]
    return o.ravel()


def test_rel_l2_matches_definition(orc):
    rng = np.random.default_rng(0)
    a = rng.standard_normal(1000).astype(np.float32)
    b = rng.standard_normal(1000).astype(np.float32)
    want = np.linalg.norm(a.astype(np.float64) - b) / (np.linalg.norm(b.astype(np.float64)) + 1e-12)
    assert abs(orc.rel_l2(a, b) - want) < 1e-6


def test_round_f16_matches_ieee(orc):
    rng = np.random.default_rng(1)
    x = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 10,
        rng.standard_normal(5000).astype(np.float32) * 1e-5,   # f16 subnormal range
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e9, -1e9, 2.0 ** -24, 2.0 ** -25,
                  3 * 2.0 ** -26, np.inf, -np.inf], np.float32),
    ])
    got = orc.round_f16(x)
    want = x.astype(np.float16).astype(np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_kv_write_places_rows(orc):
    # crates/eyebrowse-kernels/src/ops.rs:271-292
    hkv, hd, max_seq = 2, 4, 8
    cache = np.zeros(max_seq * hkv * hd, np.float32)
    src = np.arange(hkv * hd, dtype=np.float32) + 1.0
    got = orc.kv_write(cache, src, hkv, 1, hd, max_seq, 3)
    for head in range(hkv):
        for d in range(hd):
            assert got[(3 * hkv + head) * hd + d] == src[head * hd + d]
    assert got[0] == 0.0
    assert np.count_nonzero(got) == hkv * hd


def test_rope_build_tables(orc):
    # crates/eyebrowse-nn/src/tests.rs:152-177
    max_seq, hd, theta = 8, 4, 10000.0
    half = hd // 2
    cos, sin = orc.rope_tables(max_seq, hd, theta)
    for k in range(half):
        assert abs(cos[k] - 1.0) < 1e-6 and abs(sin[k]) < 1e-6
    s = 3
    for k in range(half):
        ang = s * (theta ** (-(2.0 * k) / hd))
        assert abs(cos[s * half + k] - np.cos(ang)) < 1e-5
        assert abs(sin[s * half + k] - np.sin(ang)) < 1e-5


def test_build_partial_zeros_high_frequencies(orc):
    # crates/eyebrowse-nn/src/rope.rs:82-103
    max_seq, hd = 5, 8
    half = hd // 2
    fc, fs = orc.rope_tables(max_seq, hd, 10000.0)
    pc, ps = orc.rope_tables(max_seq, hd, 10000.0, rope_angles=2)
    for s in range(max_seq):
        for k in range(2):
            assert pc[s * half + k] == fc[s * half + k] and ps[s * half + k] == fs[s * half + k]
        for k in range(2, half):
            assert pc[s * half + k] == 1.0 and ps[s * half + k] == 0.0


def test_rope_ramp(orc):
    # crates/eyebrowse-kernels/src/rope.rs:92-111 inputs
    seq, n_heads, hd, theta = 4, 2, 8, 10000.0
    cos, sin = orc.rope_tables(seq, hd, theta)
    x = (np.arange(seq * n_heads * hd, dtype=np.float32) * np.float32(0.03) - np.float32(0.5))
    got = orc.rope(x, cos, sin, seq, n_heads, hd)
    half = hd // 2
    xr = x.reshape(seq, n_heads, hd).astype(np.float64)
    want = np.empty_like(xr)
    for s in range(seq):
        ang = s * theta ** (-2.0 * np.arange(half) / hd)
        c, sn = np.cos(ang), np.sin(ang)
        want[s, :, :half] = xr[s, :, :half] * c - xr[s, :, half:] * sn
        want[s, :, half:] = xr[s, :, half:] * c + xr[s, :, :half] * sn
    assert orc.rel_l2(got, want.ravel()) < 1e-6


def test_rmsnorm_ramp(orc):
    # crates/eyebrowse-kernels/src/rmsnorm.rs:72-90 inputs
    rows, dim, eps = 3, 320, 1e-6
    i = np.arange(rows * dim)
    x = ((i % 17).astype(np.float32) * np.float32(0.05) - np.float32(0.4)).astype(np.float32)
    w = (np.float32(1.0) + np.arange(dim, dtype=np.float32) * np.float32(0.001)).astype(np.float32)
    got = orc.rmsnorm(x, w, rows, dim, eps)
    xr = x.reshape(rows, dim).astype(np.float64)
    want = xr / np.sqrt((xr ** 2).mean(1, keepdims=True) + eps) * w
    assert orc.rel_l2(got, want.ravel()) < 1e-6


def test_linear_ramp(orc):
    # crates/eyebrowse-kernels/src/matmul.rs:261-279 inputs (in_f not a multiple of 16)
    m, in_f, out_f = 5, 33, 7
    x = orc.ramp(m * in_f, -0.2, 0.01)
    w = orc.round_f16(orc.ramp(out_f * in_f, -0.3, 0.005))
    got = orc.linear(x, w, m, in_f, out_f)
    want = x.reshape(m, in_f).astype(np.float64) @ w.reshape(out_f, in_f).astype(np.float64).T
    assert orc.rel_l2(got, want.ravel()) < 1e-6
    # k summed in order in one f32 accumulator, multiply and add rounded apart
    acc = np.float32(0)
    for k in range(in_f):
        acc = np.float32(acc + np.float32(x[k] * w[k]))
    assert got[0] == acc


def test_linear_threaded_is_bit_identical(orc):
    rng = np.random.default_rng(5)
    m, in_f, out_f = 3, 200, 77
    x = rng.standard_normal(m * in_f).astype(np.float32)
    w = orc.round_f16(rng.standard_normal(out_f * in_f).astype(np.float32))
    assert np.array_equal(orc.linear(x, w, m, in_f, out_f),
                          orc.linear_threaded(x, w, m, in_f, out_f, 4))


def test_windowed_decode_batched_equals_single(orc):
    """orc_attn_decode_batched with a window = orc_attn_decode_window per
    sequence = the full decode over the window's rows only."""
    rng = np.random.default_rng(9)
    h, hkv, hd, ms, window = 4, 2, 16, 64, 10
    pos = np.array([3, 9, 10, 40, 63], np.int32)
    B = pos.size
    kc = rng.standard_normal((B, ms, hkv, hd)).astype(np.float32)
    vc = rng.standard_normal((B, ms, hkv, hd)).astype(np.float32)
    q = rng.standard_normal((B, h, hd)).astype(np.float32)
    got = orc.attn_decode_batched(q, kc, vc, pos, h, hkv, hd, ms, ms * hkv * hd, 0.25,
                                  nthreads=2, window=window).reshape(B, h * hd)
    for b, p in enumerate(pos):
        one = orc.attn_decode(q[b], kc[b], vc[b], h, hkv, int(p), hd, ms, 0.25, window=window)
        assert np.array_equal(got[b], one)
        lo = max(0, int(p) - window + 1)
        # the same rows moved to the front of a cache: a plain full decode
        sub = orc.attn_decode(q[b], kc[b, lo:p + 1], vc[b, lo:p + 1], h, hkv, int(p) - lo, hd,
                              ms, 0.25)
        assert np.array_equal(one, sub)


def test_attn_prefill_ramp(orc):
    # crates/eyebrowse-kernels/src/attention.rs:174-202 inputs
    h, hkv, s, hd = 2, 1, 5, 8
    q = orc.ramp(h * s * hd, -0.5, 0.011)
    k = orc.ramp(hkv * s * hd, -0.3, 0.007)
    v = orc.ramp(hkv * s * hd, 0.2, 0.013)
    got = orc.attn_prefill(q, k, v, h, hkv, s, hd)
    want = _attn_f64(q, k, v, h, hkv, s, hd, 1 / np.sqrt(hd))
    assert orc.rel_l2(got, want) < 1e-6


def test_attn_decode_ramp(orc):
    # crates/eyebrowse-kernels/src/attention.rs:204-233 inputs
    h, hkv, hd, max_seq, pos = 4, 2, 8, 16, 5
    q = orc.ramp(h * hd, -0.4, 0.02)
    kc = orc.ramp(hkv * max_seq * hd, -0.2, 0.005)
    vc = orc.ramp(hkv * max_seq * hd, 0.1, 0.009)
    got = orc.attn_decode(q, kc, vc, h, hkv, pos, hd, max_seq)
    want = _attn_f64(q, kc, vc, h, hkv, 1, hd, 1 / np.sqrt(hd), pos0=pos)
    assert orc.rel_l2(got, want) < 1e-6


def _load(name):
    z = np.load(os.path.join(GOLDEN, f"hf_attn_{name}.npz"))
    seq, h, hkv, hd, rope_angles = (int(x) for x in z["meta"])
    return z, seq, h, hkv, hd, rope_angles


def _window(z) -> int:
    return int(z["window"]) if "window" in z.files else 0


@pytest.mark.parametrize("name", ["qwen3", "llama", "gemma", "gemma_local", "mistral_swa"])
def test_oracle_matches_hf_prefill(orc, name):
    z, seq, h, hkv, hd, ra = _load(name)
    cos, sin = orc.rope_tables(seq, hd, float(z["theta"]), rope_angles=ra)
    vw = np.ones(hd, np.float32) if int(z["v_norm"]) else None
    o, kc, vc = orc.attention_prefill(
        z["q"], z["k"], z["v"], seq=seq, h=h, hkv=hkv, hd=hd, max_seq=seq,
        scale=float(z["scale"]), eps=float(z["eps"]),
        q_norm_w=z["q_norm_w"] if "q_norm_w" in z else None,
        k_norm_w=z["k_norm_w"] if "k_norm_w" in z else None,
        v_norm_w=vw, cos=cos, sin=sin, window=_window(z))
    assert orc.rel_l2(o, z["o"]) < 2e-5
    assert orc.rel_l2(kc, z["k_cache"]) < 2e-6
    assert orc.rel_l2(vc, z["v_cache"]) < 2e-6


@pytest.mark.parametrize("name", ["qwen3", "gemma", "gemma_local", "mistral_swa"])
def test_oracle_decode_steps_match_hf(orc, name):
    """Token-by-token decode through a fresh cache reproduces HF's causal rows
    (the pattern of eyebrowse-nn/src/tests.rs:181-244). With a sliding window
    the rows that fell out of it are poisoned before each step."""
    z, seq, h, hkv, hd, ra = _load(name)
    window = _window(z)
    cos, sin = orc.rope_tables(seq, hd, float(z["theta"]), rope_angles=ra)
    vw = np.ones(hd, np.float32) if int(z["v_norm"]) else None
    kc = np.full(seq * hkv * hd, np.nan, np.float32)   # poison: unwritten rows must not be read
    vc = np.full(seq * hkv * hd, np.nan, np.float32)
    q, k, v = (z[n].reshape(seq, -1) for n in ("q", "k", "v"))
    want = z["o"].reshape(seq, -1)
    for pos in range(seq):
        lo = max(0, pos - window + 1) * hkv * hd if window else 0
        kin, vin = kc.copy(), vc.copy()
        kin[:lo] = np.nan
        vin[:lo] = np.nan
        o, kout, vout = orc.attention_decode(
            q[pos], k[pos], v[pos], pos=pos, h=h, hkv=hkv, hd=hd, max_seq=seq,
            scale=float(z["scale"]), kcache=kin, vcache=vin, eps=float(z["eps"]),
            q_norm_w=z["q_norm_w"] if "q_norm_w" in z else None,
            k_norm_w=z["k_norm_w"] if "k_norm_w" in z else None,
            v_norm_w=vw, cos=cos, sin=sin, window=window)
        kc[lo:], vc[lo:] = kout[lo:], vout[lo:]
        assert orc.rel_l2(o, want[pos]) < 2e-5, pos
    assert orc.rel_l2(kc, z["k_cache"]) < 2e-6


def test_prng_is_xorshift(orc):
    # crates/eyebrowse-nn/src/testutil.rs:30-41: values in [-1, 1), deterministic
    a = orc.prng(64, 11)
    assert np.array_equal(a, orc.prng(64, 11))
    assert a.min() >= -1.0 and a.max() < 1.0
    assert not np.array_equal(a, orc.prng(64, 12))


def test_prefill_part_equals_full(orc):
    rng = np.random.default_rng(3)
    h, hkv, s, hd = 4, 2, 33, 16
    q = rng.standard_normal(s * h * hd).astype(np.float32)
    k = rng.standard_normal(s * hkv * hd).astype(np.float32)
    v = rng.standard_normal(s * hkv * hd).astype(np.float32)
    full = orc.attn_prefill(q, k, v, h, hkv, s, hd, 0.25)
    part = orc.attn_prefill_part(q, k, v, h, hkv, s, hd, 0.25, (0, s), (0, h), nthreads=3)
    assert np.array_equal(full, part)
