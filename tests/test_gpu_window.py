"""GPU parity of sliding-window attention (eb_attn_desc.window > 0: query row
i sees key rows i - window < j <= i), the masking of Gemma local layers and
Mistral's sliding window, which the reference defers.

- HF transformers fixtures (tests/golden/hf_attn_gemma_local.npz,
  hf_attn_mistral_swa.npz, mask from HF's sliding_window_causal_mask_function)
  through the full prefill path and token-by-token decode, with cache rows
  that fell out of the window poisoned with NaN (they must not be read).
- Long prefills against the oracle on every tensor-core kernel shape (the
  two-tile GQA-pair kernel, one tile, head_dim 64/128/256, f16/bf16 caches
  and the f32 split path) at windows that start mid-tile, on tile edges,
  of one row, and wider than the sequence (bit-identical to no window).
- Decode against the oracle for the vector kernel (f32, bf16 caches) and
  the tcgen05 kernel (f16), single and batched, and the SIMT path.
Tolerances: max-abs <= 2e-3, rel-L2 <= 1e-3 against the f32 oracle (with
the 16-bit rounding of the operands the kernels feed the tensor cores).
"""
import os

import numpy as np
import pytest

from _util import assert_close, randn, to_dev, to_np

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    z = np.load(os.path.join(GOLDEN, f"hf_attn_{name}.npz"))
    seq, h, hkv, hd, ra = (int(x) for x in z["meta"])
    return z, seq, h, hkv, hd, ra


def _layer(eb, z, hd, cos, sin):
    qw = to_dev(z["q_norm_w"]) if "q_norm_w" in z.files else None
    kw = to_dev(z["k_norm_w"]) if "k_norm_w" in z.files else None
    vw = to_dev(np.ones(hd, np.float32)) if int(z["v_norm"]) else None
    return eb.make_layer(qw, kw, vw, to_dev(cos), to_dev(sin))


@pytest.mark.parametrize("name", ["gemma_local", "mistral_swa"])
def test_window_prefill_matches_hf(eb, orc, name):
    import torch
    z, seq, h, hkv, hd, ra = _load(name)
    window = int(z["window"])
    cos, sin = eb.rope_tables(seq, hd, float(z["theta"]), rope_angles=ra)
    desc = eb.make_desc(h, hkv, hd, seq, scale=float(z["scale"]), eps=float(z["eps"]),
                        window=window)
    layer = _layer(eb, z, hd, cos, sin)
    kc = torch.zeros(seq * hkv * hd, device="cuda")
    vc = torch.zeros_like(kc)
    o = torch.full((seq * h * hd,), float("nan"), device="cuda")
    ws = eb.alloc_workspace(eb.attention_prefill_workspace_bytes(desc, seq))
    eb.attention_prefill(desc, layer, seq, to_dev(z["q"]), to_dev(z["k"]), to_dev(z["v"]), kc,
                         vc, o, ws)
    assert_close(orc, to_np(o), z["o"], what=f"{name} prefill vs HF")
    assert_close(orc, to_np(kc), z["k_cache"], max_abs=1e-4, rel_l2=1e-5, what="k cache")
    assert eb.device_error() == 0


@pytest.mark.parametrize("name", ["gemma_local", "mistral_swa"])
def test_window_decode_steps_match_hf(eb, orc, name):
    """One token at a time from an empty cache: every step's output equals
    HF's row; rows below the window hold NaN when the step runs."""
    import torch
    z, seq, h, hkv, hd, ra = _load(name)
    window = int(z["window"])
    cos, sin = eb.rope_tables(seq, hd, float(z["theta"]), rope_angles=ra)
    desc = eb.make_desc(h, hkv, hd, seq, scale=float(z["scale"]), eps=float(z["eps"]),
                        window=window)
    layer = _layer(eb, z, hd, cos, sin)
    kc = torch.full((seq, hkv, hd), float("nan"), device="cuda")
    vc = torch.full_like(kc, float("nan"))
    q, k, v = (to_dev(z[n].reshape(seq, -1)) for n in ("q", "k", "v"))
    want = z["o"].reshape(seq, -1)
    nb = eb.attention_decode_workspace_bytes(desc, 1, seq - 1)
    ws = eb.alloc_workspace(nb) if nb else None
    o = torch.empty(h * hd, device="cuda")
    for pos in range(seq):
        lo = max(0, pos - window + 1)
        kc[:lo] = float("nan")
        vc[:lo] = float("nan")
        eb.attention_decode(desc, layer, pos, q[pos], k[pos], v[pos], kc, vc, o, ws)
        assert_close(orc, to_np(o), want[pos], what=f"{name} decode pos={pos}")
    assert eb.device_error() == 0


def _prefill_case(eb, orc, hd, H, Hkv, S, window, cache, seed):
    """Prefill with no norm/RoPE (the window is the subject); returns (got, want)."""
    import torch
    code = {"f16": eb.EB_F16, "bf16": eb.EB_BF16, "f32": eb.EB_F32}[cache]
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[cache]
    rnd = {"f16": orc.round_f16, "bf16": orc.round_bf16, "f32": lambda x: x}[cache]
    q = rnd(randn((S, H, hd), seed, 0.5)).reshape(S, H, hd)
    k = rnd(randn((S, Hkv, hd), seed + 1, 0.5)).reshape(S, Hkv, hd)
    v = rnd(randn((S, Hkv, hd), seed + 2)).reshape(S, Hkv, hd)
    desc = eb.make_desc(H, Hkv, hd, S, dtype_qkv=code, dtype_cache=code, dtype_out=eb.EB_F32,
                        window=window)
    layer = eb.make_layer()
    kc = torch.zeros(S * Hkv * hd, device="cuda", dtype=tdt)
    vc = torch.zeros_like(kc)
    o = torch.full((S * H * hd,), float("nan"), device="cuda")
    ws = eb.alloc_workspace(eb.attention_prefill_workspace_bytes(desc, S))
    eb.attention_prefill(desc, layer, S, to_dev(q, tdt), to_dev(k, tdt), to_dev(v, tdt), kc, vc,
                         o, ws)
    want = orc.attn_prefill_part(q, k, v, H, Hkv, S, hd, hd ** -0.5, (0, S), (0, H),
                                 nthreads=8, window=window)
    return to_np(o), want


@pytest.mark.parametrize("hd,H,Hkv,S,window,cache", [
    (128, 32, 8, 2560, 300, "f16"),    # two-tile GQA-pair kernel, window starts mid-tile
    (128, 32, 8, 2560, 1024, "bf16"),  # window on a tile edge
    (128, 8, 2, 1000, 1, "f16"),       # each row sees only itself
    (128, 8, 2, 1000, 129, "f16"),
    (64, 4, 2, 700, 100, "bf16"),
    (256, 2, 1, 600, 200, "f16"),
    (128, 6, 2, 515, 64, "f32"),       # f32 cache: f16 hi/lo split products
    (256, 4, 2, 400, 77, "f32"),
])
def test_window_prefill_matches_oracle(eb, orc, hd, H, Hkv, S, window, cache):
    got, want = _prefill_case(eb, orc, hd, H, Hkv, S, window, cache, seed=hd + S + window)
    # bf16 caches: the tensor cores take P in bf16 too (A and B share one
    # type), whose 8-bit mantissa alone costs ~1e-3 relative error
    tol = dict(max_abs=8e-3, rel_l2=4e-3) if cache == "bf16" else {}
    assert_close(orc, got, want, what=f"window prefill hd={hd} H={H} S={S} w={window} {cache}",
                 **tol)
    assert eb.device_error() == 0


@pytest.mark.parametrize("cache", ["f16", "f32"])
def test_window_wider_than_sequence_is_causal(eb, orc, cache):
    """A window of at least S rows masks nothing: bit-identical to window 0."""
    a, _ = _prefill_case(eb, orc, 128, 16, 4, 600, 600, cache, seed=5)
    b, _ = _prefill_case(eb, orc, 128, 16, 4, 600, 0, cache, seed=5)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("cache,hd,G,pos,window", [
    ("f32", 128, 2, 3000, 1000),   # vector kernel, split-K over the window
    ("f32", 128, 2, 3000, 37),
    ("bf16", 64, 4, 2047, 513),
    ("f16", 128, 4, 5000, 700),    # tcgen05 decode
    ("f16", 256, 2, 4095, 64),
    ("f16", 128, 8, 100, 4096),    # window wider than the context
])
def test_window_decode_matches_oracle(eb, orc, cache, hd, G, pos, window):
    import torch
    Hkv = 2
    H = G * Hkv
    max_seq = pos + 64
    code = {"f16": eb.EB_F16, "bf16": eb.EB_BF16, "f32": eb.EB_F32}[cache]
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[cache]
    rnd = {"f16": orc.round_f16, "bf16": orc.round_bf16, "f32": lambda x: x}[cache]
    seed = pos + window + hd
    kc = rnd(randn((max_seq, Hkv, hd), seed)).reshape(max_seq, Hkv, hd)
    vc = rnd(randn((max_seq, Hkv, hd), seed + 1)).reshape(max_seq, Hkv, hd)
    q = rnd(randn((H, hd), seed + 2))
    k = rnd(randn((Hkv, hd), seed + 3))
    v = rnd(randn((Hkv, hd), seed + 4))
    lo = max(0, pos - window + 1)
    kp, vp = kc.copy(), vc.copy()
    kp[:lo] = np.nan   # out of the window: never read
    vp[:lo] = np.nan
    kp[pos:] = np.nan  # past the context: never reaches the output
    vp[pos:] = np.nan
    desc = eb.make_desc(H, Hkv, hd, max_seq, dtype_qkv=code, dtype_cache=code,
                        dtype_out=eb.EB_F32, window=window)
    layer = eb.make_layer()
    kcd, vcd = to_dev(kp, tdt), to_dev(vp, tdt)
    o = torch.full((H * hd,), float("nan"), device="cuda")
    nb = eb.attention_decode_workspace_bytes(desc, 1, pos)
    ws = eb.alloc_workspace(nb) if nb else None
    eb.attention_decode(desc, layer, pos, to_dev(q, tdt), to_dev(k, tdt), to_dev(v, tdt), kcd,
                        vcd, o, ws)
    kc[pos], vc[pos] = k.reshape(Hkv, hd), v.reshape(Hkv, hd)
    want = orc.attn_decode(q, kc, vc, H, Hkv, pos, hd, max_seq, hd ** -0.5, window=window)
    assert_close(orc, to_np(o), want, what=f"window decode {cache} hd={hd} G={G} pos={pos}")
    assert eb.device_error() == 0


@pytest.mark.parametrize("cache", ["f16", "f32"])
def test_window_decode_batched(eb, orc, cache):
    """Per-sequence windows inside one batched call: short contexts (fully
    inside the window) beside long ones, twice through the same workspace."""
    import torch
    B, H, Hkv, hd, max_seq, window = 5, 16, 4, 128, 9216, 1024
    code = eb.EB_F16 if cache == "f16" else eb.EB_F32
    tdt = torch.float16 if cache == "f16" else torch.float32
    rnd = orc.round_f16 if cache == "f16" else (lambda x: x)
    pos = np.array([5, 600, 1023, 3000, 9000], np.int32)
    kc = rnd(randn((B, max_seq, Hkv, hd), 11)).reshape(B, max_seq, Hkv, hd)
    vc = rnd(randn((B, max_seq, Hkv, hd), 12)).reshape(B, max_seq, Hkv, hd)
    q = rnd(randn((B, H, hd), 13)).reshape(B, H, hd)
    k = rnd(randn((B, Hkv, hd), 14)).reshape(B, Hkv, hd)
    v = rnd(randn((B, Hkv, hd), 15)).reshape(B, Hkv, hd)
    kp, vp = kc.copy(), vc.copy()
    for b, p in enumerate(pos):
        kp[b, :max(0, p - window + 1)] = np.nan
        vp[b, :max(0, p - window + 1)] = np.nan
    desc = eb.make_desc(H, Hkv, hd, max_seq, dtype_qkv=code, dtype_cache=code,
                        dtype_out=eb.EB_F32, window=window)
    layer = eb.make_layer()
    kcd, vcd = to_dev(kp, tdt), to_dev(vp, tdt)
    ws = eb.alloc_workspace(eb.attention_decode_workspace_bytes(desc, B, int(pos.max())))
    o = torch.full((B * H * hd,), float("nan"), device="cuda")
    for _ in range(2):
        eb.attention_decode_batched(desc, layer, B, to_dev(pos), int(pos.max()), to_dev(q, tdt),
                                    to_dev(k, tdt), to_dev(v, tdt), kcd, vcd,
                                    max_seq * Hkv * hd, o, ws)
    for b, p in enumerate(pos):
        kc[b, p], vc[b, p] = k[b], v[b]
    want = orc.attn_decode_batched(q, kc, vc, pos, H, Hkv, hd, max_seq, max_seq * Hkv * hd,
                                   hd ** -0.5, nthreads=4, window=window)
    assert_close(orc, to_np(o), want, what=f"batched window decode {cache}")
    assert eb.device_error() == 0


def test_window_simt_paths(eb, orc):
    """head_dim 32 (SIMT kernels) prefill and decode with a window."""
    import torch
    H, Hkv, hd, S, window = 4, 2, 32, 90, 17
    q = randn((S, H, hd), 21)
    k = randn((S, Hkv, hd), 22)
    v = randn((S, Hkv, hd), 23)
    desc = eb.make_desc(H, Hkv, hd, S, window=window)
    layer = eb.make_layer()
    kc = torch.zeros(S * Hkv * hd, device="cuda")
    vc = torch.zeros_like(kc)
    o = torch.full((S * H * hd,), float("nan"), device="cuda")
    eb.attention_prefill(desc, layer, S, to_dev(q), to_dev(k), to_dev(v), kc, vc, o)
    want = orc.attn_prefill(q, k, v, H, Hkv, S, hd, hd ** -0.5, window=window)
    assert_close(orc, to_np(o), want, what="simt window prefill")
    od = torch.empty(H * hd, device="cuda")
    pos = S - 1
    kc2, vc2 = kc.clone(), vc.clone()
    eb.attention_decode(desc, layer, pos, to_dev(q[pos]), to_dev(k[pos]), to_dev(v[pos]), kc2,
                        vc2, od)
    assert_close(orc, to_np(od), want.reshape(S, -1)[pos], what="simt window decode")
    assert eb.device_error() == 0
