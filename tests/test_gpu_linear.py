"""GPU parity of eb_linear_f16w (linear_f16w, crates/eyebrowse-kernels/src/
matmul.rs:128-149): y [m, out] = x [m, in] (f32) @ w [out, in]^T (f16).

Covers the reference's own test (matmul.rs:261-279: ramps, in_f = 33, its
rel-L2 < 2e-3 bound), the streaming kernel for m <= 8 (Qwen3-0.6B
projections and the 151936-row LM head), the tcgen05 kernel for m > 8 (k and
out not multiples of the tile, m from 9 to 2048, fused q/k/v widths), the
scalar kernel for unaligned inputs, and the workspace check.
Tolerance against float64 sums of the same f16 weights: rel-L2 <= 1e-5 and
max-abs <= 1e-4 * max|y| (the tensor-core path carries x as f16 hi + lo
planes, ~22 bits, and accumulates in f32).
"""
import numpy as np
import pytest

from _util import randn, to_dev, to_np

pytestmark = pytest.mark.gpu


def _check(orc, got, x, w, m, in_f, out_f, rel=1e-5, what=""):
    want = (x.reshape(m, in_f).astype(np.float64) @ w.reshape(out_f, in_f).astype(np.float64).T)
    got = np.asarray(got, np.float32).reshape(m, out_f)
    assert np.isfinite(got).all(), what
    rl = orc.rel_l2(got.ravel(), want.ravel())
    ma = float(np.abs(got - want).max())
    assert rl <= rel and ma <= 1e-4 * float(np.abs(want).max()), f"{what}: rel_l2={rl:.3e} max_abs={ma:.3e}"


def _run(eb, x, w16, m, in_f, out_f, ws=True):
    import torch
    xd = to_dev(x)
    wd = torch.from_numpy(np.ascontiguousarray(w16)).cuda()
    y = torch.full((m * out_f,), float("nan"), device="cuda")
    nb = eb.linear_f16w_workspace_bytes(m, in_f, out_f)
    wsd = eb.alloc_workspace(nb) if (nb and ws) else None
    eb.linear_f16w(xd, wd, y, m, in_f, out_f, wsd)
    return to_np(y)


def test_linear_reference_case(eb, orc):
    """matmul.rs:261-279: ramps, in_f = 33 (not a multiple of 16)."""
    m, in_f, out_f = 5, 33, 7
    x = orc.ramp(m * in_f, -0.2, 0.01)
    w = orc.ramp(out_f * in_f, -0.3, 0.005)
    w16 = w.astype(np.float16)
    got = _run(eb, x, w16, m, in_f, out_f)
    want = orc.linear(x, orc.round_f16(w), m, in_f, out_f)
    assert orc.rel_l2(got, want) < 2e-3  # the reference's bound
    _check(orc, got, x, w16.astype(np.float32), m, in_f, out_f, what="reference case")
    assert eb.device_error() == 0


@pytest.mark.parametrize("m,in_f,out_f", [
    (1, 1024, 4096),     # fused q/k/v of Qwen3-0.6B, one decode row
    (1, 2048, 1024),     # o_proj
    (3, 1024, 1002),
    (8, 3072, 1024),     # down_proj, 8 rows
    (1, 1024, 151936),   # the tied LM head
])
def test_linear_rows_kernel(eb, orc, m, in_f, out_f):
    x = randn((m, in_f), m + in_f)
    w16 = (randn((out_f, in_f), out_f, 0.02)).astype(np.float16)
    got = _run(eb, x, w16, m, in_f, out_f)
    _check(orc, got, x, w16.astype(np.float32), m, in_f, out_f, what=f"rows m={m}")
    assert eb.device_error() == 0


@pytest.mark.parametrize("m,in_f,out_f", [
    (9, 1024, 4096),
    (16, 1024, 6144),     # fused gate/up of Qwen3-0.6B
    (128, 2048, 1024),
    (300, 200, 260),      # k = 3 chunks + 8, out = one tile + 4 columns
    (1000, 1024, 4096),
    (2048, 4096, 6144),   # Llama-3-8B fused q/k/v
])
def test_linear_tensor_core_kernel(eb, orc, m, in_f, out_f):
    x = randn((m, in_f), 7 * m + in_f)
    w16 = (randn((out_f, in_f), out_f + 1, 0.02)).astype(np.float16)
    got = _run(eb, x, w16, m, in_f, out_f)
    _check(orc, got, x, w16.astype(np.float32), m, in_f, out_f, what=f"tc m={m} k={in_f} n={out_f}")
    assert eb.device_error() == 0


def test_linear_unaligned_input_takes_scalar_kernel(eb, orc):
    import torch
    m, in_f, out_f = 20, 64, 48
    x = randn((m, in_f), 3)
    w16 = randn((out_f, in_f), 4, 0.1).astype(np.float16)
    buf = torch.zeros(m * in_f + 1, device="cuda")
    buf[1:] = to_dev(x.ravel())
    y = torch.full((m * out_f,), float("nan"), device="cuda")
    eb.linear_f16w(buf[1:], torch.from_numpy(w16).cuda(), y, m, in_f, out_f)  # 4-byte offset
    _check(orc, to_np(y), x, w16.astype(np.float32), m, in_f, out_f, what="unaligned x")
    assert eb.device_error() == 0


def test_linear_tensor_core_needs_workspace(eb):
    import torch
    m, in_f, out_f = 64, 128, 128
    assert eb.linear_f16w_workspace_bytes(m, in_f, out_f) == 2 * m * in_f * 2
    assert eb.linear_f16w_workspace_bytes(8, in_f, out_f) == 0
    x = torch.zeros(m * in_f, device="cuda")
    w = torch.zeros(out_f * in_f, device="cuda", dtype=torch.float16)
    y = torch.zeros(m * out_f, device="cuda")
    with pytest.raises(eb.EbError) as e:
        eb.linear_f16w(x, w, y, m, in_f, out_f)
    assert e.value.status == 4  # EB_ERR_WORKSPACE, refused before any launch


def test_fused_qkv_rows_feed_attention(eb, orc):
    """One q/k/v GEMM over [Wq; Wk; Wv]: the attention reads q, k and v in
    place through the descriptor's row strides (prefill, decode, batched
    decode), bit-identical to contiguous copies of the same rows."""
    import torch
    H, Hkv, hd, S, D, B = 8, 2, 128, 40, 256, 3
    width = (H + 2 * Hkv) * hd
    x = randn((S, D), 31)
    w16 = randn((width, D), 32, 0.05).astype(np.float16)
    xd, wd = to_dev(x), torch.from_numpy(w16).cuda()
    qkv = torch.empty(S, width, device="cuda")
    nb = eb.linear_f16w_workspace_bytes(S, D, width)
    eb.linear_f16w(xd, wd, qkv, S, D, width, eb.alloc_workspace(nb))
    q, k, v = qkv[:, :H * hd], qkv[:, H * hd:(H + Hkv) * hd], qkv[:, (H + Hkv) * hd:]
    cos, sin = eb.rope_tables(S, hd, 1e6)
    layer = eb.make_layer(rope_cos=to_dev(cos), rope_sin=to_dev(sin))
    strided = eb.make_desc(H, Hkv, hd, S, q_stride=width, kv_stride=width)
    plain = eb.make_desc(H, Hkv, hd, S)
    outs = []
    for desc, (qq, kk, vv) in ((strided, (q, k, v)),
                               (plain, (q.contiguous(), k.contiguous(), v.contiguous()))):
        kc = torch.zeros(S, Hkv, hd, device="cuda")
        vc = torch.zeros_like(kc)
        o = torch.empty(S, H, hd, device="cuda")
        ws = eb.alloc_workspace(eb.attention_prefill_workspace_bytes(desc, S))
        eb.attention_prefill(desc, layer, S - B, qq, kk, vv, kc, vc, o, ws)
        od = torch.empty(H * hd, device="cuda")
        eb.attention_decode(desc, layer, S - B, qq[S - B], kk[S - B], vv[S - B], kc, vc, od)
        # batched: B sequences sharing the prefix cache, one new row each
        kcb, vcb = kc.repeat(B, 1, 1), vc.repeat(B, 1, 1)
        pos = torch.full((B,), S - B, dtype=torch.int32, device="cuda")
        ob = torch.empty(B, H * hd, device="cuda")
        dws = eb.alloc_workspace(eb.attention_decode_workspace_bytes(desc, B, S - 1))
        eb.attention_decode_batched(desc, layer, B, pos, S - 1, qq[S - B:], kk[S - B:], vv[S - B:],
                                    kcb, vcb, S * Hkv * hd, ob, dws)
        outs.append((to_np(o)[:S - B], to_np(od), to_np(ob)))
    for a, b in zip(*outs):
        assert np.array_equal(a, b)
    assert eb.device_error() == 0
