"""GPU parity of the kernel-level C-ABI drop-ins against the oracle.

The first group re-runs the reference's own kernel unit tests
(crates/eyebrowse-kernels/src/*.rs #[cfg(test)]) with the same inputs and
tolerances; the second drives the tensor-core / vector paths with seeded
inputs at the north-star tolerance.
"""
import numpy as np
import pytest

from _util import MAX_ABS, REL_L2, assert_close, randn, to_dev, to_np

pytestmark = pytest.mark.gpu


def test_attn_prefill_matches_cpu(eb, orc):
    # crates/eyebrowse-kernels/src/attention.rs:174-202
    import torch
    h, hkv, s, hd = 2, 1, 5, 8
    q = orc.ramp(h * s * hd, -0.5, 0.011)
    k = orc.ramp(hkv * s * hd, -0.3, 0.007)
    v = orc.ramp(hkv * s * hd, 0.2, 0.013)
    o = torch.empty(s * h * hd, device="cuda")
    eb.attn_prefill(to_dev(q), to_dev(k), to_dev(v), o, h, hkv, s, hd, 1.0 / np.sqrt(hd))
    want = orc.attn_prefill(q, k, v, h, hkv, s, hd)
    assert orc.rel_l2(to_np(o), want) < 1e-4


def test_attn_decode_matches_cpu(eb, orc):
    # crates/eyebrowse-kernels/src/attention.rs:204-233
    import torch
    h, hkv, hd, max_seq, pos = 4, 2, 8, 16, 5
    q = orc.ramp(h * hd, -0.4, 0.02)
    kc = orc.ramp(hkv * max_seq * hd, -0.2, 0.005)
    vc = orc.ramp(hkv * max_seq * hd, 0.1, 0.009)
    o = torch.empty(h * hd, device="cuda")
    eb.attn_decode(to_dev(q), to_dev(kc), to_dev(vc), o, h, hkv, pos, hd, max_seq,
                   1.0 / np.sqrt(hd))
    want = orc.attn_decode(q, kc, vc, h, hkv, pos, hd, max_seq)
    assert orc.rel_l2(to_np(o), want) < 1e-4


def test_rope_matches_cpu(eb, orc):
    # crates/eyebrowse-kernels/src/rope.rs:92-111
    import torch
    seq, n_heads, hd = 4, 2, 8
    cos, sin = orc.rope_tables(seq, hd, 10000.0)
    x = (np.arange(seq * n_heads * hd, dtype=np.float32) * np.float32(0.03) - np.float32(0.5))
    out = torch.empty(seq * n_heads * hd, device="cuda")
    eb.rope(to_dev(x), to_dev(cos), to_dev(sin), out, seq, n_heads, hd, 0)
    want = orc.rope(x, cos, sin, seq, n_heads, hd)
    assert orc.rel_l2(to_np(out), want) < 1e-5
    # the kernel's RoPE is the reference's exact f32 arithmetic
    assert np.array_equal(to_np(out), want)


def test_rope_base_pos_in_place(eb, orc):
    seq, n_heads, hd, base = 3, 4, 64, 9
    cos, sin = orc.rope_tables(16, hd, 1e6)
    x = randn((seq * n_heads * hd,), 1)
    xt = to_dev(x)
    eb.rope(xt, to_dev(cos), to_dev(sin), xt, seq, n_heads, hd, base)
    assert np.array_equal(to_np(xt), orc.rope(x, cos, sin, seq, n_heads, hd, base))


def test_rmsnorm_matches_cpu(eb, orc):
    # crates/eyebrowse-kernels/src/rmsnorm.rs:72-90
    import torch
    rows, dim, eps = 3, 320, 1e-6
    i = np.arange(rows * dim)
    x = ((i % 17).astype(np.float32) * np.float32(0.05) - np.float32(0.4)).astype(np.float32)
    w = (np.float32(1.0) + np.arange(dim, dtype=np.float32) * np.float32(0.001)).astype(np.float32)
    out = torch.empty(rows * dim, device="cuda")
    eb.rmsnorm(to_dev(x), to_dev(w), out, rows, dim, eps)
    assert orc.rel_l2(to_np(out), orc.rmsnorm(x, w, rows, dim, eps)) < 1e-4


def test_kv_write_places_rows(eb, orc):
    # crates/eyebrowse-kernels/src/ops.rs:271-292
    hkv, hd, max_seq = 2, 4, 8
    cache = to_dev(np.zeros(max_seq * hkv * hd, np.float32))
    src = np.arange(hkv * hd, dtype=np.float32) + 1.0
    eb.kv_write(cache, to_dev(src), hkv, 1, hd, max_seq, 3)
    got = to_np(cache)
    assert np.array_equal(got, orc.kv_write(np.zeros(max_seq * hkv * hd, np.float32), src, hkv, 1,
                                            hd, max_seq, 3))
    assert got[0] == 0.0


@pytest.mark.parametrize("hd", [64, 128, 256])
@pytest.mark.parametrize("s", [1, 77, 128, 300])
def test_attn_prefill_tensor_core_f32(eb, orc, hd, s):
    """f32 attn_prefill on tcgen05 (hi/lo split operands) vs the oracle, ragged S."""
    import torch
    h, hkv = 4, 2
    q, k, v = randn((s, h, hd), 10 + hd), randn((s, hkv, hd), 20 + hd), randn((s, hkv, hd), 30)
    o = torch.empty(s * h * hd, device="cuda")
    ws = eb.alloc_workspace(eb.attn_prefill_workspace_bytes(h, hkv, s, hd))
    scale = 1.0 / np.sqrt(hd)
    eb.attn_prefill(to_dev(q), to_dev(k), to_dev(v), o, h, hkv, s, hd, scale, ws)
    want = orc.attn_prefill(q, k, v, h, hkv, s, hd, scale)
    assert_close(orc, to_np(o), want, what=f"prefill hd={hd} s={s}")
    assert eb.device_error() == 0


@pytest.mark.parametrize("hd", [64, 128, 256])
@pytest.mark.parametrize("pos", [0, 5, 1000, 3001])
def test_attn_decode_vector_f32(eb, orc, hd, pos):
    """f32 attn_decode, split-K with a workspace and single-CTA without one."""
    import torch
    h, hkv, max_seq = 8, 2, 3072 + 64
    q = randn((h, hd), 1)
    kc = randn((max_seq, hkv, hd), 2)
    vc = randn((max_seq, hkv, hd), 3)
    kc[pos + 1:] = np.nan  # unwritten rows must never be read
    vc[pos + 1:] = np.nan
    want = orc.attn_decode(q, kc, vc, h, hkv, pos, hd, max_seq)
    qd, kd, vd = to_dev(q), to_dev(kc), to_dev(vc)
    for use_ws in (True, False):
        o = torch.empty(h * hd, device="cuda")
        ws = None
        if use_ws:
            nb = eb.attn_decode_workspace_bytes(h, hkv, pos, hd)
            ws = eb.alloc_workspace(nb) if nb else None
        for _ in range(2):  # the second call reuses the self-resetting counters
            eb.attn_decode(qd, kd, vd, o, h, hkv, pos, hd, max_seq, 1.0 / np.sqrt(hd), ws)
            assert_close(orc, to_np(o), want, what=f"decode hd={hd} pos={pos} ws={use_ws}")


def test_invalid_arguments_rejected(eb):
    import torch
    x = torch.zeros(64, device="cuda")
    with pytest.raises(eb.EbError) as e:
        eb.attn_decode(x, x, x, x, 4, 2, 16, 8, 16, 0.3)  # pos == max_seq
    assert e.value.status == 1
    with pytest.raises(eb.EbError) as e:
        eb.attn_prefill(x, x, x, x, 3, 2, 1, 8, 0.3)  # h % hkv != 0
    assert e.value.status == 1
    with pytest.raises(eb.EbError) as e:
        eb.attn_prefill(x, x, x, x, 2, 2, 1, 128, 0.3)  # tensor-core path needs a workspace
    assert e.value.status == 4
