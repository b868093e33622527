"""GPU parity of the tcgen05 decode (16-bit caches) against the oracle.

Covers f16 and bf16 caches, head_dim 64/128/256, GQA groups of 1/4/6/8
query heads, contexts inside one 64-row tile, exactly on tile edges and
across many split-K chunks, fused q/k norm + RoPE + cache write, and cache
rows past `pos` poisoned with NaN (the kernel must never let them reach the
output: their V rows are zeroed in shared memory before the PV product).
"""
import numpy as np
import pytest

from _util import assert_close, randn, to_dev, to_np

pytestmark = pytest.mark.gpu


def _round(orc, x, bf16):
    return orc.round_bf16(x) if bf16 else orc.round_f16(x)


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("hd,G", [(128, 4), (64, 8), (256, 2), (128, 1), (128, 6)])
@pytest.mark.parametrize("pos", [0, 37, 63, 64, 1000, 5000])
def test_decode_tc_matches_oracle(eb, orc, bf16, hd, G, pos):
    import torch
    Hkv = 2
    H = G * Hkv
    max_seq = 5120
    tdt = torch.bfloat16 if bf16 else torch.float16
    code = eb.EB_BF16 if bf16 else eb.EB_F16
    seed = 1000 + hd + 10 * G + pos
    kc = _round(orc, randn((max_seq, Hkv, hd), seed), bf16).reshape(max_seq, Hkv, hd)
    vc = _round(orc, randn((max_seq, Hkv, hd), seed + 1), bf16).reshape(max_seq, Hkv, hd)
    kc[pos:] = np.nan
    vc[pos:] = np.nan
    q = _round(orc, randn((H, hd), seed + 2), bf16)
    k = _round(orc, randn((Hkv, hd), seed + 3), bf16)
    v = _round(orc, randn((Hkv, hd), seed + 4), bf16)
    qw = (1 + 0.1 * randn((hd,), seed + 5)).astype(np.float32)
    kw = (1 + 0.1 * randn((hd,), seed + 6)).astype(np.float32)
    cos, sin = eb.rope_tables(max_seq, hd, 1e6)
    desc = eb.make_desc(H, Hkv, hd, max_seq, dtype_qkv=code, dtype_cache=code,
                        dtype_out=eb.EB_F32, eps=1e-6)
    layer = eb.make_layer(to_dev(qw), to_dev(kw), None, to_dev(cos), to_dev(sin))
    kcd, vcd = to_dev(kc, tdt), to_dev(vc, tdt)
    o = torch.full((H * hd,), float("nan"), device="cuda")
    nb = eb.attention_decode_workspace_bytes(desc, 1, pos)
    ws = eb.alloc_workspace(nb) if nb else None
    eb.attention_decode(desc, layer, pos, to_dev(q, tdt), to_dev(k, tdt), to_dev(v, tdt),
                        kcd, vcd, o, ws)
    # oracle: the stored new row is the 16-bit rounding of norm+RoPE(k) / v
    kn = orc.rope(orc.rmsnorm(k, kw, Hkv, hd, 1e-6), cos, sin, 1, Hkv, hd, pos)
    kc[pos] = _round(orc, kn, bf16).reshape(Hkv, hd)
    vc[pos] = v
    qn = orc.rope(orc.rmsnorm(q, qw, H, hd, 1e-6), cos, sin, 1, H, hd, pos)
    want = orc.attn_decode(qn, kc, vc, H, Hkv, pos, hd, max_seq, hd ** -0.5)
    assert_close(orc, to_np(o), want, what=f"decode tc hd={hd} G={G} pos={pos} bf16={bf16}")
    got_k = to_np(kcd).reshape(max_seq, Hkv, hd)
    assert_close(orc, got_k[pos], kc[pos], max_abs=2e-2 if bf16 else 2e-3, rel_l2=1e-2,
                 what="new k row")
    assert eb.device_error() == 0


def test_decode_tc_batched_bf16_many_chunks(eb, orc):
    """Batched bf16 decode, positions spread so some sequences need one chunk
    and some many; the per-(sequence, head) tickets must all reset."""
    import torch
    B, H, Hkv, hd, max_seq = 6, 16, 4, 128, 16384
    pos = np.array([5, 63, 64, 4095, 9000, 16383], np.int32)
    kc = orc.round_bf16(randn((B, max_seq, Hkv, hd), 1)).reshape(B, max_seq, Hkv, hd)
    vc = orc.round_bf16(randn((B, max_seq, Hkv, hd), 2)).reshape(B, max_seq, Hkv, hd)
    q = orc.round_bf16(randn((B, H, hd), 3)).reshape(B, H, hd)
    k = orc.round_bf16(randn((B, Hkv, hd), 4)).reshape(B, Hkv, hd)
    v = orc.round_bf16(randn((B, Hkv, hd), 5)).reshape(B, Hkv, hd)
    desc = eb.make_desc(H, Hkv, hd, max_seq, dtype_qkv=eb.EB_BF16, dtype_cache=eb.EB_BF16,
                        dtype_out=eb.EB_F32)
    layer = eb.make_layer()
    kcd, vcd = to_dev(kc, torch.bfloat16), to_dev(vc, torch.bfloat16)
    ws = eb.alloc_workspace(eb.attention_decode_workspace_bytes(desc, B, int(pos.max())))
    for _ in range(2):  # second call reuses the self-resetting tickets
        o = torch.full((B * H * hd,), float("nan"), device="cuda")
        eb.attention_decode_batched(desc, layer, B, to_dev(pos), int(pos.max()),
                                    to_dev(q, torch.bfloat16), to_dev(k, torch.bfloat16),
                                    to_dev(v, torch.bfloat16), kcd, vcd, max_seq * Hkv * hd, o, ws)
        kw, vw = kc.copy(), vc.copy()
        for b in range(B):
            kw[b, pos[b]] = k[b]
            vw[b, pos[b]] = v[b]
        want = orc.attn_decode_batched(q, kw, vw, pos, H, Hkv, hd, max_seq, max_seq * Hkv * hd,
                                       hd ** -0.5, nthreads=8)
        assert_close(orc, to_np(o), want, what="batched bf16")
