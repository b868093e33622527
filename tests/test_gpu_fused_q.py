"""GPU parity of the prefill with the query transform fused into the attention
kernel: when q already has the cache's 16-bit type, each query tile is
TMA-loaded raw and its softmax warpgroup applies RMSNorm(q_norm_w) and RoPE
in shared memory (crates/eyebrowse-nn/src/attention.rs:62-76) before the
tensor cores read it; no row-prep pass and no q staging.

Covers head dims 64/128/256, f16 and bf16, with and without QK-norm, full and
partial rotary, contiguous q and q read in place from a fused q/k/v
projection output (row stride (H + 2 Hkv) hd), the two-tile (GQA pair) and
one-tile kernels, and a ragged last query tile. Checked against the oracle
(the reference's attention order; K/V cache rows rounded as stored) at the
north-star tolerance (bf16: the tensor cores take q and P in bf16, ~1e-3
relative, as in the other bf16 tests), and against the row-prep path on the
same values: f32 q holding the same 16-bit values still goes through the
row pass, and the two outputs agree to within the 16-bit rounding of q."""
import numpy as np
import pytest

from _util import assert_close, randn, to_dev, to_np

pytestmark = pytest.mark.gpu


def _run(eb, orc, hd, H, Hkv, S, dt, qk_norm, rope_angles, fused_qkv, seed):
    import torch
    code = eb.EB_F16 if dt == "f16" else eb.EB_BF16
    tdt = torch.float16 if dt == "f16" else torch.bfloat16
    rnd = orc.round_f16 if dt == "f16" else orc.round_bf16
    q = rnd(randn((S, H, hd), seed, 0.5)).reshape(S, H, hd)
    k = rnd(randn((S, Hkv, hd), seed + 1, 0.5)).reshape(S, Hkv, hd)
    v = rnd(randn((S, Hkv, hd), seed + 2)).reshape(S, Hkv, hd)
    qw = (1 + 0.1 * randn((hd,), seed + 3)).astype(np.float32) if qk_norm else None
    kw = (1 + 0.1 * randn((hd,), seed + 4)).astype(np.float32) if qk_norm else None
    cos, sin = eb.rope_tables(S, hd, 1e6, rope_angles)
    dev = lambda w: None if w is None else to_dev(w)
    width = (H + 2 * Hkv) * hd
    if fused_qkv:
        qkv = np.concatenate([q.reshape(S, -1), k.reshape(S, -1), v.reshape(S, -1)], axis=1)
        buf = to_dev(qkv, tdt)
        qd, kd, vd = buf[:, :H * hd], buf[:, H * hd:(H + Hkv) * hd], buf[:, (H + Hkv) * hd:]
        strides = dict(q_stride=width, kv_stride=width)
    else:
        qd, kd, vd = to_dev(q, tdt), to_dev(k, tdt), to_dev(v, tdt)
        strides = {}
    layer = eb.make_layer(dev(qw), dev(kw), None, to_dev(cos), to_dev(sin))

    def prefill(q_in, k_in, v_in, desc_code, st):
        desc = eb.make_desc(H, Hkv, hd, S, dtype_qkv=desc_code, dtype_cache=code,
                            dtype_out=eb.EB_F32, eps=1e-6, **st)
        kc = torch.zeros(S * Hkv * hd, device="cuda", dtype=tdt)
        vc = torch.zeros_like(kc)
        o = torch.full((S * H * hd,), float("nan"), device="cuda")
        nb = eb.attention_prefill_workspace_bytes(desc, S)
        ws = eb.alloc_workspace(nb) if nb else None
        eb.attention_prefill(desc, layer, S, q_in, k_in, v_in, kc, vc, o, ws)
        return to_np(o), nb

    got, nb = prefill(qd, kd, vd, code, strides)
    assert nb == 0  # the fused path stages nothing
    # the row-prep path on the same values: f32 q, k and v (contiguous)
    f32 = lambda x: x.float().contiguous()
    ref_prep, nb32 = prefill(f32(qd), f32(kd), f32(vd), eb.EB_F32, {})
    assert nb32 > 0
    want, _, _ = orc.attention_prefill(
        q, k, v, seq=S, h=H, hkv=Hkv, hd=hd, max_seq=S, scale=hd ** -0.5, eps=1e-6,
        q_norm_w=qw, k_norm_w=kw, cos=cos, sin=sin,
        cache_round=orc.F16 if dt == "f16" else orc.BF16)
    return got, want, ref_prep


@pytest.mark.parametrize("hd,H,Hkv,S,dt,qk_norm,rope_angles,fused_qkv", [
    (128, 32, 8, 1100, "f16", False, None, False),   # config 3's layout, ragged tile
    (128, 16, 8, 700, "f16", True, None, True),      # Qwen3-style QK-norm, fused q/k/v rows
    (128, 8, 2, 515, "bf16", True, None, False),     # one-tile kernel (small grid)
    (64, 32, 8, 900, "f16", True, None, True),
    (256, 8, 4, 600, "f16", True, 32, False),        # Gemma-style partial rotary
    (256, 4, 2, 333, "bf16", False, 16, True),
    (128, 6, 2, 400, "f16", True, 8, False),         # odd group: one-tile kernel
])
def test_fused_q_prefill(eb, orc, hd, H, Hkv, S, dt, qk_norm, rope_angles, fused_qkv):
    got, want, ref_prep = _run(eb, orc, hd, H, Hkv, S, dt, qk_norm, rope_angles, fused_qkv,
                               seed=hd + H + S)
    tol = dict(max_abs=8e-3, rel_l2=4e-3) if dt == "bf16" else {}
    what = f"fused q hd={hd} H={H} S={S} {dt} norm={qk_norm} ra={rope_angles} qkv={fused_qkv}"
    assert_close(orc, got, want, what=what + " vs oracle", **tol)
    assert_close(orc, got, ref_prep, what=what + " vs row-prep path", **tol)
    assert eb.device_error() == 0
