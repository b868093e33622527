"""GPU parity of the f32-cache prefill at head_dim 256, where the attention
kernel prepares q itself: each softmax thread reads its raw query row (f32,
f16 or bf16, contiguous or read in place from a fused q/k/v projection
output), applies RMSNorm(q_norm_w) and RoPE (crates/eyebrowse-nn/src/
attention.rs:62-76) and splits the result into f16 hi/lo planes (hi in
tensor memory, lo in shared memory) for the Qh.Kh + Qh.Kl + Ql.Kh product.
No q pass runs and the workspace holds only the K/V planes.

Checked against the oracle on the same input values (16-bit inputs are
rounded before the oracle sees them; the f32 cache stores the rows exactly)
at the north-star tolerance, with scale 1.0 and QK-norm as Gemma uses them,
full and partial rotary, and a ragged last query tile."""
import numpy as np
import pytest

from _util import assert_close, randn, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("H,Hkv,S,dt,qk_norm,rope_angles,fused_qkv,scale", [
    (8, 4, 700, "f16", True, 32, False, 1.0),     # Gemma-style: scale 1.0, partial rotary
    (8, 4, 515, "bf16", True, 32, True, 1.0),     # bf16 rows read in place (fused q/k/v)
    (4, 2, 333, "f32", False, None, True, None),  # f32 rows in place, full rotary, 1/sqrt(hd)
    (4, 1, 260, "f16", False, None, False, None),  # group of 4
])
def test_split_q_prefill_hd256(eb, orc, H, Hkv, S, dt, qk_norm, rope_angles, fused_qkv, scale):
    import torch
    hd = 256
    code = {"f16": eb.EB_F16, "bf16": eb.EB_BF16, "f32": eb.EB_F32}[dt]
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[dt]
    rnd = {"f16": orc.round_f16, "bf16": orc.round_bf16, "f32": lambda x: x}[dt]
    seed = S + H
    q = rnd(randn((S, H, hd), seed)).reshape(S, H, hd)
    k = rnd(randn((S, Hkv, hd), seed + 1)).reshape(S, Hkv, hd)
    v = rnd(randn((S, Hkv, hd), seed + 2)).reshape(S, Hkv, hd)
    qw = (1 + 0.1 * randn((hd,), seed + 3)).astype(np.float32) if qk_norm else None
    kw = (1 + 0.1 * randn((hd,), seed + 4)).astype(np.float32) if qk_norm else None
    cos, sin = eb.rope_tables(S, hd, 1e6, rope_angles)
    sc = hd ** -0.5 if scale is None else scale
    width = (H + 2 * Hkv) * hd
    if fused_qkv:
        qkv = np.concatenate([q.reshape(S, -1), k.reshape(S, -1), v.reshape(S, -1)], axis=1)
        buf = to_dev(qkv, tdt)
        qd, kd, vd = buf[:, :H * hd], buf[:, H * hd:(H + Hkv) * hd], buf[:, (H + Hkv) * hd:]
        strides = dict(q_stride=width, kv_stride=width)
    else:
        qd, kd, vd = to_dev(q, tdt), to_dev(k, tdt), to_dev(v, tdt)
        strides = {}
    dev = lambda w: None if w is None else to_dev(w)
    layer = eb.make_layer(dev(qw), dev(kw), None, to_dev(cos), to_dev(sin))
    desc = eb.make_desc(H, Hkv, hd, S, dtype_qkv=code, dtype_cache=eb.EB_F32,
                        dtype_out=eb.EB_F32, eps=1e-6, scale=sc, **strides)
    nb = eb.attention_prefill_workspace_bytes(desc, S)
    assert nb == 4 * S * Hkv * hd * 2  # the K/V hi/lo planes only: no q planes
    ws = eb.alloc_workspace(nb)
    kc = torch.zeros(S * Hkv * hd, device="cuda")
    vc = torch.zeros_like(kc)
    o = torch.full((S * H * hd,), float("nan"), device="cuda")
    eb.attention_prefill(desc, layer, S, qd, kd, vd, kc, vc, o, ws)
    want, _, _ = orc.attention_prefill(q, k, v, seq=S, h=H, hkv=Hkv, hd=hd, max_seq=S, scale=sc,
                                       eps=1e-6, q_norm_w=qw, k_norm_w=kw, cos=cos, sin=sin)
    assert_close(orc, to_np(o), want,
                 what=f"f32 cache hd256 q={dt} H={H} S={S} norm={qk_norm} qkv={fused_qkv}")
    assert eb.device_error() == 0
