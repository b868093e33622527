"""Generate golden attention fixtures with HuggingFace transformers.

The eyebrowse reference pins its model numerics against HF transformers
(golden/gen_golden.py, golden/gen_mistral_golden.py, golden/gen_gemma4_golden.py
in the reference repo). Its attention path cannot run here (Rust + wgpu), so
these fixtures take HF's own attention building blocks -- Qwen3RMSNorm,
the default and "proportional" (partial-rotary) RoPE tables,
apply_rotary_pos_emb and eager_attention_forward -- on seeded inputs, and
record the post-projection attention output. They pin the oracle's semantics:
half-split rotation, per-head RMSNorm, GQA head mapping (kv = h // group),
causal masking, scale, and partial rotary (pairs >= rope_angles pass through).
The sliding-window cases take their mask from HF's own
masking_utils.sliding_window_causal_mask_function (Gemma local layers,
Mistral sliding window); the reference itself has no sliding window yet.

Run from the repo root:  python tests/golden/gen_hf_golden.py [case ...]
Writes tests/golden/hf_attn_<case>.npz (a few KB each); all cases by default.
"""
from __future__ import annotations

import os
import types

import numpy as np
import torch
from transformers.masking_utils import causal_mask_function, sliding_window_causal_mask_function
from transformers.modeling_rope_utils import _compute_proportional_rope_parameters
from transformers.models.qwen3 import modeling_qwen3 as q3

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = {
    # Qwen3-style: per-head QK-RMSNorm, full rotary, scale 1/sqrt(hd)
    "qwen3": dict(seq=12, h=4, hkv=2, hd=32, theta=1e6, qk_norm=True, v_norm=False,
                  partial=1.0, scale=None, seed=0),
    # Llama/Mistral-style: no norms, full rotary
    "llama": dict(seq=9, h=6, hkv=2, hd=64, theta=5e5, qk_norm=False, v_norm=False,
                  partial=1.0, scale=None, seed=1),
    # Gemma-4-global-style: QK-norm, weightless V-norm, 25% partial rotary, scale 1.0
    "gemma": dict(seq=10, h=4, hkv=2, hd=64, theta=1e6, qk_norm=True, v_norm=True,
                  partial=0.25, scale=1.0, seed=2),
    # Gemma-local-style: QK-norm, weightless V-norm, full rotary (theta 1e4),
    # scale 1.0, sliding window of 7 keys
    "gemma_local": dict(seq=40, h=4, hkv=2, hd=64, theta=1e4, qk_norm=True, v_norm=True,
                        partial=1.0, scale=1.0, seed=3, window=7),
    # Mistral-style sliding window: no norms, full rotary, head_dim 128
    "mistral_swa": dict(seq=33, h=8, hkv=2, hd=128, theta=1e6, qk_norm=False, v_norm=False,
                        partial=1.0, scale=None, seed=4, window=16),
}
EPS = 1e-6


def rope_tables_hf(seq: int, hd: int, theta: float, partial: float):
    cfg = types.SimpleNamespace(
        head_dim=hd, hidden_size=hd, num_attention_heads=1,
        rope_parameters={"rope_theta": theta, "partial_rotary_factor": partial},
        standardize_rope_params=lambda: None)
    inv_freq, _ = _compute_proportional_rope_parameters(cfg, device="cpu")
    rope_angles = int(partial * hd // 2)
    pos = torch.arange(seq, dtype=torch.float32)
    freqs = pos[:, None] * inv_freq[None, :].float()
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin(), rope_angles


def make_case(name: str, c: dict) -> None:
    g = torch.Generator().manual_seed(c["seed"])
    seq, h, hkv, hd = c["seq"], c["h"], c["hkv"], c["hd"]
    q = torch.randn(seq, h, hd, generator=g)
    k = torch.randn(seq, hkv, hd, generator=g)
    v = torch.randn(seq, hkv, hd, generator=g)
    qw = (1.0 + 0.1 * torch.randn(hd, generator=g)) if c["qk_norm"] else None
    kw = (1.0 + 0.1 * torch.randn(hd, generator=g)) if c["qk_norm"] else None
    scale = c["scale"] if c["scale"] is not None else hd ** -0.5

    def norm(x, w):
        m = q3.Qwen3RMSNorm(hd, eps=EPS)
        with torch.no_grad():
            m.weight.copy_(w)
        return m(x)

    qn = norm(q, qw) if qw is not None else q
    kn = norm(k, kw) if kw is not None else k
    vn = norm(v, torch.ones(hd)) if c["v_norm"] else v

    cos, sin, rope_angles = rope_tables_hf(seq, hd, c["theta"], c["partial"])
    # [1, heads, seq, hd] as HF expects
    qh = qn.permute(1, 0, 2)[None]
    kh = kn.permute(1, 0, 2)[None]
    vh = vn.permute(1, 0, 2)[None]
    qr, kr = q3.apply_rotary_pos_emb(qh, kh, cos[None], sin[None])
    window = c.get("window", 0)
    fn = sliding_window_causal_mask_function(window) if window else causal_mask_function
    idx = torch.arange(seq)
    allowed = fn(torch.tensor(0), torch.tensor(0), idx[:, None], idx[None, :])
    allowed = allowed.expand(seq, seq)
    mask = torch.zeros(seq, seq).masked_fill(~allowed, float("-inf"))[None, None]
    module = types.SimpleNamespace(num_key_value_groups=h // hkv, training=False)
    out, _ = q3.eager_attention_forward(module, qr, kr, vh, mask, scaling=scale)
    o = out[0]  # [seq, h, hd] after the transpose inside eager_attention_forward
    k_cache = kr[0].permute(1, 0, 2)  # post-RoPE keys, [seq, hkv, hd]
    v_cache = vh[0].permute(1, 0, 2)

    arrs = dict(q=q, k=k, v=v, o=o, k_cache=k_cache, v_cache=v_cache)
    if qw is not None:
        arrs.update(q_norm_w=qw, k_norm_w=kw)
    meta = np.array([seq, h, hkv, hd, rope_angles], dtype=np.int64)
    np.savez_compressed(
        os.path.join(HERE, f"hf_attn_{name}.npz"),
        meta=meta, theta=np.float32(c["theta"]), scale=np.float32(scale),
        eps=np.float32(EPS), v_norm=np.int64(int(c["v_norm"])), window=np.int64(window),
        **{k_: t.detach().contiguous().numpy().astype(np.float32) for k_, t in arrs.items()})
    print(f"wrote hf_attn_{name}.npz (seq={seq} h={h} hkv={hkv} hd={hd} "
          f"rope_angles={rope_angles} scale={scale:.5f} window={window})")


if __name__ == "__main__":
    torch.set_num_threads(1)
    import sys
    for n in (sys.argv[1:] or list(CASES)):
        make_case(n, CASES[n])
