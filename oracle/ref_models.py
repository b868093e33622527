"""CPU oracle of the reference's model driver for the architectures its golden
tests cover (Qwen3, Mistral/Llama, dense Gemma 4): TEST INFRASTRUCTURE ONLY,
used by tests/ to check eyebrowse_b200.decoder.DecoderModel against the
reference's own HF-generated fixtures; never by the library.

A numpy restatement of crates/eyebrowse-models:
  config      crates/eyebrowse-load/src/config.rs:59-91 (head_dim defaults to
              hidden / heads, theta from rope_theta or rope_parameters)
  driver      model.rs:68-130: embed (f16 table, x sqrt(hidden) for Gemma),
              blocks, final RMSNorm of the last row, LM head (lm_head.weight
              or the tied embedding), Gemma's softcap cap * tanh(x / cap)
  standard    decoder.rs:34-55, :57-160: x += Attn(RMSNorm(x));
              x += down(silu(gate(h)) * up(h)) with h = RMSNorm(x);
              QK-norm only for Qwen3; scale 1/sqrt(head_dim)
  Gemma 4     gemma4.rs:72-101, :104-263: sandwich norms
              x2 = x + post_attn_ln(Attn(input_ln(x))),
              x3 = x2 + post_ff_ln(GeGLU-MLP(pre_ff_ln(x2))), x_out = x3 * layer_scalar;
              per-layer head_dim (head_dim for sliding layers, global_head_dim
              for full layers) and RoPE (sliding: full rotary at
              rope_parameters.sliding_attention.rope_theta; full: the first
              floor(partial_rotary_factor * global_head_dim / 2) pairs at
              full_attention.rope_theta); QK-norm, weightless V-norm, scale 1.0
with the reference's element-wise kernels (crates/eyebrowse-kernels/src/
ops.rs:6-36: silu = g / (1 + exp(-g)); gelu = 0.5 g (1 + tanh(0.7978845608028654
(g + 0.044715 g^3)))), linear_f16w as f32 x @ (f16-valued W)^T, and the
attention (norms, RoPE, cache write, prefill, decode) from the C oracle.

Sliding layers pass their window to the attention oracle (HF's semantics;
the reference itself does not window, README.md:25); the fixtures' prompts
are shorter than the window, where both agree.
"""
from __future__ import annotations

import json
import math

import numpy as np

from . import oracle as orc


def load_fixture(path: str):
    """(weights {name: f32 array}, config dict, input ids, golden last logits)."""
    z = np.load(path)
    cfg = json.loads(bytes(z["__config__"]).decode())
    w = {k: z[k].astype(np.float32) for k in z.files if not k.startswith("__")}
    return w, cfg, [int(i) for i in z["__input_ids__"]], z["__last_logits__"].astype(np.float32)


def model_spec(cfg: dict) -> dict:
    """The per-layer attention geometry the reference's loaders derive from
    config.json (decoder.rs:69-95, gemma4.rs:122-205)."""
    arch = cfg.get("model_type", "unknown")
    H = cfg["num_attention_heads"]
    Hkv = cfg.get("num_key_value_heads") or H
    hd = cfg.get("head_dim") or cfg["hidden_size"] // H
    L = cfg["num_hidden_layers"]
    rp = cfg.get("rope_parameters") or {}
    gemma = arch.startswith("gemma4")
    layers = []
    if gemma:
        ghd = cfg["global_head_dim"]
        loc, glob = rp["sliding_attention"], rp["full_attention"]
        angles = int(math.floor(glob["partial_rotary_factor"] * ghd / 2.0))
        for l in range(L):
            full = cfg["layer_types"][l] == "full_attention"
            layers.append(dict(
                head_dim=ghd if full else hd,
                theta=float(np.float32(glob["rope_theta"] if full else loc["rope_theta"])),
                rope_angles=angles if full else (ghd if full else hd) // 2,
                window=0 if full else int(cfg.get("sliding_window") or 0),
                qk_norm=True, v_norm=True, scale=1.0))
    else:
        theta = cfg.get("rope_theta") or rp.get("rope_theta") or 10000.0
        for _ in range(L):
            layers.append(dict(head_dim=hd, theta=float(np.float32(theta)), rope_angles=hd // 2,
                               window=0, qk_norm=arch == "qwen3", v_norm=False,
                               scale=float(np.float32(1.0) / np.sqrt(np.float32(hd)))))
    cap = cfg.get("final_logit_softcapping") or 0.0
    return dict(arch=arch, gemma=gemma, hidden=cfg["hidden_size"], heads=H, kv_heads=Hkv,
                layers=layers, eps=float(np.float32(cfg["rms_norm_eps"])),
                embed_scale=float(np.sqrt(np.float32(cfg["hidden_size"]))) if gemma else None,
                softcap=float(np.float32(cap)) if cap else None)


class RefOracleModel:
    def __init__(self, weights: dict, cfg: dict, max_seq: int):
        self.w, self.s, self.max_seq = weights, model_spec(cfg), max_seq
        self.tables = [orc.rope_tables(max_seq, ly["head_dim"], ly["theta"], ly["rope_angles"])
                       for ly in self.s["layers"]]
        self.reset()

    def reset(self):
        s = self.s
        self.kc = [np.zeros(self.max_seq * s["kv_heads"] * ly["head_dim"], np.float32)
                   for ly in s["layers"]]
        self.vc = [np.zeros_like(c) for c in self.kc]

    def _norm(self, x, w):
        rows, dim = x.shape
        return orc.rmsnorm(x, w, rows, dim, self.s["eps"]).reshape(rows, dim)

    def _attention(self, i, h, base_pos):
        s, w, ly = self.s, self.w, self.s["layers"][i]
        p = f"model.layers.{i}"
        H, Hkv, hd = s["heads"], s["kv_heads"], ly["head_dim"]
        rows = h.shape[0]
        q = h @ w[f"{p}.self_attn.q_proj.weight"].T
        k = h @ w[f"{p}.self_attn.k_proj.weight"].T
        v = h @ w[f"{p}.self_attn.v_proj.weight"].T
        cos, sin = self.tables[i]
        common = dict(h=H, hkv=Hkv, hd=hd, max_seq=self.max_seq, scale=ly["scale"],
                      eps=s["eps"], cos=cos, sin=sin, window=ly["window"],
                      q_norm_w=w[f"{p}.self_attn.q_norm.weight"] if ly["qk_norm"] else None,
                      k_norm_w=w[f"{p}.self_attn.k_norm.weight"] if ly["qk_norm"] else None,
                      v_norm_w=np.ones(hd, np.float32) if ly["v_norm"] else None)
        if base_pos == 0 and rows > 1:  # attention.rs:40: a fresh multi-row prompt
            o, self.kc[i], self.vc[i] = orc.attention_prefill(
                q, k, v, seq=rows, kcache=self.kc[i], vcache=self.vc[i], **common)
        else:  # one decode step over the first row
            o, self.kc[i], self.vc[i] = orc.attention_decode(
                q[:1], k[:1], v[:1], pos=base_pos, kcache=self.kc[i], vcache=self.vc[i],
                **common)
            rows = 1
        return o.reshape(rows, H * hd) @ w[f"{p}.self_attn.o_proj.weight"].T

    def _mlp(self, p, h):
        w = self.w
        g = h @ w[f"{p}.mlp.gate_proj.weight"].T
        u = h @ w[f"{p}.mlp.up_proj.weight"].T
        if self.s["gemma"]:
            a = np.float32(0.5) * g * (np.float32(1) + np.tanh(
                np.float32(0.7978845608028654) * (g + np.float32(0.044715) * g * g * g)))
        else:
            a = g / (np.float32(1) + np.exp(-g))
        return (a * u).astype(np.float32) @ w[f"{p}.mlp.down_proj.weight"].T

    def logits(self, ids, base_pos: int) -> np.ndarray:
        """[vocab] logits of the last row after ids at positions base_pos..
        (updates the caches); softcapped for Gemma (model.rs:119-125)."""
        s, w = self.s, self.w
        x = w["model.embed_tokens.weight"][np.asarray(ids)].astype(np.float32)
        if s["embed_scale"] is not None:
            x = x * np.float32(s["embed_scale"])
        for i in range(len(s["layers"])):
            p = f"model.layers.{i}"
            if s["gemma"]:
                a = self._norm(self._attention(i, self._norm(x, w[f"{p}.input_layernorm.weight"]),
                                               base_pos), w[f"{p}.post_attention_layernorm.weight"])
                x2 = x[: a.shape[0]] + a
                m = self._norm(self._mlp(p, self._norm(x2, w[f"{p}.pre_feedforward_layernorm.weight"])),
                               w[f"{p}.post_feedforward_layernorm.weight"])
                x = (x2 + m) * np.float32(w[f"{p}.layer_scalar"][0])
            else:
                a = self._attention(i, self._norm(x, w[f"{p}.input_layernorm.weight"]), base_pos)
                x2 = x[: a.shape[0]] + a
                x = x2 + self._mlp(p, self._norm(x2, w[f"{p}.post_attention_layernorm.weight"]))
        xn = self._norm(x[-1:], w["model.norm.weight"])
        head = w.get("lm_head.weight", w["model.embed_tokens.weight"])
        out = (xn @ head.T)[0].astype(np.float32)
        if s["softcap"]:
            cap = np.float32(s["softcap"])
            out = (cap * np.tanh(out / cap)).astype(np.float32)
        return out
