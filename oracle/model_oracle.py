"""CPU oracle of the greedy-decode model: TEST INFRASTRUCTURE ONLY (used by
tests/ to check eyebrowse_b200.qwen3.GreedyModel; never by the library).

A numpy restatement of the reference decoder driver and standard block
(crates/eyebrowse-models/src/model.rs:82-175, decoder.rs:34-55):

    x = embed[ids]; per layer: x += Attention(RMSNorm(x)); x += MLP(RMSNorm(x))
    next = argmax(RMSNorm(x_last) @ embed^T)

with the layer RMSNorm restated from crates/eyebrowse-kernels/src/rmsnorm.rs
(via the C oracle), linear_f16w as f32 x (f16-valued W)^T
(crates/eyebrowse-kernels/src/matmul.rs:84-144), SwiGLU as
g / (1 + exp(-g)) * up (crates/eyebrowse-kernels/src/ops.rs:6-20), and the
attention -- QK-norm, RoPE, cache write, prefill and decode -- from the C
oracle's attention_prefill / attention_decode (eyebrowse-nn attention.rs:
49-185). The argmax takes the first maximum (the reference's WGSL argmax,
crates/eyebrowse-kernels/src/sampling.rs:6-40, differs only on exact ties).
"""
from __future__ import annotations

import numpy as np

from . import oracle as orc


class OracleModel:
    def __init__(self, weights: dict, max_seq: int, geometry: dict):
        self.w, self.g, self.max_seq = weights, geometry, max_seq
        hd = geometry["head_dim"]
        self.cos, self.sin = orc.rope_tables(max_seq, hd, geometry["theta"])
        self.reset()

    def reset(self):
        g = self.g
        n = self.max_seq * g["kv_heads"] * g["head_dim"]
        self.kc = [np.zeros(n, np.float32) for _ in range(g["layers"])]
        self.vc = [np.zeros(n, np.float32) for _ in range(g["layers"])]

    def _norm(self, x, w):
        rows, dim = x.shape
        return orc.rmsnorm(x, w, rows, dim, self.g["eps"]).reshape(rows, dim)

    def _forward(self, ids, base_pos: int):
        g, w = self.g, self.w
        rows = len(ids)
        H, Hkv, hd = g["heads"], g["kv_heads"], g["head_dim"]
        x = w["model.embed_tokens.weight"][np.asarray(ids)].astype(np.float32)
        for i in range(g["layers"]):
            p = f"model.layers.{i}"
            h = self._norm(x, w[f"{p}.input_layernorm.weight"])
            q = h @ w[f"{p}.self_attn.q_proj.weight"].T
            k = h @ w[f"{p}.self_attn.k_proj.weight"].T
            v = h @ w[f"{p}.self_attn.v_proj.weight"].T
            common = dict(h=H, hkv=Hkv, hd=hd, max_seq=self.max_seq, scale=hd ** -0.5,
                          eps=g["eps"], q_norm_w=w[f"{p}.self_attn.q_norm.weight"],
                          k_norm_w=w[f"{p}.self_attn.k_norm.weight"], cos=self.cos,
                          sin=self.sin)
            if base_pos == 0:
                o, self.kc[i], self.vc[i] = orc.attention_prefill(
                    q, k, v, seq=rows, kcache=self.kc[i], vcache=self.vc[i], **common)
            else:
                o, self.kc[i], self.vc[i] = orc.attention_decode(
                    q, k, v, pos=base_pos, kcache=self.kc[i], vcache=self.vc[i], **common)
            x = x + o.reshape(rows, H * hd) @ w[f"{p}.self_attn.o_proj.weight"].T
            h2 = self._norm(x, w[f"{p}.post_attention_layernorm.weight"])
            gt = h2 @ w[f"{p}.mlp.gate_proj.weight"].T
            up = h2 @ w[f"{p}.mlp.up_proj.weight"].T
            act = (gt / (np.float32(1) + np.exp(-gt))) * up
            x = x + act @ w[f"{p}.mlp.down_proj.weight"].T
        return self._norm(x[-1:], w["model.norm.weight"])

    def logits(self, ids, base_pos: int) -> np.ndarray:
        """[vocab] logits after ids at positions base_pos.. (updates the caches)."""
        return (self._forward(ids, base_pos) @ self.w["model.embed_tokens.weight"].T)[0]

    def next_id(self, ids, base_pos: int) -> int:
        return int(np.argmax(self.logits(ids, base_pos)))

    def generate(self, prompt, n_new: int) -> list:
        self.reset()
        out = [self.next_id(list(prompt), 0)]
        pos = len(prompt)
        while len(out) < n_new:
            out.append(self.next_id([out[-1]], pos))
            pos += 1
        return out
