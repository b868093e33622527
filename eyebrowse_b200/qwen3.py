"""Greedy decoding of a random-init Qwen3-0.6B-geometry decoder on the B200
attention path: the harness for the token-id gate (identical greedy ids to
the reference model on seeded prompts).

The model follows the reference driver and block exactly
(crates/eyebrowse-models/src/model.rs:82-175, decoder.rs:34-55):

    x = embed[ids]                                  (f16 table -> f32)
    per layer:  h = RMSNorm(x) ; x = x + Attention(h)
                h = RMSNorm(x) ; x = x + down(silu(gate(h)) * up(h))
    logits = RMSNorm(x_last) @ embed^T              (tied LM head)
    next id = argmax(logits)

Linear weights are f16 values used in f32 arithmetic (linear_f16w,
crates/eyebrowse-kernels/src/matmul.rs:84-144, HF layout [out, in]); norm
weights are f32. Attention is eyebrowse-nn's Attention (QK-RMSNorm per head,
RoPE theta 1e6, GQA 16/8, head_dim 128).

What runs where: every layer's attention -- QK-norm, RoPE, the KV-cache
write, the causal prefill over the prompt and each single-token decode step
-- goes through this library's C ABI (eb_attention_prefill /
eb_attention_decode on f32 caches, the tensor-core path); every projection
through eb_linear_f16w: one fused q/k/v GEMM whose output rows the attention
reads in place (q_stride = kv_stride = the fused width), o_proj, one fused
gate/up GEMM, down_proj and the tied LM head; the block and final RMSNorms
through eb_rmsnorm. The embedding gather, the residual adds, SiLU * up and
the argmax are plain torch element-wise operations.
"""
from __future__ import annotations

import numpy as np

# Qwen3-0.6B geometry (crates/eyebrowse-load/tests/load.rs:26-36).
GEOMETRY = dict(hidden=1024, layers=28, heads=16, kv_heads=8, head_dim=128, inter=3072,
                vocab=151936, theta=1e6, eps=1e-6)


def _f16(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float16).astype(np.float32)


def make_weights(seed: int = 0, geometry: dict = GEOMETRY, std: float = 0.02) -> dict:
    """Seeded random-init weights under HF names: linear and embedding weights
    N(0, std) rounded to f16 (as the reference stores them), norm weights
    1 + 0.1 N(0, 1) in f32. Deterministic for a given seed (numpy PCG64)."""
    g = geometry
    rng = np.random.default_rng(seed)
    H, D, hd, inter = g["heads"], g["hidden"], g["head_dim"], g["inter"]
    Hkv = g["kv_heads"]

    def lin(out_f, in_f):
        return _f16(rng.standard_normal((out_f, in_f), dtype=np.float32) * np.float32(std))

    def norm(n):
        return (1 + 0.1 * rng.standard_normal(n, dtype=np.float32)).astype(np.float32)

    w = {"model.embed_tokens.weight": lin(g["vocab"], D)}
    for i in range(g["layers"]):
        p = f"model.layers.{i}"
        w[f"{p}.input_layernorm.weight"] = norm(D)
        w[f"{p}.self_attn.q_proj.weight"] = lin(H * hd, D)
        w[f"{p}.self_attn.k_proj.weight"] = lin(Hkv * hd, D)
        w[f"{p}.self_attn.v_proj.weight"] = lin(Hkv * hd, D)
        w[f"{p}.self_attn.o_proj.weight"] = lin(D, H * hd)
        w[f"{p}.self_attn.q_norm.weight"] = norm(hd)
        w[f"{p}.self_attn.k_norm.weight"] = norm(hd)
        w[f"{p}.post_attention_layernorm.weight"] = norm(D)
        w[f"{p}.mlp.gate_proj.weight"] = lin(inter, D)
        w[f"{p}.mlp.up_proj.weight"] = lin(inter, D)
        w[f"{p}.mlp.down_proj.weight"] = lin(D, inter)
    w["model.norm.weight"] = norm(D)
    return w


def make_prompts(seed: int, n_prompts: int, length: int, vocab: int = GEOMETRY["vocab"]):
    """Seeded prompts of random token ids."""
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, size=length).astype(np.int64).tolist()
            for _ in range(n_prompts)]


class GreedyModel:
    """The model on one GPU. `weights` as from make_weights (numpy, HF names)."""

    def __init__(self, weights: dict, max_seq: int, geometry: dict = GEOMETRY):
        import torch

        import eyebrowse_b200 as eb
        self.eb, self.g, self.max_seq = eb, geometry, max_seq
        g = geometry
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        f16 = lambda *names: dev(np.concatenate([weights[n] for n in names]).astype(np.float16))
        H, Hkv, hd, D, inter = g["heads"], g["kv_heads"], g["head_dim"], g["hidden"], g["inter"]
        self.qkv_w = (H + 2 * Hkv) * hd  # fused q/k/v output width
        self.norms = {k: dev(v) for k, v in weights.items() if k.endswith("norm.weight")}
        self.embed = dev(weights["model.embed_tokens.weight"])      # f32 rows for the gather
        self.lm_head = f16("model.embed_tokens.weight")             # tied, f16 [vocab, hidden]
        self.lin = []
        for i in range(g["layers"]):
            p = f"model.layers.{i}"
            self.lin.append(dict(
                qkv=f16(f"{p}.self_attn.q_proj.weight", f"{p}.self_attn.k_proj.weight",
                        f"{p}.self_attn.v_proj.weight"),
                o=f16(f"{p}.self_attn.o_proj.weight"),
                gate_up=f16(f"{p}.mlp.gate_proj.weight", f"{p}.mlp.up_proj.weight"),
                down=f16(f"{p}.mlp.down_proj.weight")))
        cos, sin = eb.rope_tables(max_seq, hd, g["theta"])
        self.cos, self.sin = dev(cos), dev(sin)
        self.desc = eb.make_desc(H, Hkv, hd, max_seq, eps=g["eps"], q_stride=self.qkv_w,
                                 kv_stride=self.qkv_w)
        self.layers = [
            eb.make_layer(self.norms[f"model.layers.{i}.self_attn.q_norm.weight"],
                          self.norms[f"model.layers.{i}.self_attn.k_norm.weight"], None,
                          self.cos, self.sin) for i in range(g["layers"])]
        self.ws_prefill = eb.alloc_workspace(eb.attention_prefill_workspace_bytes(self.desc,
                                                                                  max_seq))
        self.ws_decode = eb.alloc_workspace(eb.attention_decode_workspace_bytes(self.desc, 1,
                                                                                max_seq - 1))
        nb = max(eb.linear_f16w_workspace_bytes(max_seq, k, n)
                 for k, n in ((D, self.qkv_w), (H * hd, D), (D, 2 * inter), (inter, D)))
        self.ws_linear = eb.alloc_workspace(nb) if nb else None
        self.reset()

    def reset(self):
        import torch
        g = self.g
        shape = (self.max_seq, g["kv_heads"], g["head_dim"])
        self.kc = [torch.zeros(shape, device="cuda") for _ in range(g["layers"])]
        self.vc = [torch.zeros(shape, device="cuda") for _ in range(g["layers"])]

    def _norm(self, x, w):
        import torch
        out = torch.empty_like(x)
        self.eb.rmsnorm(x, w, out, x.shape[0], x.shape[1], self.g["eps"])
        return out

    def _linear(self, x, w):
        """eb_linear_f16w: x [rows, in] f32 @ w [out, in]^T (f16) -> [rows, out] f32."""
        import torch
        rows, in_f = x.shape
        out_f = w.shape[0]
        y = torch.empty(rows, out_f, device="cuda")
        self.eb.linear_f16w(x, w, y, rows, in_f, out_f, self.ws_linear)
        return y

    def _forward(self, ids, base_pos: int):
        """Hidden state of the last row after the final norm; ids at positions
        base_pos.. (a prompt at 0, or one token at base_pos)."""
        import torch
        g, N, eb = self.g, self.norms, self.eb
        rows = len(ids)
        H, Hkv, hd, inter = g["heads"], g["kv_heads"], g["head_dim"], g["inter"]
        x = self.embed[torch.tensor(ids, device="cuda")].contiguous()
        o = torch.empty(rows, H, hd, device="cuda")
        for i in range(g["layers"]):
            p, L = f"model.layers.{i}", self.lin[i]
            h = self._norm(x, N[f"{p}.input_layernorm.weight"])
            qkv = self._linear(h, L["qkv"])  # rows of [q | k | v], read in place
            q, k, v = qkv[:, :H * hd], qkv[:, H * hd:(H + Hkv) * hd], qkv[:, (H + Hkv) * hd:]
            if base_pos == 0:
                eb.attention_prefill(self.desc, self.layers[i], rows, q, k, v, self.kc[i],
                                     self.vc[i], o, self.ws_prefill)
            else:
                assert rows == 1
                eb.attention_decode(self.desc, self.layers[i], base_pos, q, k, v, self.kc[i],
                                    self.vc[i], o, self.ws_decode)
            x = x + self._linear(o.view(rows, H * hd), L["o"])
            h2 = self._norm(x, N[f"{p}.post_attention_layernorm.weight"])
            gu = self._linear(h2, L["gate_up"])
            gt, up = gu[:, :inter], gu[:, inter:]
            x = x + self._linear(((gt / (1.0 + torch.exp(-gt))) * up).contiguous(), L["down"])
        return self._norm(x[-1:].contiguous(), N["model.norm.weight"])

    def logits(self, ids, base_pos: int):
        """[vocab] logits after ids at positions base_pos.. (updates the caches)."""
        return self._linear(self._forward(ids, base_pos), self.lm_head)[0]

    def next_id(self, ids, base_pos: int) -> int:
        import torch
        return int(torch.argmax(self.logits(ids, base_pos)).item())

    def generate(self, prompt, n_new: int) -> list:
        """Greedy: prefill the prompt, then decode one token at a time."""
        if len(prompt) + n_new > self.max_seq:
            raise ValueError("prompt + n_new exceeds max_seq")
        self.reset()
        out = [self.next_id(list(prompt), 0)]
        pos = len(prompt)
        while len(out) < n_new:
            out.append(self.next_id([out[-1]], pos))
            pos += 1
        return out
