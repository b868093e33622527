"""Decoder models built from a HuggingFace config.json and weights, with every
attention on this library: the reference's model families (Qwen3,
Mistral/Llama, dense Gemma 4) as eyebrowse-models builds them, so a model
the reference loads runs here with its attention on the B200 path.

The structure follows the reference loaders and driver:
  config          crates/eyebrowse-load/src/config.rs:59-91
  driver          crates/eyebrowse-models/src/model.rs:68-130 (embedding of the
                  f16 table, x sqrt(hidden) for Gemma; final RMSNorm of the last
                  row; LM head = lm_head.weight or the tied embedding; Gemma's
                  softcap cap * tanh(x / cap))
  standard block  decoder.rs:34-55 (pre-norm attention and SwiGLU MLP; QK-norm
                  for Qwen3 only; scale 1/sqrt(head_dim))
  Gemma 4 block   gemma4.rs:72-101, :104-263 (sandwich norms, GeGLU, per-layer
                  residual scalar; per-layer head_dim and RoPE: sliding layers
                  full rotary at head_dim, full layers the first
                  floor(partial_rotary_factor * global_head_dim / 2) pairs at
                  global_head_dim; QK-norm, weightless V-norm, scale 1.0)

What runs where: each layer's attention -- q/k/v RMSNorm, RoPE, the KV-cache
write, causal prefill and single-token decode -- through eb_attention_prefill
/ eb_attention_decode (any head_dim: 64/128/256 on the tensor cores, others
such as Gemma 4 tiny's 16 and 32 on the SIMT kernel); every projection through
eb_linear_f16w (fused q/k/v read in place by the attention, fused gate/up);
the RMSNorms through eb_rmsnorm. The embedding gather, residual adds, the
gated activations, the residual scalar and the softcap are torch
element-wise operations. Sliding-window layers get their window in the
descriptor (HF's semantics; the reference itself does not window yet).
"""
from __future__ import annotations

import math

import numpy as np


def spec_from_config(cfg: dict) -> dict:
    """Per-layer attention geometry as the reference's loaders derive it."""
    arch = cfg.get("model_type", "unknown")
    H = cfg["num_attention_heads"]
    Hkv = cfg.get("num_key_value_heads") or H
    hd = cfg.get("head_dim") or cfg["hidden_size"] // H
    n_layers = cfg["num_hidden_layers"]
    rp = cfg.get("rope_parameters") or {}
    gemma = arch.startswith("gemma4")
    layers = []
    if gemma:
        if cfg.get("hidden_size_per_layer_input") or cfg.get("num_experts") or \
                cfg.get("enable_moe_block"):
            raise ValueError("gemma4: per-layer inputs and MoE are not supported (as in the "
                             "reference loader, gemma4.rs:108-118)")
        ghd = cfg["global_head_dim"]
        loc, glob = rp["sliding_attention"], rp["full_attention"]
        angles = int(math.floor(glob["partial_rotary_factor"] * ghd / 2.0))
        for l in range(n_layers):
            full = cfg["layer_types"][l] == "full_attention"
            d = ghd if full else hd
            layers.append(dict(head_dim=d, theta=glob["rope_theta"] if full else loc["rope_theta"],
                               rope_angles=angles if full else d // 2,
                               window=0 if full else int(cfg.get("sliding_window") or 0),
                               qk_norm=True, v_norm=True, scale=1.0))
    else:
        theta = cfg.get("rope_theta") or rp.get("rope_theta") or 10000.0
        for _ in range(n_layers):
            layers.append(dict(head_dim=hd, theta=theta, rope_angles=hd // 2, window=0,
                               qk_norm=arch == "qwen3", v_norm=False,
                               scale=float(np.float32(1.0) / np.sqrt(np.float32(hd)))))
    cap = cfg.get("final_logit_softcapping") or 0.0
    return dict(arch=arch, gemma=gemma, hidden=cfg["hidden_size"], heads=H, kv_heads=Hkv,
                inter=cfg["intermediate_size"], vocab=cfg["vocab_size"], layers=layers,
                eps=cfg["rms_norm_eps"],
                embed_scale=float(np.sqrt(np.float32(cfg["hidden_size"]))) if gemma else None,
                softcap=float(cap) if cap else None)


class DecoderModel:
    """A decoder on one GPU. `weights`: {HF tensor name: numpy array} (linear
    and embedding weights f16-valued, as the reference stores them)."""

    def __init__(self, weights: dict, config: dict, max_seq: int):
        import torch

        import eyebrowse_b200 as eb
        self.eb, self.s, self.max_seq = eb, spec_from_config(config), max_seq
        s = self.s
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()
        f16 = lambda *names: torch.from_numpy(np.ascontiguousarray(
            np.concatenate([weights[n] for n in names]).astype(np.float16))).cuda()
        H, Hkv, D, inter = s["heads"], s["kv_heads"], s["hidden"], s["inter"]
        self.vec = {k: dev(v) for k, v in weights.items()
                    if k.endswith("norm.weight") or k.endswith("layer_scalar")}
        self.embed = dev(weights["model.embed_tokens.weight"])
        self.lm_head = f16("lm_head.weight" if "lm_head.weight" in weights
                           else "model.embed_tokens.weight")
        self.L = []
        nb_lin = 0
        for i, ly in enumerate(s["layers"]):
            p, hd = f"model.layers.{i}", ly["head_dim"]
            width = (H + 2 * Hkv) * hd  # fused q/k/v rows, read in place
            cos, sin = eb.rope_tables(max_seq, hd, ly["theta"], ly["rope_angles"])
            cos, sin = dev(cos), dev(sin)
            desc = eb.make_desc(H, Hkv, hd, max_seq, eps=s["eps"], scale=ly["scale"],
                                q_stride=width, kv_stride=width, window=ly["window"])
            vw = torch.ones(hd, device="cuda") if ly["v_norm"] else None
            qn = self.vec[f"{p}.self_attn.q_norm.weight"] if ly["qk_norm"] else None
            kn = self.vec[f"{p}.self_attn.k_norm.weight"] if ly["qk_norm"] else None
            shape = (max_seq, Hkv, hd)
            self.L.append(dict(
                hd=hd, width=width, desc=desc, layer=eb.make_layer(qn, kn, vw, cos, sin),
                keep=(cos, sin, vw),
                qkv=f16(f"{p}.self_attn.q_proj.weight", f"{p}.self_attn.k_proj.weight",
                        f"{p}.self_attn.v_proj.weight"),
                o=f16(f"{p}.self_attn.o_proj.weight"),
                gate_up=f16(f"{p}.mlp.gate_proj.weight", f"{p}.mlp.up_proj.weight"),
                down=f16(f"{p}.mlp.down_proj.weight"),
                kc=torch.zeros(shape, device="cuda"), vc=torch.zeros(shape, device="cuda"),
                ws_prefill=eb.alloc_workspace(eb.attention_prefill_workspace_bytes(desc,
                                                                                   max_seq)),
                ws_decode=eb.alloc_workspace(eb.attention_decode_workspace_bytes(
                    desc, 1, max_seq - 1))))
            nb_lin = max([nb_lin] + [eb.linear_f16w_workspace_bytes(max_seq, k, n) for k, n in
                                     ((D, width), (H * hd, D), (D, 2 * inter), (inter, D))])
        self.ws_linear = eb.alloc_workspace(nb_lin) if nb_lin else None

    def reset(self):
        for ly in self.L:
            ly["kc"].zero_()
            ly["vc"].zero_()

    def _norm(self, x, w):
        import torch
        out = torch.empty_like(x)
        self.eb.rmsnorm(x, w, out, x.shape[0], x.shape[1], self.s["eps"])
        return out

    def _linear(self, x, w):
        import torch
        x = x.contiguous()
        rows, in_f = x.shape
        y = torch.empty(rows, w.shape[0], device="cuda")
        self.eb.linear_f16w(x, w, y, rows, in_f, w.shape[0], self.ws_linear)
        return y

    def _attention(self, i, h, base_pos):
        import torch
        s, ly, eb = self.s, self.L[i], self.eb
        H, Hkv, hd = s["heads"], s["kv_heads"], ly["hd"]
        prefill = base_pos == 0 and h.shape[0] > 1  # attention.rs:40
        rows = h.shape[0] if prefill else 1
        qkv = self._linear(h[:rows], ly["qkv"])
        q, k, v = qkv[:, :H * hd], qkv[:, H * hd:(H + Hkv) * hd], qkv[:, (H + Hkv) * hd:]
        o = torch.empty(rows, H * hd, device="cuda")
        if prefill:
            eb.attention_prefill(ly["desc"], ly["layer"], rows, q, k, v, ly["kc"], ly["vc"], o,
                                 ly["ws_prefill"])
        else:
            eb.attention_decode(ly["desc"], ly["layer"], base_pos, q, k, v, ly["kc"], ly["vc"],
                                o, ly["ws_decode"])
        return self._linear(o, ly["o"])

    def _mlp(self, i, h):
        import torch
        inter = self.s["inter"]
        gu = self._linear(h, self.L[i]["gate_up"])
        g, u = gu[:, :inter], gu[:, inter:]
        if self.s["gemma"]:
            a = 0.5 * g * (1.0 + torch.tanh(0.7978845608028654 * (g + 0.044715 * g * g * g)))
        else:
            a = g / (1.0 + torch.exp(-g))
        return self._linear(a * u, self.L[i]["down"])

    def logits(self, ids, base_pos: int):
        """[vocab] logits (torch, f32) of the last row after ids at positions
        base_pos.. ; updates the caches. Softcapped for Gemma."""
        import torch
        s, V = self.s, self.vec
        x = self.embed[torch.tensor(ids, device="cuda")].contiguous()
        if s["embed_scale"] is not None:
            x = x * torch.tensor(np.float32(s["embed_scale"]), device="cuda")
        for i in range(len(s["layers"])):
            p = f"model.layers.{i}"
            if s["gemma"]:
                a = self._norm(self._attention(i, self._norm(x, V[f"{p}.input_layernorm.weight"]),
                                               base_pos), V[f"{p}.post_attention_layernorm.weight"])
                x2 = x[: a.shape[0]] + a
                m = self._norm(self._mlp(i, self._norm(x2, V[f"{p}.pre_feedforward_layernorm.weight"])),
                               V[f"{p}.post_feedforward_layernorm.weight"])
                x = (x2 + m) * V[f"{p}.layer_scalar"]
            else:
                a = self._attention(i, self._norm(x, V[f"{p}.input_layernorm.weight"]), base_pos)
                x2 = x[: a.shape[0]] + a
                x = x2 + self._mlp(i, self._norm(x2, V[f"{p}.post_attention_layernorm.weight"]))
        out = self._linear(self._norm(x[-1:].contiguous(), V["model.norm.weight"]),
                           self.lm_head)[0]
        if s["softcap"]:
            cap = float(np.float32(s["softcap"]))
            out = cap * torch.tanh(out / cap)
        return out

    def generate(self, prompt, n_new: int) -> list:
        """Greedy ids: prefill the prompt, then decode one token at a time."""
        import torch
        if len(prompt) + n_new > self.max_seq:
            raise ValueError("prompt + n_new exceeds max_seq")
        self.reset()
        out = [int(torch.argmax(self.logits(list(prompt), 0)).item())]
        pos = len(prompt)
        while len(out) < n_new:
            out.append(int(torch.argmax(self.logits([out[-1]], pos)).item()))
            pos += 1
        return out
