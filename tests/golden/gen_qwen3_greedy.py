"""Golden greedy token ids for the Qwen3-0.6B-geometry harness, from
HuggingFace transformers.

The reference pins its Qwen3 model against HF transformers greedy ids
(golden/gen_golden.py, golden/qwen3-golden.json in the reference repo) with
the real checkpoint, which is not available here. This script builds the
same architecture in HF (Qwen3ForCausalLM: QK-RMSNorm, RoPE theta 1e6,
SwiGLU, tied embeddings, f32, eager attention), loads the seeded random-init
weights of eyebrowse_b200.qwen3.make_weights (f16-valued linear weights as
the reference stores them), and records the greedy continuation of seeded
prompts. Each step recomputes the whole sequence (no KV cache), so the ids
do not depend on HF's cache code. It also records each step's gap between
the two largest logits, the margin a correct implementation must not cross.

Run from the repo root:  python tests/golden/gen_qwen3_greedy.py
Writes tests/golden/qwen3_greedy_ids.json (a few KB).
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from eyebrowse_b200.qwen3 import GEOMETRY, make_prompts, make_weights  # noqa: E402

WEIGHT_SEED, PROMPT_SEED, N_PROMPTS, PROMPT_LEN, N_NEW = 0, 1, 2, 12, 8


def main() -> None:
    import transformers
    from transformers import Qwen3Config, Qwen3ForCausalLM

    g = GEOMETRY
    cfg = Qwen3Config(hidden_size=g["hidden"], intermediate_size=g["inter"],
                      num_hidden_layers=g["layers"], num_attention_heads=g["heads"],
                      num_key_value_heads=g["kv_heads"], head_dim=g["head_dim"],
                      vocab_size=g["vocab"], rms_norm_eps=g["eps"],
                      rope_parameters={"rope_theta": g["theta"], "rope_type": "default"},
                      tie_word_embeddings=True, attention_bias=False,
                      max_position_embeddings=4096, hidden_act="silu")
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    model = Qwen3ForCausalLM(cfg).float().eval()
    w = make_weights(WEIGHT_SEED)
    missing, unexpected = model.load_state_dict({k: torch.from_numpy(v) for k, v in w.items()},
                                                strict=False)
    assert not unexpected, unexpected
    assert set(missing) <= {"lm_head.weight"}, missing
    assert model.lm_head.weight.data_ptr() == model.model.embed_tokens.weight.data_ptr()

    prompts = make_prompts(PROMPT_SEED, N_PROMPTS, PROMPT_LEN)
    out, gaps = [], []
    with torch.no_grad():
        for prompt in prompts:
            ids = list(prompt)
            gen, gp = [], []
            for _ in range(N_NEW):
                logits = model(torch.tensor([ids])).logits[0, -1].double().numpy()
                top = np.argsort(logits)[-2:]
                nxt = int(np.argmax(logits))
                gp.append(float(logits[top[1]] - logits[top[0]]))
                gen.append(nxt)
                ids.append(nxt)
            out.append(gen)
            gaps.append(gp)
            print("prompt", prompt, "->", gen, "min top-2 gap %.4f" % min(gp), flush=True)
    rec = {"weight_seed": WEIGHT_SEED, "prompt_seed": PROMPT_SEED, "n_prompts": N_PROMPTS,
           "prompt_len": PROMPT_LEN, "n_new": N_NEW, "geometry": g, "prompts": prompts,
           "ids": out, "top2_gap": gaps, "transformers": transformers.__version__,
           "torch": torch.__version__}
    with open(os.path.join(HERE, "qwen3_greedy_ids.json"), "w") as f:
        json.dump(rec, f, indent=1)


if __name__ == "__main__":
    main()
