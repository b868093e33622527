"""Regenerate the reference-pinned model fixtures: runs eyebrowse's own golden
generators UNMODIFIED and converts their outputs into small fixtures here.

    python tests/golden/gen_ref_golden.py [path/to/eyebrowse]

The reference repository ships two generators that build tiny random-init
HuggingFace models and record HF's last-position logits, which its Rust
tests compare against at rel-L2 < 2e-2:

  golden/gen_mistral_golden.py  -> crates/eyebrowse/tests/mistral.rs:46-57
      2-layer Mistral (hidden 128, 4/2 heads, head_dim 32, vocab 320,
      theta 1e6, untied lm_head), seed 0, ids [1, 5, 9, 13, 17]
  golden/gen_gemma4_golden.py   -> crates/eyebrowse/tests/gemma4.rs:46-56
      3-layer dense Gemma 4 (two sliding layers at head_dim 16 theta 1e4, one
      full layer at head_dim 32 with 25% "proportional" rotary theta 1e6,
      QK-norm, weightless V-norm, scale 1.0, GeGLU, sandwich norms, layer
      scalars, x sqrt(hidden) embedding, final softcap 30), seed 0,
      ids [1, 5, 9, 13]

The scripts write next to themselves (../models/<name>/ and golden/), so
they are copied into a temporary directory laid out like the reference
checkout and run there with this interpreter (transformers 5.5, CPU, f32);
nothing of the reference is copied into this repository. Each fixture
ref_<name>.npz holds what the reference's loader consumes -- the model's
tensors (projection and embedding weights as f16, exactly what the
reference keeps on the GPU after its f16 upload, crates/eyebrowse-models/src/
upload.rs:38-42; norm weights and layer scalars as f32) and config.json --
plus HF's input ids and last-position logits, and the sha256 of the
generator script that produced them.

Test infrastructure only: tests/test_ref_golden_models.py (CPU oracle model)
and tests/test_gpu_ref_golden.py (the GPU path) read these fixtures.
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GENERATORS = {
    # fixture name: (generator script, directory it saves the model under)
    "mistral_tiny": ("gen_mistral_golden.py", "mistral-tiny"),
    "gemma4_tiny": ("gen_gemma4_golden.py", "gemma4-tiny"),
}


def _f16_tensor(name: str) -> bool:
    """Tensors the reference uploads as packed f16: embeddings and linear weights."""
    return name.endswith(("_proj.weight", "embed_tokens.weight", "lm_head.weight"))


def generate(ref_root: str, out_dir: str = HERE) -> list:
    from safetensors.numpy import load_file

    written = []
    with tempfile.TemporaryDirectory() as tmp:
        os.makedirs(os.path.join(tmp, "golden"))
        for fixture, (script, model_dir) in GENERATORS.items():
            src = os.path.join(ref_root, "golden", script)
            dst = os.path.join(tmp, "golden", script)
            shutil.copyfile(src, dst)
            env = dict(os.environ, CUDA_VISIBLE_DEVICES="", PYTHONHASHSEED="0")
            subprocess.run([sys.executable, dst], cwd=tmp, env=env, check=True,
                           stdout=subprocess.DEVNULL)
            mdir = os.path.join(tmp, "models", model_dir)
            tensors = load_file(os.path.join(mdir, "model.safetensors"))
            with open(os.path.join(mdir, "config.json")) as f:
                config = f.read()
            golden_path = os.path.join(tmp, "golden", f"{model_dir}-golden.json")
            with open(golden_path) as f:
                golden = json.load(f)
            arrays = {}
            for name, t in tensors.items():
                t = np.asarray(t, dtype=np.float32)
                arrays[name] = t.astype(np.float16) if _f16_tensor(name) else t
            arrays["__config__"] = np.frombuffer(config.encode(), dtype=np.uint8)
            arrays["__input_ids__"] = np.asarray(golden["input_ids"], dtype=np.int64)
            arrays["__last_logits__"] = np.asarray(golden["last_logits"], dtype=np.float32)
            with open(src, "rb") as f:
                digest = hashlib.sha256(f.read()).hexdigest()
            arrays["__generator_sha256__"] = np.frombuffer(digest.encode(), dtype=np.uint8)
            out = os.path.join(out_dir, f"ref_{fixture}.npz")
            np.savez_compressed(out, **arrays)
            written.append(out)
    return written


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("EYEBROWSE_REF", "")
    if not root or not os.path.isdir(os.path.join(root, "golden")):
        raise SystemExit("usage: gen_ref_golden.py <eyebrowse checkout with golden/gen_*.py>")
    for p in generate(root):
        print(p, os.path.getsize(p))
