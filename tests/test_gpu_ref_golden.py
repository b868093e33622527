"""The reference's own golden models on the GPU path: the tiny Mistral and
dense Gemma 4 fixtures that eyebrowse's golden generators produce (see
tests/golden/gen_ref_golden.py), run through eyebrowse_b200.decoder with
every attention on this library's C ABI (head_dim 32 for Mistral; 16 and 32
for Gemma 4, its partial rotary, softcap and sliding-window layers).

Checked three ways: the prefill's last-position logits against HF's golden
at the reference's own bound, rel-L2 < 2e-2 (crates/eyebrowse/tests/
mistral.rs:46-57, gemma4.rs:46-56); the same logits against the oracle
model at the north-star tolerance (max-abs <= 2e-3, rel-L2 <= 1e-3); and
six greedy decode steps, whose ids and logits must match the oracle's."""
import os

import numpy as np
import pytest

from _util import assert_close

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("name", ["mistral_tiny", "gemma4_tiny"])
def test_reference_golden_model_on_gpu(eb, orc, name):
    from eyebrowse_b200.decoder import DecoderModel
    from oracle.ref_models import RefOracleModel, load_fixture
    w, cfg, ids, gold = load_fixture(os.path.join(ROOT, "tests", "golden", f"ref_{name}.npz"))
    model = DecoderModel(w, cfg, 64)
    ref = RefOracleModel(w, cfg, 64)
    got = model.logits(ids, 0).cpu().numpy()
    want = ref.logits(ids, 0)
    rel = float(np.linalg.norm(got - gold) / (np.linalg.norm(gold) + 1e-12))
    assert rel < 2e-2, f"{name}: rel-L2 vs HF golden {rel:.3e}"
    assert_close(orc, got, want, what=f"{name} prefill logits vs oracle")
    assert int(np.argmax(got)) == int(np.argmax(gold))
    tok, pos = int(np.argmax(want)), len(ids)
    for step in range(6):
        g = model.logits([tok], pos).cpu().numpy()
        r = ref.logits([tok], pos)
        assert_close(orc, g, r, what=f"{name} decode step {step}")
        assert int(np.argmax(g)) == int(np.argmax(r))
        tok, pos = int(np.argmax(r)), pos + 1
    assert eb.device_error() == 0
