"""The oracle model (oracle/ref_models.py) pinned to the reference's own
golden fixtures: tiny Mistral and dense Gemma 4 models built and run by
eyebrowse's golden/gen_mistral_golden.py and golden/gen_gemma4_golden.py
(unmodified, via tests/golden/gen_ref_golden.py), whose HF last-position
logits the reference's Rust tests check at rel-L2 < 2e-2
(crates/eyebrowse/tests/mistral.rs:46-57, gemma4.rs:46-56). The same bound
holds here, and the oracle's greedy token matches HF's."""
import hashlib
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FIXTURES = ("mistral_tiny", "gemma4_tiny")
SCRIPTS = {"mistral_tiny": "gen_mistral_golden.py", "gemma4_tiny": "gen_gemma4_golden.py"}


def _fixture(name):
    return os.path.join(ROOT, "tests", "golden", f"ref_{name}.npz")


@pytest.mark.parametrize("name", FIXTURES)
def test_oracle_model_matches_reference_golden(orc, name):
    from oracle.ref_models import RefOracleModel, load_fixture
    w, cfg, ids, gold = load_fixture(_fixture(name))
    got = RefOracleModel(w, cfg, 64).logits(ids, 0)
    rel = float(np.linalg.norm(got - gold) / (np.linalg.norm(gold) + 1e-12))
    assert rel < 2e-2, f"{name}: rel-L2 {rel:.3e} (the reference's bound is 2e-2)"
    assert int(np.argmax(got)) == int(np.argmax(gold))


@pytest.mark.parametrize("name", FIXTURES)
def test_fixture_came_from_the_reference_generator(name):
    """The fixture records the sha256 of the generator script that made it;
    where the reference checkout is present, it must be the current script."""
    z = np.load(_fixture(name))
    digest = bytes(z["__generator_sha256__"]).decode()
    # the reference checkout: $EYEBROWSE_REF, else a "reference" folder beside this repository
    ref = os.environ.get("EYEBROWSE_REF", os.path.join(os.path.dirname(ROOT), "reference"))
    src = os.path.join(ref, "golden", SCRIPTS[name])
    if not os.path.exists(src):
        pytest.skip("reference checkout not present")
    with open(src, "rb") as f:
        assert hashlib.sha256(f.read()).hexdigest() == digest


def test_gemma4_spec_follows_the_reference_loader():
    """Per-layer geometry gemma4.rs derives from the config: head_dim 16 on
    the two sliding layers, 32 on the full layer with floor(0.25*32/2) = 4
    rotary pairs, scale 1.0, QK-norm and weightless V-norm everywhere."""
    from oracle.ref_models import load_fixture, model_spec
    _, cfg, _, _ = load_fixture(_fixture("gemma4_tiny"))
    s = model_spec(cfg)
    assert [ly["head_dim"] for ly in s["layers"]] == [16, 16, 32]
    assert [ly["rope_angles"] for ly in s["layers"]] == [8, 8, 4]
    assert [ly["theta"] for ly in s["layers"]] == [1e4, 1e4, 1e6]
    assert all(ly["scale"] == 1.0 and ly["qk_norm"] and ly["v_norm"] for ly in s["layers"])
    assert s["softcap"] == 30.0 and abs(s["embed_scale"] - 8.0) < 1e-6
