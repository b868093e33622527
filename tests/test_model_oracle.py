"""The greedy-decode model oracle (oracle/model_oracle.py, a numpy
restatement of the reference decoder driver with the C oracle's attention)
reproduces the HF transformers greedy ids of tests/golden/qwen3_greedy_ids.json
for the seeded random-init Qwen3-0.6B-geometry model. This pins the model
oracle that tests/test_gpu_model.py checks the GPU harness against."""
import json
import os

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def gold():
    with open(os.path.join(HERE, "golden", "qwen3_greedy_ids.json")) as f:
        return json.load(f)


def test_oracle_model_matches_hf_greedy_ids(gold):
    from eyebrowse_b200.qwen3 import GEOMETRY, make_prompts, make_weights
    from oracle.model_oracle import OracleModel
    assert gold["geometry"] == GEOMETRY
    assert gold["prompts"] == make_prompts(gold["prompt_seed"], gold["n_prompts"],
                                           gold["prompt_len"])
    w = make_weights(gold["weight_seed"])
    m = OracleModel(w, gold["prompt_len"] + gold["n_new"], GEOMETRY)
    for prompt, want in zip(gold["prompts"], gold["ids"]):
        assert m.generate(prompt, gold["n_new"]) == want
