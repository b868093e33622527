"""Greedy decode of the random-init Qwen3-0.6B-geometry model with every
layer's attention on this library (eyebrowse_b200.qwen3.GreedyModel): the
token ids equal the HF transformers golden ids (and so the model oracle's),
and the logits of a prefill step and a decode step match the model oracle's
at max-abs <= 2e-3 and rel-L2 <= 1e-3."""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def setup():
    from eyebrowse_b200.qwen3 import GEOMETRY, make_weights
    with open(os.path.join(HERE, "golden", "qwen3_greedy_ids.json")) as f:
        gold = json.load(f)
    return gold, make_weights(gold["weight_seed"]), GEOMETRY


def test_gpu_model_greedy_ids_match_golden(eb, setup):
    from eyebrowse_b200.qwen3 import GreedyModel
    gold, w, geo = setup
    m = GreedyModel(w, gold["prompt_len"] + gold["n_new"], geo)
    for prompt, want in zip(gold["prompts"], gold["ids"]):
        assert m.generate(prompt, gold["n_new"]) == want
    assert eb.device_error() == 0


def test_gpu_model_logits_match_oracle(eb, orc, setup):
    from eyebrowse_b200.qwen3 import GreedyModel
    from oracle.model_oracle import OracleModel
    gold, w, geo = setup
    max_seq = gold["prompt_len"] + gold["n_new"]
    gm, om = GreedyModel(w, max_seq, geo), OracleModel(w, max_seq, geo)
    prompt, first = gold["prompts"][0], gold["ids"][0][0]
    for ids, pos in ((prompt, 0), ([first], len(prompt))):
        got = gm.logits(ids, pos).cpu().numpy()
        want = om.logits(ids, pos)
        assert np.argmax(got) == np.argmax(want)
        assert orc.max_abs(got, want) <= 2e-3 and orc.rel_l2(got, want) <= 1e-3, (
            pos, orc.max_abs(got, want), orc.rel_l2(got, want))
