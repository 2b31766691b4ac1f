"""BASELINE configs[3] at its own shape: the whole 28-layer Qwen3-1.7B-shaped model, random-init,
on this library's DetQwen3 against the reference's own DetQwen3 (runtime/detrt/qwen3.py:286-329)
run on the host by tests/golden/make_golden_c4.py: every layer's residual, the final-norm hidden,
the last positions' log-probabilities and a 4-token greedy decode (graph-replayed and eager), bit
for bit. The model is rebuilt here from the same seed (tests/model_fixture.py) and checked against
the fixture's weight fingerprint first."""
import json
import os

import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def c4(dev):
    pytest.importorskip("transformers")
    import model_fixture as mf
    from uwc_b200.detmodel import DetQwen3
    with open(os.path.join(GOLDEN, "c4_golden.json")) as f:
        meta = json.load(f)
    hf = mf.c4_model()
    assert mf.sampled_weights_sha(hf) == meta["weights_sha"], "the host built different weights"
    model = DetQwen3(hf, dev, hadamard_block=mf.C4_HADAMARD_BLOCK)
    del hf
    return model, mf.c4_prompt().to(dev), meta


def test_c4_prefill_equals_detrt(c4):
    from uwc_b200.detmodel import sha
    model, prompt, meta = c4
    B, T = prompt.shape
    assert model.rope_sha == meta["rope_sha"]
    hashes: list = []
    h = model.forward(prompt, model.new_cache(B, T), 0, layer_hashes=hashes)
    assert hashes == meta["layer_hashes"]
    assert sha(h) == meta["hidden_sha"]
    assert sha(model.logprobs(h[:, -1:])) == meta["lp_last_sha"]


@pytest.mark.parametrize("graph", [True, False])
def test_c4_greedy_decode_equals_detrt(c4, graph):
    from uwc_b200.detmodel import sha
    model, prompt, meta = c4
    toks, step_h = model.generate_greedy(prompt, meta["n_new"], graph=graph)
    assert toks.cpu().tolist() == meta["toks"]
    assert sha(step_h) == meta["step_h_sha"]
