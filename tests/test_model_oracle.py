"""CPU: the attention / log-softmax oracle (oracle/detq.py) and the model's rotary tables against
vectors and artifacts of the reference's own runtime (tests/golden/make_golden_model.py)."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN


@pytest.fixture(scope="module")
def mg():
    with open(os.path.join(GOLDEN, "model_golden.json")) as f:
        meta = json.load(f)
    return meta, dict(np.load(os.path.join(GOLDEN, "model_golden.npz")))


@pytest.mark.parametrize("tag", ["a", "b"])
def test_oracle_attention_matches_detgpu_reference(mg, tag):
    import detq as D
    _, g = mg
    B, T, H, Hkv = (int(v) for v in g[f"att{tag}_shape"])
    o = D.attention(g[f"att{tag}_qq"].reshape(B, T, H, 128), g[f"att{tag}_qs"].reshape(B, T, H),
                    g[f"att{tag}_kq"].reshape(B, T, Hkv, 128), g[f"att{tag}_ks"].reshape(B, T, Hkv),
                    g[f"att{tag}_vq"].reshape(B, T, Hkv, 128), g[f"att{tag}_vs"].reshape(B, T, Hkv), 0,
                    float(g["inv_sqrt_hd"][0]))
    assert np.array_equal(o.reshape(B * T, H * 128).view(np.int32), g[f"att{tag}_o"].view(np.int32))


def test_rope_tables_equal_the_reference_artifacts(mg):
    """The model computes its cos / sin tables; they equal every table the reference pins."""
    from uwc_b200.detmodel import rope_table
    meta, _ = mg
    assert meta["rope_tables"]
    for name, t in meta["rope_tables"].items():
        sc = None
        if t["llama3"]:
            f, lo, hi, orig = t["llama3"]
            sc = dict(factor=f, low_freq_factor=lo, high_freq_factor=hi, original_max_position_embeddings=orig)
        assert rope_table(t["theta"], t["hd"], t["pos"], sc)[2] == t["sha"], name


def test_oracle_logprobs_of_the_tiny_model(mg):
    """lm_head (DetLinear on the tied embedding) + logprobs through the oracle == detrt's."""
    pytest.importorskip("transformers")
    import detq as D
    import model_fixture as mf
    meta, g = mg
    hf = mf.tiny_model()
    assert mf.weights_sha(hf) == meta["weights_sha"], "the tiny model did not regenerate identically"
    W = hf.lm_head.weight.detach().float().numpy()
    bs = min(mf.HADAMARD_BLOCK, W.shape[1] & -W.shape[1])
    Wq, sw = D.quant_act(W, bs)
    h = g["hidden"][:, -1]
    q, sx = D.quant_act(h, bs)
    acc = q.astype(np.int64) @ Wq.astype(np.int64).T
    lg = D.fmul(D.fmul(acc.astype(np.float32), sx[:, None]), sw[None, :])
    assert np.array_equal(D.logprobs(lg).view(np.int32), g["lp_last"].view(np.int32))
