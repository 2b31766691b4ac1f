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


def test_oracle_forward_of_the_tiny_model(mg):
    """The oracle's layer composition (quantized linears, qkv_post, attention, MLP, final norm)
    reproduces detrt's prefill hidden of the tiny model bit for bit."""
    pytest.importorskip("transformers")
    import detq as D
    import model_fixture as mf
    from uwc_b200.detmodel import rope_table
    meta, g = mg
    hf = mf.tiny_model()
    cfg, hb = mf.CFG, mf.HADAMARD_BLOCK
    f = lambda t: t.detach().float().numpy()
    cos, sin, sha = rope_table(cfg["rope_parameters"]["rope_theta"], cfg["head_dim"], 8192)
    assert sha == meta["rope_sha"]
    B, T = g["prompt"].shape
    x = f(hf.model.embed_tokens.weight)[g["prompt"].reshape(-1)]
    inv = float(np.float32(1.0 / np.sqrt(cfg["head_dim"])))
    import torch
    for lay in hf.model.layers:
        at, mlp = lay.self_attn, lay.mlp
        L = dict(in_norm=f(lay.input_layernorm.weight), post_norm=f(lay.post_attention_layernorm.weight),
                 q_norm=f(at.q_norm.weight), k_norm=f(at.k_norm.weight),
                 qkv=D.quantize_linear(f(torch.cat([at.q_proj.weight, at.k_proj.weight, at.v_proj.weight])), hb),
                 o=D.quantize_linear(f(at.o_proj.weight), hb),
                 gu=D.quantize_linear(f(torch.cat([mlp.gate_proj.weight, mlp.up_proj.weight])), hb),
                 down=D.quantize_linear(f(mlp.down_proj.weight), hb))
        x = D.layer_forward(L, x, B, T, cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["rms_norm_eps"],
                            cos, sin, inv)
    h = D.det_rmsnorm(x, f(hf.model.norm.weight), cfg["rms_norm_eps"]).reshape(B, T, -1)
    assert np.array_equal(h.view(np.int32), g["hidden"].view(np.int32))
