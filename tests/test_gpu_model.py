"""GPU: the attention, final-norm and log-softmax kernels and the whole deterministic forward
(uwc_b200.detmodel.DetQwen3) against the reference's own detrt outputs and the CPU oracle, plus
the reference's determinism properties (runtime/tests/test_detrt.py:54-71)."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mg():
    with open(os.path.join(GOLDEN, "model_golden.json")) as f:
        meta = json.load(f)
    return meta, dict(np.load(os.path.join(GOLDEN, "model_golden.npz")))


def bits(t):
    a = t.detach().cpu().numpy() if hasattr(t, "detach") else np.asarray(t)
    return np.ascontiguousarray(a, np.float32).view(np.int32)


@pytest.mark.parametrize("tag", ["a", "b"])
def test_attention_prefill_golden(dev, mg, tag):
    import torch
    from uwc_b200 import detgpu
    _, g = mg
    B, T, H, Hkv = (int(v) for v in g[f"att{tag}_shape"])
    c = lambda k: torch.from_numpy(g[f"att{tag}_{k}"]).to(dev)
    o = detgpu.attention(c("qq"), c("qs"), c("kq"), c("ks"), c("vq"), c("vs"), B, T, H, Hkv, float(g["inv_sqrt_hd"][0]))
    assert np.array_equal(bits(o), g[f"att{tag}_o"].view(np.int32))


@pytest.mark.parametrize("B,start,Tq,H,Hkv,maxlen", [(3, 299, 1, 4, 2, 320), (2, 100, 5, 8, 2, 128),
                                                      (1, 0, 70, 2, 2, 70), (2, 1000, 17, 4, 4, 1040),
                                                      (1, 2175, 1, 16, 8, 2176), (2, 0, 1, 2, 2, 16),
                                                      (1, 5, 1, 8, 2, 8), (2, 1100, 1, 8, 1, 1104),
                                                      (1, 4095, 1, 4, 1, 4096)])
def test_attention_cache_vs_oracle(dev, B, start, Tq, H, Hkv, maxlen):
    """New tokens at positions start .. start+Tq-1 over a KV cache (decode and chunked prefill).
    Tq = 1 runs the cluster decode kernel: 1, 2, 4 and 8 query heads per KV head, and key counts
    below the cluster size (CTAs without keys) as well as across several V tiles per CTA."""
    import torch

    import detq as D
    from uwc_b200 import detgpu
    rng = np.random.default_rng(start * 7 + Tq)
    S = start + Tq
    K = rng.integers(-127, 128, (B, S, Hkv, 128)).astype(np.int8)
    V = rng.integers(-127, 128, (B, S, Hkv, 128)).astype(np.int8)
    SK = (rng.random((B, S, Hkv)) * 0.03 + 1e-4).astype(np.float32)
    SV = (rng.random((B, S, Hkv)) * 0.03 + 1e-4).astype(np.float32)
    qq = rng.integers(-127, 128, (B, Tq, H, 128)).astype(np.int8)
    qs = (rng.random((B, Tq, H)) * 0.03 + 1e-4).astype(np.float32)
    inv = float(np.float32(1 / np.sqrt(128)))
    want = D.attention(qq, qs, K, SK, V, SV, start, inv)
    cache = dict(k=torch.zeros(B, Hkv, maxlen, 128, dtype=torch.int8), v=torch.zeros(B, Hkv, maxlen, 128, dtype=torch.int8),
                 sk=torch.zeros(B, Hkv, maxlen, 1), sv=torch.zeros(B, Hkv, maxlen, 1))
    cache["k"][:, :, :S] = torch.from_numpy(K).transpose(1, 2)
    cache["v"][:, :, :S] = torch.from_numpy(V).transpose(1, 2)
    cache["sk"][:, :, :S, 0] = torch.from_numpy(SK).transpose(1, 2)
    cache["sv"][:, :, :S, 0] = torch.from_numpy(SV).transpose(1, 2)
    cache = {k: v.to(dev).contiguous() for k, v in cache.items()}
    got = detgpu.attention_cache(torch.from_numpy(qq.reshape(B * Tq, H, 128)).to(dev),
                                 torch.from_numpy(qs.reshape(B * Tq, H, 1)).to(dev), cache, B, Tq, start, H, Hkv, inv)
    assert np.array_equal(bits(got), want.reshape(B * Tq, H * 128).view(np.int32))


def test_rmsnorm_and_logprobs_vs_oracle(dev):
    import torch

    import detq as D
    from uwc_b200 import detgpu
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((9, 2048)) * rng.choice([1e-3, 1.0, 30.0], (9, 1))).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(2048)).astype(np.float32)
    got = detgpu.rmsnorm(torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev), 1e-6)
    assert np.array_equal(bits(got), D.det_rmsnorm(x, w, 1e-6).view(np.int32))
    lg = (rng.standard_normal((5, 151936)) * 4).astype(np.float32)
    lg[1, [7, 99, 150000]] = lg[1].max() + 1.0          # a three-way tie: the first index wins
    lp, tok = detgpu.logprobs(torch.from_numpy(lg).to(dev))
    want = D.logprobs(lg)
    assert np.array_equal(bits(lp), want.view(np.int32))
    assert tok.cpu().tolist() == [int(np.argmax(r)) for r in want] and tok[1].item() == 7


@pytest.fixture(scope="module")
def model(mg):
    pytest.importorskip("transformers")
    import torch

    import model_fixture as mf
    from uwc_b200.detmodel import DetQwen3
    meta, _ = mg
    hf = mf.tiny_model()
    assert mf.weights_sha(hf) == meta["weights_sha"], "the tiny model did not regenerate identically"
    m = DetQwen3(hf, torch.device("cuda:0"), hadamard_block=mf.HADAMARD_BLOCK)
    assert m.rope_sha == meta["rope_sha"]
    return m


def test_forward_logprobs_greedy_equal_detrt(dev, mg, model):
    import torch
    _, g = mg
    prompt = torch.from_numpy(g["prompt"]).to(dev)
    h = model.forward(prompt, model.new_cache(2, 37), 0)
    assert np.array_equal(bits(h), g["hidden"].view(np.int32)), "prefill hidden differs from detrt"
    lp = model.logprobs(h[:, -1:])
    assert np.array_equal(bits(lp[:, 0]), g["lp_last"].view(np.int32)), "log-probabilities differ"
    for graph in (False, True):
        toks, step_h = model.generate_greedy(prompt, 12, graph=graph)
        assert toks.cpu().numpy().tolist() == g["toks"].tolist(), f"greedy tokens differ (graph={graph})"
        assert np.array_equal(bits(step_h), g["step_h"].view(np.int32)), f"decode hiddens differ (graph={graph})"


def test_prefill_equals_decode_equals_teacher_forcing(dev, model):
    import torch
    g = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, 1024, (2, 37), generator=g).to(dev)
    toks, step_h = model.generate_greedy(prompt, 12)
    full = torch.cat([prompt, toks[:, :-1]], 1)
    h_tf = model.forward(full, model.new_cache(2, full.shape[1]), 0)
    assert torch.equal(h_tf[:, 36:], step_h)


def test_batch_composition_invariance(dev, model):
    import torch
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, 1024, (4, 50), generator=g).to(dev)
    h4 = model.forward(ids, model.new_cache(4, 50), 0)
    h1 = model.forward(ids[2:3], model.new_cache(1, 50), 0)
    assert torch.equal(h4[2:3], h1)
