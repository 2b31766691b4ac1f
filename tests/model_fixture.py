"""The tiny random Qwen3 used by the model parity tests, built the way the reference's own
determinism tests build theirs (runtime/tests/test_detrt.py:13-24), with head_dim 128 (the width
of the attention kernels) and Qwen3-1.7B's rope theta 1e6 (a table the reference pins)."""
from __future__ import annotations

import hashlib

CFG = dict(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
           num_key_value_heads=2, head_dim=128, max_position_embeddings=4096, rms_norm_eps=1e-6,
           tie_word_embeddings=True, rope_parameters={"rope_theta": 1e6, "rope_type": "default"})
HADAMARD_BLOCK = 64


def tiny_model():
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM
    torch.manual_seed(0)
    m = Qwen3ForCausalLM(Qwen3Config(**CFG)).eval()
    with torch.no_grad():                      # move the weights off the near-zero init
        for p in m.parameters():
            p.add_(torch.randn_like(p) * 0.05)
    return m


def weights_sha(m) -> str:
    h = hashlib.sha256()
    for k, v in sorted(m.state_dict().items()):
        h.update(k.encode())
        h.update(v.detach().float().contiguous().numpy().tobytes())
    return h.hexdigest()
