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


# Qwen3-1.7B's shape, random-init (HF's N(0, 0.02) linears and embedding,
# unit norms), tied embedding as in the released model.
C4_CFG = dict(vocab_size=151936, hidden_size=2048, intermediate_size=6144, num_hidden_layers=28,
              num_attention_heads=16, num_key_value_heads=8, head_dim=128, max_position_embeddings=40960,
              rms_norm_eps=1e-6, tie_word_embeddings=True, initializer_range=0.02,
              rope_parameters={"rope_theta": 1e6, "rope_type": "default"})
C4_HADAMARD_BLOCK = 512
C4_SEED = 1234


def c4_model():
    """The configs[3] model on the host, the same bits on every machine with this torch and
    transformers (CPU generator, seeded)."""
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM
    torch.manual_seed(C4_SEED)
    return Qwen3ForCausalLM(Qwen3Config(**C4_CFG)).eval()


def c4_prompt():
    import torch
    g = torch.Generator().manual_seed(C4_SEED + 1)
    return torch.randint(0, C4_CFG["vocab_size"], (2, 48), generator=g)


def sampled_weights_sha(m, stride: int = 251) -> str:
    """sha256 over every parameter's name, shape and every stride-th value (a cheap fingerprint of a
    model too large to hash whole in a test)."""
    h = hashlib.sha256()
    for k, v in sorted(m.state_dict().items()):
        h.update(k.encode())
        h.update(str(tuple(v.shape)).encode())
        h.update(v.detach().float().reshape(-1)[::stride].contiguous().numpy().tobytes())
    return h.hexdigest()
