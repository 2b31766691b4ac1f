"""Generate tests/golden/model_golden.npz from the reference's own DetQwen3 (runtime/detrt) on CPU.

Run in a checkout that has the reference next to it (not needed by the tests themselves):
    python tests/golden/make_golden_model.py <path to srivassid/useful-work-coin>

The model is tests/model_fixture.py's tiny random Qwen3 (head_dim 128). Outputs: a prefill
forward's final-norm hidden, its last-position log-probabilities, a 12-token greedy decode (tokens
and step hiddens), and runtime/detgpu/stages.py's attention_torch on seeded quantized q, k, v.
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref: str) -> None:
    sys.path.insert(0, os.path.join(ref, "runtime"))
    sys.path.insert(0, os.path.dirname(HERE))
    import torch
    from detrt import core
    from detrt.qwen3 import DetQwen3
    from detgpu.stages import attention_torch

    import model_fixture as mf

    core.setup_determinism()
    hf = mf.tiny_model()
    m = DetQwen3(hf, "cpu", hadamard_block=mf.HADAMARD_BLOCK, mine=False)
    out: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, mf.CFG["vocab_size"], (2, 37), generator=g)
    h = m.forward(prompt, m.new_cache(2, 37), 0)
    lp = m.logprobs(h[:, -1:])
    toks, step_h = m.generate_greedy(prompt, 12)
    out.update(prompt=prompt.numpy(), hidden=h.numpy(), lp_last=lp[:, 0].numpy(), toks=toks.numpy(),
               step_h=step_h.numpy())

    # attention alone, prefill layout, several query blocks and key tiles
    rng = np.random.default_rng(7)
    for tag, (B, T, H, Hkv) in {"a": (2, 40, 4, 2), "b": (1, 150, 2, 1)}.items():
        N = B * T
        qq = rng.integers(-127, 128, (N, H, 128)).astype(np.int8)
        kq = rng.integers(-127, 128, (N, Hkv, 128)).astype(np.int8)
        vq = rng.integers(-127, 128, (N, Hkv, 128)).astype(np.int8)
        qs = (rng.random((N, H, 1)) * 0.02 + 1e-4).astype(np.float32)
        ks = (rng.random((N, Hkv, 1)) * 0.02 + 1e-4).astype(np.float32)
        vs = (rng.random((N, Hkv, 1)) * 0.02 + 1e-4).astype(np.float32)
        mm = types.SimpleNamespace(H=H, Hkv=Hkv, hd=128, inv_sqrt_hd=m.inv_sqrt_hd)
        tt = lambda a: torch.from_numpy(a)
        o = attention_torch(mm, tt(qq).float(), tt(qs), tt(kq).float(), tt(ks), tt(vq).float(), tt(vs), B, T)
        out.update({f"att{tag}_qq": qq, f"att{tag}_kq": kq, f"att{tag}_vq": vq, f"att{tag}_qs": qs,
                    f"att{tag}_ks": ks, f"att{tag}_vs": vs, f"att{tag}_o": o.numpy(),
                    f"att{tag}_shape": np.array([B, T, H, Hkv])})
    out["inv_sqrt_hd"] = np.array([m.inv_sqrt_hd], np.float32)
    # every rotary table the reference pins, by its parameters (runtime/artifacts/*.npz)
    import glob
    import hashlib
    import re
    tables = {}
    for path in sorted(glob.glob(os.path.join(ref, "runtime", "artifacts", "rope_*.npz"))):
        name = os.path.basename(path)
        mt = re.match(r"rope_theta([0-9.e+]+)_hd(\d+)_pos(\d+)(?:_llama3_([0-9.e+]+)_([0-9.e+]+)_([0-9.e+]+)_(\d+))?\.npz", name)
        if not mt:
            continue
        d = np.load(path)
        tables[name] = dict(theta=float(mt.group(1)), hd=int(mt.group(2)), pos=int(mt.group(3)),
                            llama3=[float(mt.group(4)), float(mt.group(5)), float(mt.group(6)), int(mt.group(7))]
                            if mt.group(4) else None,
                            sha=hashlib.sha256(d["cos"].tobytes() + d["sin"].tobytes()).hexdigest())
    meta = dict(weights_sha=mf.weights_sha(hf), rope_sha=m.rope_sha, rope_tables=tables)
    np.savez_compressed(os.path.join(HERE, "model_golden.npz"), **out)
    import json
    with open(os.path.join(HERE, "model_golden.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print({k: v.shape for k, v in out.items()}, meta)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ["UWC_REFERENCE"])
