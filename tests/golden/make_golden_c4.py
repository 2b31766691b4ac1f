"""Generate tests/golden/c4_golden.json from the reference's own DetQwen3 (runtime/detrt) on CPU at
BASELINE configs[3]'s shape: the whole 28-layer Qwen3-1.7B-shaped model, random-init.

Run in a checkout that has the reference next to it (the tests only read the JSON it writes):
    python tests/golden/make_golden_c4.py <path to srivassid/useful-work-coin>

Records, for tests/model_fixture.py's c4_model() and c4_prompt() (2 sequences x 48 tokens): the
sampled weight fingerprint, detrt's per-layer residual hashes and final-norm hidden hash of the
prefill, the last positions' log-probability hash, and a 4-token greedy decode (tokens, hash of
the step hiddens). Hashes are detrt's own sha() (sha256 of the float32 bytes, 20 hex digits).
"""
from __future__ import annotations

import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref: str) -> None:
    sys.path.insert(0, os.path.join(ref, "runtime"))
    sys.path.insert(0, os.path.dirname(HERE))
    import torch
    from detrt import core
    from detrt.qwen3 import DetQwen3, sha

    import model_fixture as mf

    core.setup_determinism()
    t0 = time.time()
    hf = mf.c4_model()
    fp = mf.sampled_weights_sha(hf)
    print(f"model built and fingerprinted in {time.time() - t0:.0f} s", flush=True)
    m = DetQwen3(hf, "cpu", hadamard_block=mf.C4_HADAMARD_BLOCK, mine=False)
    print(f"DetQwen3 ready at {time.time() - t0:.0f} s", flush=True)
    prompt = mf.c4_prompt()
    B, T = prompt.shape
    layer_hashes: list = []
    h = m.forward(prompt, m.new_cache(B, T), 0, layer_hashes=layer_hashes)
    lp = m.logprobs(h[:, -1:])
    print(f"prefill at {time.time() - t0:.0f} s", flush=True)
    n_new = 4
    toks, step_h = m.generate_greedy(prompt, n_new)
    print(f"greedy decode at {time.time() - t0:.0f} s", flush=True)
    meta = dict(weights_sha=fp, rope_sha=m.rope_sha, prompt_shape=[B, T], n_new=n_new, layer_hashes=layer_hashes,
                hidden_sha=sha(h), lp_last_sha=sha(lp), toks=toks.tolist(), step_h_sha=sha(step_h),
                hidden_last_head=[float(v) for v in h[0, -1, :8]])
    with open(os.path.join(HERE, "c4_golden.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print(meta)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ["UWC_REFERENCE"])
