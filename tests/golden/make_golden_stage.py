"""Generate tests/golden/stage_golden.npz from the reference's own stage commitments
(runtime/agent/proto.py stage_output_root / stage_out_leaves over runtime/detrt/stage.py).

    python tests/golden/make_golden_stage.py <path to srivassid/useful-work-coin>
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = [(1, 1), (3, 255), (37, 256), (5, 300), (40, 1024), (3, 8192)]   # (T, D)


def main(ref: str) -> None:
    sys.path.insert(0, os.path.join(ref, "runtime"))
    from agent import proto
    rng = np.random.default_rng(99)
    out = {}
    for i, (T, D) in enumerate(CASES):
        rows = (rng.standard_normal((T, D)) * 10 ** rng.uniform(-3, 3)).astype(np.float32)
        out[f"rows{i}"] = rows
        out[f"root{i}"] = np.frombuffer(proto.stage_output_root(list(rows)), np.uint8)
        out[f"leaves{i}"] = np.stack([np.frombuffer(x, np.uint8) for x in proto.stage_out_leaves(list(rows))])
    np.savez_compressed(os.path.join(HERE, "stage_golden.npz"), **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ["UWC_REFERENCE"])
