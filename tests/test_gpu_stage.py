"""GPU: stage-output commitments (uwc_b200.sha) == the reference's agent.proto roots and leaves
(golden) and == the oracle on batched, ragged shapes."""
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def test_stage_roots_and_leaves_golden(dev):
    import torch

    from uwc_b200 import sha
    g = dict(np.load(os.path.join(GOLDEN, "stage_golden.npz")))
    n = 0
    while f"rows{n}" in g:
        rows = torch.from_numpy(g[f"rows{n}"]).to(dev)[None]
        assert sha.stage_output_roots(rows) == [bytes(g[f"root{n}"])], n
        assert np.array_equal(sha.sout_leaves(rows)[0], g[f"leaves{n}"]), n
        n += 1


@pytest.mark.parametrize("B,T,D", [(4, 7, 2048), (2, 300, 130), (3, 1, 4096), (8, 64, 256)])
def test_batched_stage_roots_vs_oracle(dev, B, T, D):
    import torch

    import stage as S
    from uwc_b200 import sha
    rng = np.random.default_rng(B * 1000 + T + D)
    out = (rng.standard_normal((B, T, D)) * 3).astype(np.float32)
    got = sha.stage_output_roots(torch.from_numpy(out).to(dev))
    assert got == [S.stage_output_root(out[b]) for b in range(B)]
