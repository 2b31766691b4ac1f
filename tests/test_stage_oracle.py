"""CPU: the stage-commitment oracle (oracle/stage.py) against roots and leaves the reference's
runtime/agent/proto.py computed (tests/golden/make_golden_stage.py), and the bottom-up tree order
the GPU kernels use against RFC 6962's recursive split."""
import hashlib
import os

import numpy as np
import pytest

from conftest import GOLDEN


@pytest.fixture(scope="module")
def sg():
    return dict(np.load(os.path.join(GOLDEN, "stage_golden.npz")))


def test_oracle_stage_roots_match_reference(sg):
    import stage as S
    n = 0
    while f"rows{n}" in sg:
        rows = sg[f"rows{n}"]
        assert S.stage_output_root(rows) == bytes(sg[f"root{n}"]), n
        leaves = [S.stage_out_leaf(t, S.row_root(r)) for t, r in enumerate(rows)]
        assert leaves == [bytes(x) for x in sg[f"leaves{n}"]], n
        n += 1
    assert n >= 5


def test_bottom_up_tree_equals_rfc6962_split():
    import stage as S
    for n in range(1, 300):
        leaves = [hashlib.sha256(i.to_bytes(4, "little")).digest() for i in range(n)]
        assert S.merkle_root_bottom_up(leaves) == S.merkle_root(leaves), n
