"""Parity at the BASELINE configs' own shapes, against the oracle port of
the reference's reference.py, with the reference's noise:

  C2  4096 x 4096 x 4096 mined forward, r = 64 and 128: the int32 output == A B^T exactly, and the
      hash of every one of the 131072 tiles == the oracle's (a target every tile meets makes each
      tile report itself once), and the winner set at the config's 2^-20 target;
  C3  8192 x 14336 x 4096 noise mining, r = 64 and 128: all 917504 tile hashes and the 2^-20
      winner set, as the reference's known-answer test does at small size
      (miner/ampere/tests/test_kernels.py:94-125).

Inputs follow the configs: A, B^T uniform in [-64, 63] from seeded numpy generators, a seeded
32-byte job key standing in for Pearl's header hash (parity of the header step is out of reach
without pearl_mining). The oracle's fold runs in C on the host's threads (about 10 s at C3)."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

ALL = O.bound_words((1 << 256) - 1)            # every tile wins: each reports its own hash
CONFIG_TARGET = O.bound_words(((1 << 256) - 1) >> 20)


@pytest.fixture(scope="module")
def ops(dev):
    from uwc_b200 import _lib, ops
    _lib.device_status(clear=True)
    yield ops
    assert _lib.device_status(clear=True) == 0, "a kernel reported a device-side timeout"


def _operands(m, n, k):
    A = np.random.default_rng(1).integers(-64, 64, size=(m, k), dtype=np.int8)
    Bt = np.random.default_rng(2).integers(-64, 64, size=(n, k), dtype=np.int8)
    return A, Bt, np.random.default_rng(3).bytes(32)


def _records(w, m):
    """Every win record of the last call, sorted: [(row_off, col_off, hash bytes)]."""
    words = w.buffers(m)["wins"].cpu().numpy().view(np.uint32)
    cnt = int(words[0])
    assert cnt <= w.max_wins
    recs = words[1:1 + cnt * 10].reshape(cnt, 10)
    return sorted((int(x[0]), int(x[1]), x[2:].astype("<u4").tobytes()) for x in recs)


def _under(records, target_words):
    t = int.from_bytes(np.asarray(target_words, np.uint32).astype("<u4").tobytes(), "little")
    return [rec for rec in records if int.from_bytes(rec[2], "little") <= t]


@pytest.mark.parametrize("r", [64, 128])
def test_c2_mined_forward_exact_and_every_tile(ops, r):
    m = n = k = 4096
    A, Bt, key = _operands(m, n, k)
    a_seed, _, want_all, _ = O.mined_reference(A, Bt, key, r, ALL)
    assert len(want_all) == m * n // 128
    w = ops.MinedWeight(Bt=torch.from_numpy(Bt).cuda(), b_scale=torch.ones(n, device="cuda"), r=r,
                        max_wins=m * n // 128)
    w.setup_block(key, ALL)
    out = w.forward(torch.from_numpy(A).cuda(), torch.ones(m, device="cuda"), out_mode=ops.OUT_I32)
    assert ops.words_to_bytes(w.buffers(m)["a_seed"]) == a_seed
    assert np.array_equal(out.cpu().numpy(), O.gemm_i32_blas(A, Bt))
    got_all = _records(w, m)
    assert got_all == want_all
    # the config's own target: the same tiles through the kernel's target compare
    w.setup_block(key, CONFIG_TARGET)
    w.forward(torch.from_numpy(A).cuda(), torch.ones(m, device="cuda"), out=out, out_mode=ops.OUT_I32)
    assert _records(w, m) == _under(want_all, CONFIG_TARGET)


@pytest.mark.parametrize("r", [64, 128])
def test_c3_noise_mining_every_tile(ops, r):
    m, n, k = 8192, 14336, 4096
    A, Bt, key = _operands(m, n, k)
    a_seed, _, want_all, _ = O.mined_reference(A, Bt, key, r, ALL)
    assert len(want_all) == m * n // 128
    w = ops.MinedWeight(Bt=torch.from_numpy(Bt).cuda(), b_scale=torch.ones(n, device="cuda"), r=r,
                        max_wins=m * n // 128)
    w.setup_block(key, ALL)
    Ad = torch.from_numpy(A).cuda()
    w.noise_mine(Ad)
    assert ops.words_to_bytes(w.buffers(m)["a_seed"]) == a_seed
    assert _records(w, m) == want_all
    w.setup_block(key, CONFIG_TARGET)
    w.noise_mine(Ad)
    assert _records(w, m) == _under(want_all, CONFIG_TARGET)
