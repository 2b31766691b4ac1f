"""The device-timeout error path, with no fault: a GEMM launched while the test hook withholds its
copies has a wait that nothing will satisfy (its first stage never arrives). With the bound of
every wait cut to 5 ms, each CTA's MMA warp gives up, raises the CTA's abort flag and the sticky
UWC_DEV_TIMEOUT bit, the other warps see the flag and unwind, TMEM is freed, and the call
returns. The host reads the bit with uwc_device_status; the context stays usable: the same GEMM
right afterwards, hooks cleared, gives the oracle's exact results."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture()
def hooks(dev):
    from uwc_b200 import _lib
    L = _lib.lib()
    _lib.device_status(clear=True)
    yield L
    assert L.uwc_test_hook(_lib.HOOK_WITHHOLD, 0) == 0
    assert L.uwc_test_hook(_lib.HOOK_WAIT_NS, 0) == 0


@pytest.mark.parametrize("flags", [1, 0])
def test_wait_runs_out_reports_timeout_and_context_survives(hooks, flags):
    from uwc_b200 import _lib, glue, ops
    L = hooks
    m, n, k, r = 256, 512, 1024, 64
    rng = np.random.default_rng(31)
    A = rng.integers(-64, 65, (m, k), dtype=np.int8)
    B = rng.integers(-64, 65, (n, k), dtype=np.int8)
    key = rng.bytes(32)
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    keyw = torch.from_numpy(O.words(key).view(np.int32).copy()).cuda()
    target = glue.target_for(m, n, 20)
    tgt = torch.from_numpy(target.view(np.int32).copy()).cuda()
    wins = torch.zeros(1 + 4096 * 10, dtype=torch.int32, device="cuda")
    out = torch.zeros((m, n), dtype=torch.int32, device="cuda")
    kw = dict(r=r, flags=1, key=keyw, target=tgt, wins=wins, max_wins=4096) if flags else dict(out=out,
                                                                                          out_mode=ops.OUT_I32)
    assert L.uwc_test_hook(_lib.HOOK_WAIT_NS, 5_000_000) == 0
    assert L.uwc_test_hook(_lib.HOOK_WITHHOLD, 1) == 0
    ops.gemm(Ad, Bd, **kw)                                   # returns; the kernel unwinds by itself
    assert _lib.device_status(clear=True) & _lib.DEV_TIMEOUT
    assert L.uwc_test_hook(_lib.HOOK_WITHHOLD, 0) == 0
    assert L.uwc_test_hook(_lib.HOOK_WAIT_NS, 0) == 0
    wins.zero_()
    ops.gemm(Ad, Bd, **kw)
    assert _lib.device_status(clear=True) == 0
    if flags:
        want = O.winners(O.jackpot_msgs(A, B, r), key, target)
        h = wins.cpu().numpy().view(np.uint32)
        recs = h[1:1 + int(h[0]) * 10].reshape(-1, 10)
        got = sorted((int(x[0]), int(x[1]), x[2:].astype("<u4").tobytes()) for x in recs)
        assert want and got == want
    else:
        assert np.array_equal(out.cpu().numpy(), O.gemm_i32(A, B))


def test_hook_arguments_are_checked(dev):
    from uwc_b200 import _lib
    L = _lib.lib()
    assert L.uwc_test_hook(99, 0) == _lib.ERR_ARG
    assert L.uwc_test_hook(_lib.HOOK_WITHHOLD, 2) == _lib.ERR_ARG
    assert L.uwc_test_hook(_lib.HOOK_WAIT_NS, -1) == _lib.ERR_ARG
