"""det.patch_detlinear: the monkey-patch of DetLinear.int_gemm (runtime/detrt/qwen3.py:106-119)
that runtime/agent/mining.py:49-65 applies, pointed at this library. On the host it must leave the
reference's CPU path in place (checked on the reference's own class when a checkout is at hand,
UWC_REFERENCE); on a GPU a layer with the reference's attributes gets the exact int32 product, and
a mining layer gets MinedWeight.forward's int32 output on rows padded to 64."""
import os
import sys

import numpy as np
import pytest
import torch

import oracle as O


class _StandIn:
    """The attributes DetLinear.int_gemm reads: device, Wq, mine, mw."""

    def __init__(self, Wq, device, mw=None):
        self.device, self.Wq, self.mine, self.mw = torch.device(device), Wq, mw is not None, mw
        self.n, self.k = Wq.shape

    def int_gemm(self, q):
        return q.to(torch.float64) @ self.Wq.to(torch.float64).t()


def test_patch_keeps_the_reference_cpu_path():
    ref = os.environ.get("UWC_REFERENCE")
    if not ref or not os.path.isdir(os.path.join(ref, "runtime", "detrt")):
        pytest.skip("no reference checkout (UWC_REFERENCE) to take DetLinear from")
    sys.path.insert(0, os.path.join(ref, "runtime"))
    from detrt.qwen3 import DetLinear

    from uwc_b200 import det
    W = torch.randn(96, 256, generator=torch.Generator().manual_seed(3)) * 0.02
    lin = DetLinear(W, "cpu", 64, False)
    q = torch.randint(-127, 128, (5, 256), dtype=torch.int8, generator=torch.Generator().manual_seed(4))
    before = lin.int_gemm(q)
    det.patch_detlinear(DetLinear)
    det.patch_detlinear(DetLinear)          # idempotent
    try:
        assert DetLinear._uwc_b200_patched and DetLinear._orig_int_gemm is not DetLinear.int_gemm
        after = lin.int_gemm(q)
        assert torch.equal(before, after) and after.dtype == torch.float64
        assert np.array_equal(after.numpy().astype(np.int64), O.gemm_i32(q.numpy(), lin.Wq.numpy()))
    finally:
        DetLinear.int_gemm = DetLinear._orig_int_gemm
        del DetLinear._uwc_b200_patched


@pytest.mark.gpu
def test_patched_int_gemm_on_gpu(dev):
    from uwc_b200 import det, glue, ops

    class Layer(_StandIn):
        pass

    det.patch_detlinear(Layer)
    rng = np.random.default_rng(8)
    Wq = rng.integers(-64, 65, (512, 2048), dtype=np.int8)
    q = rng.integers(-127, 128, (37, 2048), dtype=np.int8)
    want = O.gemm_i32(q, Wq)
    plain = Layer(torch.from_numpy(Wq).cuda(), "cuda")
    got = plain.int_gemm(torch.from_numpy(q).cuda())
    assert got.dtype == torch.int32 and np.array_equal(got.cpu().numpy(), want)
    mw = ops.MinedWeight(Bt=torch.from_numpy(Wq).cuda(), b_scale=torch.ones(512, device="cuda"), r=128)
    mw.setup_block(bytes(range(32)), glue.target_for(64, 512, 4))
    mined = Layer(torch.from_numpy(Wq).cuda(), "cuda", mw=mw)
    qm = rng.integers(-64, 65, (37, 2048), dtype=np.int8)   # mined operands stay in [-64, 64] (quant_sym(64))
    got = mined.int_gemm(torch.from_numpy(qm).cuda())
    assert got.shape == (37, 512) and np.array_equal(got.cpu().numpy(), O.gemm_i32(qm, Wq))
    cpu = Layer(torch.from_numpy(Wq), "cpu")
    assert np.array_equal(cpu.int_gemm(torch.from_numpy(q)).numpy().astype(np.int64), want)
