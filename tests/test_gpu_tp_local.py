"""The tensor-parallel exchange kernels on one GPU (the driver's GPU tests run on one):

  - a one-rank exchange (every value sent to itself through the tagged-word protocol) gives the
    local kernels' bits: uwc_quant_act_tp == uwc_quant_act, uwc_gemm_stream_tp == uwc_gemm_stream,
    eagerly and over many CUDA-graph replays with device-side barriers between them (the call
    counter on the device advances per call);
  - the bounded wait: a two-rank exchange whose second rank never writes (its buffer is a second
    local allocation nothing writes into) ends with UWC_DEV_TIMEOUT after the shortened wait bound,
    and the context stays usable. No GPU fault, no hang: the wait simply runs out."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mods(dev):
    from uwc_b200 import _lib, detgpu, ops, tp
    _lib.device_status(clear=True)
    return _lib, detgpu, ops, tp


@pytest.mark.parametrize("two_phase_min", [8, 1])
def test_one_rank_exchange_matches_local_kernels(mods, two_phase_min):
    """two_phase_min 1: the GEMM's exchange in its reduce-scatter + all-gather form."""
    _lib, detgpu, ops, tp = mods
    assert _lib.lib().uwc_test_hook(_lib.HOOK_TP_TWO_PHASE, two_phase_min) == 0
    ex = tp.PeerExchange(64, 4096, 0, 1, torch.device("cuda", 0))
    try:
        g = torch.Generator(device="cuda").manual_seed(4)
        K = tp.GPUKernels()
        for m, k, n in ((32, 4096, 4096), (7, 14336, 4096), (64, 2048, 1024)):
            x = torch.randn(m, k, device="cuda", generator=g)
            W = torch.randint(-64, 65, (n, k), dtype=torch.int8, device="cuda", generator=g)
            sw = torch.rand(n, device="cuda", generator=g) * 1e-3 + 1e-5
            res = torch.randn(m, n, device="cuda", generator=g)
            q, s = detgpu.quant_act(x, 512)
            qt, st = K.quant_act_tp(x, 512, ex)
            assert torch.equal(qt, q) and torch.equal(st, s)
            want = ops.gemm_stream(q, W, ops.SEPI_RESID, x_scale=s, w_scale=sw, resid=res)
            assert torch.equal(K.linear_resid_tp(q, s, W, sw, res, ex), want)
        # a captured pair of calls replayed many times: each replay is a new epoch on the device
        m, k, n = 32, 4096, 4096
        x = torch.randn(m, k, device="cuda", generator=g)
        W = torch.randint(-64, 65, (n, k), dtype=torch.int8, device="cuda", generator=g)
        sw = torch.rand(n, device="cuda", generator=g) * 1e-3 + 1e-5
        q, s = detgpu.quant_act(x, 512)
        want = ops.gemm_stream(q, W, ops.SEPI_RESID, x_scale=s, w_scale=sw, resid=x[:, :n].contiguous())

        def step():
            qt, st = K.quant_act_tp(x, 512, ex)
            return K.linear_resid_tp(qt, st, W, sw, x[:, :n].contiguous(), ex)

        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            y = step()
        for _ in range(7):
            ex.barrier()                   # a call of its own in the same sequence
            graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(y, want)
        del graph
        assert _lib.device_status(clear=True) == 0
    finally:
        ex.close()
        _lib.lib().uwc_test_hook(_lib.HOOK_TP_TWO_PHASE, 8)


def test_exchange_wait_runs_out_and_reports(mods):
    _lib, detgpu, ops, tp = mods
    L = _lib.lib()
    bufs = []
    for _ in range(2):
        b = ctypes.c_void_p()
        _lib.check(L.uwc_tp_alloc(64, 1024, ctypes.byref(b)), "tp_alloc")
        bufs.append(b)
    t = tp._UwcTP(0, 2, 64, 1024)
    t.base[0], t.base[1] = bufs[0].value, bufs[1].value
    x = torch.randn(8, 1024, device="cuda")
    q = torch.empty(8, 1024, dtype=torch.int8, device="cuda")
    s = torch.empty(8, device="cuda")
    _lib.device_status(clear=True)
    assert L.uwc_test_hook(_lib.HOOK_WAIT_NS, 5_000_000) == 0          # 5 ms
    try:
        rc = L.uwc_quant_act_tp(ops._p(x), 8, 1024, 512, ops._p(q), ops._p(s), ctypes.byref(t), ops._stream())
        assert rc == 0
        torch.cuda.synchronize()
        assert _lib.device_status(clear=True) & _lib.DEV_TIMEOUT
    finally:
        assert L.uwc_test_hook(_lib.HOOK_WAIT_NS, 0) == 0
        for b in bufs:
            L.uwc_tp_free(b)
    # the context is intact: the local quantizer gives its usual result
    q2, s2 = detgpu.quant_act(x, 512)
    torch.cuda.synchronize()
    assert q2.shape == (8, 1024) and _lib.device_status(clear=True) == 0
