"""The weight-streaming GEMM (uwc_gemm_stream, m <= 64) against the exact product and the library's
separately tested output kernels:

  I32     == A W^T exactly (the oracle's float64 BLAS product, exact at these magnitudes);
  F32     == detgpu.dequant of the exact product (qwen3.py:125), BF16 its RNE rounding;
  RESID   == detgpu.dequant_residual (detgpu kernels.py:346-354);
  SWIGLU  == detgpu.swiglu of the gate/up product in the original row order (kernels.py:356-396).

Shapes cover ragged m (1 .. 64), n not a multiple of the 128-row block, k from one 16-byte step to
the C5 down projection's 14336, and the cluster split from 1 to 8 CTAs per row block. uwc_gemm
takes the same path for plain calls with m <= 64, and a CUDA-graph replay of a chain with
programmatic dependent launch matches eager calls without it."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib(dev):
    from uwc_b200 import _lib, detgpu, ops
    _lib.device_status(clear=True)
    yield ops, detgpu, _lib
    assert _lib.device_status(clear=True) == 0, "a kernel reported a device-side timeout"


def _operands(m, n, k, seed):
    rng = np.random.default_rng(seed)
    X = rng.integers(-64, 65, size=(m, k), dtype=np.int8)
    W = rng.integers(-64, 65, size=(n, k), dtype=np.int8)
    sx = (rng.random(m, dtype=np.float32) * 1e-2 + 1e-4).astype(np.float32)
    sw = (rng.random(n, dtype=np.float32) * 1e-3 + 1e-5).astype(np.float32)
    return X, W, sx, sw


SHAPES = [(1, 128, 16), (7, 200, 112), (16, 384, 4096), (17, 6144, 4096), (32, 4096, 4096),
          (33, 1024, 14336), (64, 512, 2048), (32, 4096, 14336), (5, 128, 4096 + 48)]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_stream_i32_exact(lib, m, n, k):
    ops, _, _ = lib
    X, W, _, _ = _operands(m, n, k, m * 7 + n + k)
    got = ops.gemm_stream(torch.from_numpy(X).cuda(), torch.from_numpy(W).cuda(), ops.SEPI_I32)
    assert np.array_equal(got.cpu().numpy(), O.gemm_i32_blas(X, W))


@pytest.mark.parametrize("m,n,k", [(32, 6144, 4096), (9, 200, 2048), (64, 4096, 14336)])
def test_stream_scaled_epilogues(lib, m, n, k):
    ops, detgpu, _ = lib
    X, W, sx, sw = _operands(m, n, k, 11 + m)
    Xd, Wd = torch.from_numpy(X).cuda(), torch.from_numpy(W).cuda()
    sxd, swd = torch.from_numpy(sx).cuda(), torch.from_numpy(sw).cuda()
    acc = torch.from_numpy(O.gemm_i32_blas(X, W)).cuda()
    want = detgpu.dequant(acc, sxd, swd)
    f32 = ops.gemm_stream(Xd, Wd, ops.SEPI_F32, x_scale=sxd, w_scale=swd)
    assert torch.equal(f32, want)
    bf = ops.gemm_stream(Xd, Wd, ops.SEPI_BF16, x_scale=sxd, w_scale=swd)
    assert torch.equal(bf, want.to(torch.bfloat16))         # torch's float -> bf16 is RNE
    if n % 4 == 0:
        x = torch.randn(m, n, device="cuda", generator=torch.Generator(device="cuda").manual_seed(5))
        res = ops.gemm_stream(Xd, Wd, ops.SEPI_RESID, x_scale=sxd, w_scale=swd, resid=x)
        assert torch.equal(res, detgpu.dequant_residual(acc, sxd, swd, x))
        assert torch.equal(ops.gemm_stream(Xd, Wd, ops.SEPI_RESID, x_scale=sxd, w_scale=swd), want)


@pytest.mark.parametrize("m,two_i,k", [(32, 28672, 4096), (3, 256, 1024), (1, 384, 128), (64, 1024, 2048)])
def test_stream_swiglu(lib, m, two_i, k):
    ops, detgpu, _ = lib
    X, W, sx, sw = _operands(m, two_i, k, 21 + m)
    Xd, Wd = torch.from_numpy(X).cuda(), torch.from_numpy(W).cuda()
    sxd, swd = torch.from_numpy(sx).cuda(), torch.from_numpy(sw).cuda()
    acc = torch.from_numpy(O.gemm_i32_blas(X, W)).cuda()
    want = detgpu.swiglu(acc, sxd, swd)
    got = ops.gemm_stream(Xd, Wd, ops.SEPI_SWIGLU, x_scale=sxd, w_scale=swd)
    assert got.shape == (m, two_i // 2)
    assert torch.equal(got, want)


def test_uwc_gemm_routes_small_m(lib):
    ops, detgpu, _ = lib
    m, n, k = 32, 4096, 4096
    X, W, sx, sw = _operands(m, n, k, 3)
    Xd, Wd = torch.from_numpy(X).cuda(), torch.from_numpy(W).cuda()
    sxd, swd = torch.from_numpy(sx).cuda(), torch.from_numpy(sw).cuda()
    assert int(ops.lib().uwc_gemm_workspace_bytes(m, n, 0, ops.OUT_F32)) == 0
    out = torch.empty(m, n, dtype=torch.float32, device="cuda")
    l0 = ops.launches()
    ops.gemm(Xd, Wd, a_scale=sxd, b_scale=swd, out=out, out_mode=ops.OUT_F32)
    assert ops.launches() - l0 == 1                          # one launch: no memset, no scaling pass
    assert torch.equal(out, ops.gemm_stream(Xd, Wd, ops.SEPI_F32, x_scale=sxd, w_scale=swd))


def test_graph_chain_with_pdl_matches_eager(lib):
    """quantizer -> stream GEMM chains, captured with programmatic dependent launch (weights streamed
    early where the caller allows it), replay to the same bits as eager calls launched without it."""
    ops, detgpu, _lib = lib
    g = torch.Generator(device="cuda").manual_seed(9)
    m, d, n2 = 32, 4096, 8192
    x = torch.randn(m, d, device="cuda", generator=g)
    W1 = torch.randint(-64, 65, (n2, d), dtype=torch.int8, device="cuda", generator=g)
    W2 = torch.randint(-64, 65, (d, n2 // 2), dtype=torch.int8, device="cuda", generator=g)
    s1 = torch.rand(n2, device="cuda", generator=g) * 1e-3 + 1e-5
    s2 = torch.rand(d, device="cuda", generator=g) * 1e-3 + 1e-5

    def chain(xin):
        q, s = detgpu.quant_act(xin, 512)
        h = ops.gemm_stream(q, W1, ops.SEPI_SWIGLU, x_scale=s, w_scale=s1, early_w=True)
        q2, sq2 = detgpu.quant_act(h, 512)
        y = ops.gemm_stream(q2, W2, ops.SEPI_RESID, x_scale=sq2, w_scale=s2, resid=xin, early_w=True)
        q3, sq3 = detgpu.rmsnorm_quant(y, s2 * 1e3, 1e-5, 512)
        return ops.gemm_stream(q3, W1, ops.SEPI_F32, x_scale=sq3, w_scale=s1)

    _lib.lib().uwc_test_hook(_lib.HOOK_STREAM_PDL, 0)
    try:
        want = chain(x)
        torch.cuda.synchronize()
    finally:
        _lib.lib().uwc_test_hook(_lib.HOOK_STREAM_PDL, 1)
    xs = x.clone()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        chain(xs)
    torch.cuda.current_stream().wait_stream(st)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ys = chain(xs)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(ys, want)
    del graph


def test_stream_rejects_bad_calls(lib):
    ops, _, _lib = lib
    X = torch.zeros(65, 128, dtype=torch.int8, device="cuda")
    W = torch.zeros(128, 128, dtype=torch.int8, device="cuda")
    out = torch.empty(65, 128, dtype=torch.int32, device="cuda")
    L = ops.lib()
    assert L.uwc_gemm_stream(ops._p(X), ops._p(W), 65, 128, 128, None, None, None, ops._p(out), 0, None) \
        == _lib.ERR_SHAPE                                     # m > 64
    assert L.uwc_gemm_stream(ops._p(X), ops._p(W), 8, 128, 24, None, None, None, ops._p(out), 0, None) \
        == _lib.ERR_SHAPE                                     # k % 16
    assert L.uwc_gemm_stream(ops._p(X), ops._p(W), 8, 128, 128, None, None, None, ops._p(out), 1, None) \
        == _lib.ERR_ARG                                       # F32 without scales
    assert L.uwc_gemm_stream(ops._p(X), ops._p(W), 8, 192, 128, ops._p(out), ops._p(out), None, ops._p(out), 4,
                             None) == _lib.ERR_SHAPE          # SWIGLU needs n % 128


@pytest.mark.parametrize("k,bs", [(4096, 512), (14336, 512), (6144, 512), (1024, 128), (2048, 32), (4096, 1024),
                                  (2048, 1), (512, 512)])
def test_few_row_quantizers_match_one_cta_rows(lib, k, bs):
    """A row's quantization does not depend on how many rows the call has: with 512-element blocks
    every call keeps each row in registers (one warp per block); with other block sizes decode-sized
    calls (fewer rows than SMs) stage each row in shared memory with 1024 threads and larger calls
    with 256. Both give the same bits for the same row (the oracle tests pin each path)."""
    ops, detgpu, _ = lib
    g = torch.Generator(device="cuda").manual_seed(k + bs)
    big = 160
    x = torch.randn(big, k, device="cuda", generator=g) * 3
    w = 1 + 0.1 * torch.randn(k, device="cuda", generator=g)
    qa, sa = detgpu.quant_act(x, bs)
    qr, sr = detgpu.rmsnorm_quant(x, w, 1e-6, bs)
    for m in (1, 32, 33):
        q1, s1 = detgpu.quant_act(x[:m].contiguous(), bs)
        assert torch.equal(q1, qa[:m]) and torch.equal(s1, sa[:m])
        q2, s2 = detgpu.rmsnorm_quant(x[:m].contiguous(), w, 1e-6, bs)
        assert torch.equal(q2, qr[:m]) and torch.equal(s2, sr[:m])


@pytest.mark.parametrize("m,n,k", [(300, 2048, 1024), (128, 512, 4096), (1000, 400, 2048), (2048, 4096, 1024),
                                   (48, 1024, 2048)])
def test_gemm_epi_any_m(lib, m, n, k):
    """uwc_gemm_epi: the same epilogues at prefill-sized m, in the tcgen05 GEMM's epilogue (SwiGLU
    from 128 gate rows over their up rows per tile; the residual add in the fp32 store, also after
    a skinny shape's split-K sum), == the separate output kernels on the exact product."""
    ops, detgpu, _ = lib
    X, W, sx, sw = _operands(m, n, k, 31 + m)
    Xd, Wd = torch.from_numpy(X).cuda(), torch.from_numpy(W).cuda()
    sxd, swd = torch.from_numpy(sx).cuda(), torch.from_numpy(sw).cuda()
    acc = torch.from_numpy(O.gemm_i32_blas(X, W)).cuda()
    x = torch.randn(m, n, device="cuda", generator=torch.Generator(device="cuda").manual_seed(m))
    assert torch.equal(ops.gemm_epi(Xd, Wd, ops.SEPI_I32), acc)
    assert torch.equal(ops.gemm_epi(Xd, Wd, ops.SEPI_F32, x_scale=sxd, w_scale=swd), detgpu.dequant(acc, sxd, swd))
    assert torch.equal(ops.gemm_epi(Xd, Wd, ops.SEPI_RESID, x_scale=sxd, w_scale=swd, resid=x),
                       detgpu.dequant_residual(acc, sxd, swd, x))
    h = ops.gemm_epi(Xd, Wd, ops.SEPI_SWIGLU, x_scale=sxd, w_scale=swd)
    assert h.shape == (m, n // 2)
    assert torch.equal(h, detgpu.swiglu(acc, sxd, swd))
