"""GPU: the batched tcgen05 GEMM (causal block skipping and causal k ranges) against exact integer
products, and the tensor-core attention against the SIMT attention kernel and the oracle, bit for
bit (prefill from a KV cache, chunked prefill with start > 0, grouped query heads, ragged Tq)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.detach().contiguous().cpu().numpy().view(np.int32)


@pytest.mark.parametrize("nbatch,m,n,k,bdiv", [(3, 256, 512, 128, 1), (4, 128, 260, 256, 2), (2, 384, 128, 1024, 2)])
def test_gemm_batched_plain(dev, nbatch, m, n, k, bdiv):
    from uwc_b200 import _lib
    from uwc_b200._lib import check, lib
    g = torch.Generator(device=dev).manual_seed(m + n + k)
    nkv = (nbatch - 1) // bdiv + 1
    A = torch.randint(-127, 128, (nbatch * m, k), dtype=torch.int8, device=dev, generator=g)
    B = torch.randint(-127, 128, (nkv * n, k), dtype=torch.int8, device=dev, generator=g)
    out = torch.zeros((nbatch, m, n), dtype=torch.int32, device=dev)
    check(lib().uwc_gemm_batched(A.data_ptr(), B.data_ptr(), m, n, k, nbatch, m, n, bdiv, 0, 0, 0, out.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream), "gemm_batched")
    for bt in range(nbatch):
        a = A[bt * m:(bt + 1) * m].cpu().numpy().astype(np.int64)
        b = B[(bt // bdiv) * n:(bt // bdiv + 1) * n].cpu().numpy().astype(np.int64)
        assert np.array_equal(out[bt].cpu().numpy(), (a @ b.T).astype(np.int32)), bt
    assert _lib.device_status(clear=True) == 0


def test_gemm_batched_causal_blocks(dev):
    """causal 1: every output element some row sees is the exact product (others are not written)."""
    from uwc_b200._lib import check, lib
    nbatch, m, n, k, cshift = 2, 384, 700, 128, 200
    g = torch.Generator(device=dev).manual_seed(3)
    A = torch.randint(-127, 128, (nbatch * m, k), dtype=torch.int8, device=dev, generator=g)
    B = torch.randint(-127, 128, (nbatch * 704, k), dtype=torch.int8, device=dev, generator=g)
    out = torch.full((nbatch, m, n), -7, dtype=torch.int32, device=dev)
    check(lib().uwc_gemm_batched(A.data_ptr(), B.data_ptr(), m, n, k, nbatch, m, 704, 1, 1, cshift, 0,
                                 out.data_ptr(), torch.cuda.current_stream().cuda_stream), "gemm_batched")
    o = out.cpu().numpy()
    for bt in range(nbatch):
        a = A[bt * m:(bt + 1) * m].cpu().numpy().astype(np.int64)
        b = B[bt * 704:bt * 704 + n].cpu().numpy().astype(np.int64)
        want = (a @ b.T).astype(np.int32)
        seen = np.arange(n)[None, :] <= cshift + np.arange(m)[:, None]
        assert np.array_equal(o[bt][seen], want[seen]), bt


def test_gemm_batched_causal_k(dev):
    """causal 2: a 128-row block's k range ends after key cshift + (m0 % qrows) + 127; with the A
    rows zero past their visible keys the product equals the full product."""
    from uwc_b200._lib import check, lib
    nbatch, qrows, k, cshift = 3, 256, 640, 100
    m, n = 2 * qrows, 128
    rng = np.random.default_rng(4)
    A = rng.integers(-127, 128, (nbatch, m, k), dtype=np.int64)
    t = np.arange(m) % qrows
    A[:, np.arange(k)[None, :] > cshift + t[:, None]] = 0
    B = rng.integers(-127, 128, (nbatch * n, k), dtype=np.int64)
    Ad = torch.from_numpy(A.astype(np.int8).reshape(nbatch * m, k)).to(dev)
    Bd = torch.from_numpy(B.astype(np.int8)).to(dev)
    out = torch.zeros((nbatch, m, n), dtype=torch.int32, device=dev)
    check(lib().uwc_gemm_batched(Ad.data_ptr(), Bd.data_ptr(), m, n, k, nbatch, m, n, 1, 2, cshift, qrows,
                                 out.data_ptr(), torch.cuda.current_stream().cuda_stream), "gemm_batched")
    for bt in range(nbatch):
        assert np.array_equal(out[bt].cpu().numpy(), (A[bt] @ B[bt * n:(bt + 1) * n].T).astype(np.int32)), bt


def _cache(dev, B, S, Hkv, maxlen, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    c = dict(k=torch.randint(-127, 128, (B, Hkv, maxlen, 128), dtype=torch.int8, device=dev, generator=g),
             v=torch.randint(-127, 128, (B, Hkv, maxlen, 128), dtype=torch.int8, device=dev, generator=g),
             sk=torch.rand(B, Hkv, maxlen, 1, device=dev, generator=g) * 0.03 + 1e-4,
             sv=torch.rand(B, Hkv, maxlen, 1, device=dev, generator=g) * 0.03 + 1e-4)
    return c, g


@pytest.mark.parametrize("B,start,Tq,H,Hkv", [(2, 0, 300, 4, 2), (1, 0, 1024, 16, 8), (3, 200, 130, 2, 2),
                                             (2, 1000, 257, 8, 1), (1, 0, 128, 4, 4), (8, 0, 2048, 16, 8)])
def test_attention_tc_equals_simt(dev, B, start, Tq, H, Hkv):
    from uwc_b200 import _lib, detgpu
    S = start + Tq
    cache, g = _cache(dev, B, S, Hkv, S + 5, B * 1000 + S)
    qq = torch.randint(-127, 128, (B * Tq, H, 128), dtype=torch.int8, device=dev, generator=g)
    qs = torch.rand(B * Tq, H, 1, device=dev, generator=g) * 0.03 + 1e-4
    inv = float(np.float32(1 / np.sqrt(128)))
    a = detgpu.attention_cache(qq, qs, cache, B, Tq, start, H, Hkv, inv, path="simt")
    b = detgpu.attention_cache(qq, qs, cache, B, Tq, start, H, Hkv, inv, path="tc")
    assert np.array_equal(_bits(a), _bits(b))
    assert _lib.device_status(clear=True) == 0


def test_attention_tc_vs_oracle(dev):
    """Against the CPU restatement of detrt's attention (oracle/detq.py) on a small prefill."""
    import detq as D
    from uwc_b200 import detgpu
    B, start, Tq, H, Hkv = 2, 40, 140, 4, 2
    rng = np.random.default_rng(17)
    S = start + Tq
    K = rng.integers(-127, 128, (B, S, Hkv, 128)).astype(np.int8)
    V = rng.integers(-127, 128, (B, S, Hkv, 128)).astype(np.int8)
    SK = (rng.random((B, S, Hkv)) * 0.03 + 1e-4).astype(np.float32)
    SV = (rng.random((B, S, Hkv)) * 0.03 + 1e-4).astype(np.float32)
    qq = rng.integers(-127, 128, (B, Tq, H, 128)).astype(np.int8)
    qs = (rng.random((B, Tq, H)) * 0.03 + 1e-4).astype(np.float32)
    inv = float(np.float32(1 / np.sqrt(128)))
    want = D.attention(qq, qs, K, SK, V, SV, start, inv)
    cache = dict(k=torch.from_numpy(K).transpose(1, 2).contiguous().to(dev),
                 v=torch.from_numpy(V).transpose(1, 2).contiguous().to(dev),
                 sk=torch.from_numpy(SK).transpose(1, 2)[..., None].contiguous().to(dev),
                 sv=torch.from_numpy(SV).transpose(1, 2)[..., None].contiguous().to(dev))
    got = detgpu.attention_cache(torch.from_numpy(qq.reshape(B * Tq, H, 128)).to(dev),
                                 torch.from_numpy(qs.reshape(B * Tq, H, 1)).to(dev), cache, B, Tq, start, H, Hkv, inv,
                                 path="tc")
    assert np.array_equal(_bits(got), want.reshape(B * Tq, H * 128).view(np.int32))
