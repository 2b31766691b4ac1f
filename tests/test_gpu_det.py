"""The deterministic linear's producers and consumers on the GPU (csrc/detq.cu) against the detrt
golden vectors (tests/golden/det_golden.npz, made by detrt itself) and against oracle/detq.py on
larger seeded inputs: every output bit-identical (mirrors runtime tests test_detgpu.py /
test_detrt.py:54-95, which compare detgpu to detrt bit for bit)."""
import numpy as np
import pytest
import torch

import detq as D
import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dg(dev):
    from uwc_b200 import _lib, detgpu
    _lib.device_status(clear=True)
    yield detgpu
    assert _lib.device_status(clear=True) == 0


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def same(got, want):
    got = got.cpu().numpy() if isinstance(got, torch.Tensor) else np.asarray(got)
    want = np.asarray(want)
    got = got.reshape(want.shape).astype(want.dtype)
    if want.dtype == np.float32:
        got, want = got.view(np.uint32), want.view(np.uint32)
    bad = np.flatnonzero(got != want)
    assert bad.size == 0, f"{bad.size} mismatches, first at {bad[:5]}"


@pytest.mark.parametrize("bs", [0, 64, 512])
def test_quant_act_golden(dg, det_golden, bs):
    g = det_golden
    q, s = dg.quant_act(cu(g[f"qa{bs}_x"]), bs)
    same(q, g[f"qa{bs}_q"])
    same(s, g[f"qa{bs}_s"])


def test_rmsnorm_quant_golden(dg, det_golden):
    g = det_golden
    q, s = dg.rmsnorm_quant(cu(g["rq_x"]), cu(g["rq_w"]), 1e-6, 128)
    same(q, g["rq_q"])
    same(s, g["rq_s"])


def test_swiglu_quant_golden(dg, det_golden):
    g = det_golden
    q, s = dg.swiglu_quant(cu(g["sg_acc"]), cu(g["sg_s3"]), cu(g["sg_sw"]), 256)
    same(q, g["sg_q"])
    same(s, g["sg_s"])


def test_dequant_residual_golden(dg, det_golden):
    g = det_golden
    same(dg.dequant_residual(cu(g["dr_acc"]), cu(g["dr_s"]), cu(g["dr_sw"]), cu(g["dr_x"])), g["dr_out"])


@pytest.mark.parametrize("qk", [1, 0])
def test_qkv_post_golden(dg, det_golden, qk):
    g = det_golden
    res = dg.qkv_post(cu(g["qp_acc"]), cu(g["qp_s1"]), cu(g["qp_sw"]), cu(g["qp_qnw"]), cu(g["qp_knw"]),
                      cu(g["qp_cos"]), cu(g["qp_sin"]), 3, 2, 1, 1e-6, bool(qk))
    for name, a in zip(("qq", "qs", "kq", "ks", "vq", "vs"), res):
        same(a, g[f"qp{qk}_{name}"])


def _rows(rng, m, k):
    return (rng.standard_normal((m, k)) * rng.choice([1e-4, 0.02, 1.0, 300.0], (m, 1))).astype(np.float32)


@pytest.mark.parametrize("k,bs", [(4096, 0), (4096, 128), (2048, 512), (14336, 512), (6144, 512), (36, 4)])
def test_quant_act_against_oracle(dg, k, bs):
    rng = np.random.default_rng(k + bs)
    x = _rows(rng, 37, k)
    x[3] = 0.0
    q, s = dg.quant_act(cu(x), bs)
    wq, ws = D.quant_act(x, bs)
    same(q, wq)
    same(s, ws)


def test_quant_rows_had_bf16(dg):
    rng = np.random.default_rng(3)
    x = torch.from_numpy(_rows(rng, 19, 2048)).to(torch.bfloat16)
    q, s = dg.quant_rows_had(x.cuda(), 128)
    wq, ws = O.quant_rows_had(x.float().numpy(), 128)
    same(q, wq)
    same(s, ws)


def test_row_parallel_quantizer_equals_full_row(dg):
    """fwht_absmax per column shard + MAX + quant_act_global == quant_act of the whole row."""
    rng = np.random.default_rng(11)
    x = _rows(rng, 24, 4096)
    xd = cu(x)
    q, s = dg.quant_act(xd, 256)
    shards = torch.chunk(xd, 4, dim=1)
    amax = torch.stack([dg.fwht_absmax(sh, 256) for sh in shards]).amax(0)
    parts = [dg.quant_act_global(sh, 256, amax) for sh in shards]
    assert torch.equal(torch.cat([p[0] for p in parts], 1), q)
    for p in parts:
        assert torch.equal(p[1].view(torch.int32), s.view(torch.int32))


@pytest.mark.parametrize("k,bs", [(2048, 512), (4096, 128), (1024, 0)])
def test_rmsnorm_quant_against_oracle(dg, k, bs):
    rng = np.random.default_rng(k)
    x = _rows(rng, 21, k)
    w = (1.0 + 0.2 * rng.standard_normal(k)).astype(np.float32)
    q, s = dg.rmsnorm_quant(cu(x), cu(w), 1e-6, bs)
    wq, ws = D.rmsnorm_quant(x, w, 1e-6, bs)
    same(q, wq)
    same(s, ws)


@pytest.mark.parametrize("I,bs", [(6144, 512), (14336, 512), (1024, 0)])
def test_swiglu_quant_against_oracle(dg, I, bs):
    rng = np.random.default_rng(I)
    acc = rng.integers(-(1 << 22), 1 << 22, size=(9, 2 * I), dtype=np.int32)
    s3 = (rng.random(9) * 1e-4 + 1e-7).astype(np.float32)
    sw = (rng.random(2 * I) * 1e-2 + 1e-5).astype(np.float32)
    q, s = dg.swiglu_quant(cu(acc), cu(s3), cu(sw), bs)
    wq, ws = D.swiglu_quant(acc, s3, sw, bs)
    same(q, wq)
    same(s, ws)


def test_dequant_residual_against_oracle(dg):
    rng = np.random.default_rng(5)
    acc = rng.integers(-(1 << 26), 1 << 26, size=(33, 2048), dtype=np.int32)
    s = (rng.random(33) * 1e-4).astype(np.float32)
    sw = (rng.random(2048) * 1e-2).astype(np.float32)
    x = _rows(rng, 33, 2048)
    same(dg.dequant_residual(cu(acc), cu(s), cu(sw), cu(x)), D.dequant_residual(acc, s, sw, x))


@pytest.mark.parametrize("qk", [True, False])
def test_qkv_post_qwen3_heads_against_oracle(dg, qk):
    rng = np.random.default_rng(int(qk))
    T, B, H, Hkv, hd = 16, 2, 16, 8, 128
    N = B * T
    acc = rng.integers(-(1 << 22), 1 << 22, size=(N, (H + 2 * Hkv) * hd), dtype=np.int32)
    s1 = (rng.random(N) * 1e-4 + 1e-7).astype(np.float32)
    sw = (rng.random((H + 2 * Hkv) * hd) * 1e-2 + 1e-5).astype(np.float32)
    qnw = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    knw = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    ang = np.arange(64)[:, None] * (1.0 / (1e6 ** (np.arange(0, hd, 2) / hd)))[None, :]
    emb = np.concatenate([ang, ang], axis=1)
    cos, sin = np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)
    got = dg.qkv_post(cu(acc), cu(s1), cu(sw), cu(qnw), cu(knw), cu(cos), cu(sin), T, H, Hkv, 1e-6, qk)
    want = D.qkv_post(acc, s1, sw, qnw, knw, cos, sin, T, H, Hkv, 1e-6, qk)
    for a, b in zip(got, want):
        same(a, b)


class _Lin:
    """A DetLinear-shaped layer: Wq = quant_sym(fwht(W, bs), 64), sw folded with 1/sqrt(bs)."""

    def __init__(self, rng, n, k, bs):
        W = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        q, s = D.quant_act(W, bs)
        self.bs, self.Wq_np, self.sw_np = bs, q, s
        self.Wq, self.sw = cu(q), cu(s)


def test_mlp_block_matches_detrt_composition(dg):
    """rmsnorm_quant -> gate/up GEMM -> swiglu_quant -> down GEMM -> dequant_residual, end to end
    against the oracle's detrt composition (detrt/fast.py:182-189)."""
    rng = np.random.default_rng(9)
    D_, I, N = 1024, 2048, 40
    gu, down = _Lin(rng, 2 * I, D_, 512), _Lin(rng, D_, I, 512)
    wn = (1.0 + 0.1 * rng.standard_normal(D_)).astype(np.float32)
    r1 = _rows(rng, N, D_)
    got = dg.mlp_residual(gu, down, cu(wn), cu(r1), 1e-6)
    q3, s3 = D.rmsnorm_quant(r1, wn, 1e-6, 512)
    q4, s4 = D.swiglu_quant(O.gemm_i32(q3, gu.Wq_np), s3, gu.sw_np, 512)
    want = D.dequant_residual(O.gemm_i32(q4, down.Wq_np), s4, down.sw_np, r1)
    same(got, want)


def test_norm_linear_matches_oracle(dg):
    rng = np.random.default_rng(10)
    lin = _Lin(rng, 768, 2048, 128)
    wn = (1.0 + 0.1 * rng.standard_normal(2048)).astype(np.float32)
    x = _rows(rng, 50, 2048)
    got = dg.norm_linear(lin, cu(wn), cu(x), 1e-6)
    q, s = D.rmsnorm_quant(x, wn, 1e-6, 128)
    same(got, O.det_dequant(O.gemm_i32(q, lin.Wq_np), s, lin.sw_np))


def test_many_rows_path_matches_oracle(dg):
    """At least as many rows as SMs take the 256-thread row CTAs (fewer rows use 1024 threads)."""
    rng = np.random.default_rng(300)
    x = _rows(rng, 300, 2048)
    w = (1.0 + 0.2 * rng.standard_normal(2048)).astype(np.float32)
    q, s = dg.quant_act(cu(x), 512)
    wq, ws = D.quant_act(x, 512)
    same(q, wq)
    same(s, ws)
    q, s = dg.rmsnorm_quant(cu(x), cu(w), 1e-6, 128)
    wq, ws = D.rmsnorm_quant(x, w, 1e-6, 128)
    same(q, wq)
    same(s, ws)
    acc = rng.integers(-(1 << 22), 1 << 22, size=(300, 2 * 1024), dtype=np.int32)
    s3 = (rng.random(300) * 1e-4 + 1e-7).astype(np.float32)
    sw = (rng.random(2048) * 1e-2 + 1e-5).astype(np.float32)
    q, s = dg.swiglu_quant(cu(acc), cu(s3), cu(sw), 256)
    wq, ws = D.swiglu_quant(acc, s3, sw, 256)
    same(q, wq)
    same(s, ws)


@pytest.mark.parametrize("B,T,start,maxlen", [(8, 1, 2099, 2176), (2, 3, 10, 64), (3, 4, 62, 64)])
def test_qkv_post_kv_equals_post_at_then_append(dg, B, T, start, maxlen):
    """The decode step's fused qkv_post + KV-cache store == qkv_post_at followed by kv_append,
    including tokens whose cache position falls past maxlen (left unwritten by both)."""
    H, Hkv = 16, 8
    g = torch.Generator(device="cuda").manual_seed(B * 100 + T)
    N, width = B * T, (H + 2 * Hkv) * 128
    acc = torch.randint(-2 ** 20, 2 ** 20, (N, width), dtype=torch.int32, device="cuda", generator=g)
    s1 = torch.rand(N, device="cuda", generator=g) * 1e-3 + 1e-5
    sw = torch.rand(width, device="cuda", generator=g) * 1e-3 + 1e-5
    qnw = 1 + 0.1 * torch.randn(128, device="cuda", generator=g)
    knw = 1 + 0.1 * torch.randn(128, device="cuda", generator=g)
    ang = torch.arange(maxlen + 8, device="cuda")[:, None] * (1e-4 ** (torch.arange(64, device="cuda") / 64))[None]
    cos = torch.cat([torch.cos(ang), torch.cos(ang)], 1).float().contiguous()
    sin = torch.cat([torch.sin(ang), torch.sin(ang)], 1).float().contiguous()
    pos = torch.tensor([start], dtype=torch.int32, device="cuda")

    def cache():
        z = lambda *s, dt=torch.int8: torch.full(s, 7, dtype=dt, device="cuda")
        return dict(k=z(B, Hkv, maxlen, 128), sk=z(B, Hkv, maxlen, 1, dt=torch.float32),
                    v=z(B, Hkv, maxlen, 128), sv=z(B, Hkv, maxlen, 1, dt=torch.float32))

    want_c = cache()
    qq, qs, kq, ks, vq, vs = dg.qkv_post_at(acc, s1, sw, qnw, knw, cos, sin, pos, T, H, Hkv, 1e-6)
    dg.kv_append(kq, ks, vq, vs, want_c, B, T, pos)
    got_c = cache()
    qq2, qs2 = dg.qkv_post_kv(acc, s1, sw, qnw, knw, cos, sin, pos, T, H, Hkv, 1e-6, got_c)
    assert torch.equal(qq2, qq) and torch.equal(qs2.view(-1).view(torch.int32), qs.view(-1).view(torch.int32))
    for key in ("k", "v"):
        assert torch.equal(got_c[key], want_c[key]), key
    for key in ("sk", "sv"):
        assert torch.equal(got_c[key].view(torch.int32), want_c[key].view(torch.int32)), key
