"""Each sm_100a kernel against the CPU oracle, bit-exact (mirrors miner/ampere/tests/test_kernels.py).

All calls go through the C ABI (libuwcb200.so) via uwc_b200.ops."""
import hashlib

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def sha(x):
    return hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def ops(dev):
    from uwc_b200 import _lib, ops
    _lib.device_status(clear=True)
    yield ops
    assert _lib.device_status(clear=True) == 0, "a kernel reported a device-side timeout"


@pytest.mark.parametrize("nchunks", [1, 2, 3, 63, 64, 65, 127, 128, 129, 130, 1000, 4097, 65536, 131073, 300_001])
def test_tree_hash_matches_blake3(ops, nchunks):
    blake3 = pytest.importorskip("blake3").blake3
    rng = np.random.default_rng(nchunks)
    data = rng.integers(0, 256, size=nchunks * 1024, dtype=np.uint8)
    key = rng.bytes(32)
    root = torch.zeros(8, dtype=torch.int32, device="cuda")
    ops.b3_root_and_seed(torch.from_numpy(data).cuda(), ops.words(key), root_out=root)
    assert ops.words_to_bytes(root) == blake3(data.tobytes(), key=key).digest()


def test_seed_derivation_matches_reference(ops, golden):
    meta, _ = golden
    s = meta["seeds"]
    rng = np.random.default_rng(s["seed"])
    A = rng.integers(-64, 65, size=(s["m"], s["k"]), dtype=np.int8)
    Bt = rng.integers(-64, 65, size=(s["n"], s["k"]), dtype=np.int8)
    job_key = rng.bytes(32)
    jk = ops.words(job_key)
    bs = torch.zeros(8, dtype=torch.int32, device="cuda")
    ops.b3_root_and_seed(torch.from_numpy(Bt).cuda().view(-1), jk, prefix=jk, salt=ops.SALT_B.cuda(), dim=s["n"],
                         seed_out=bs)
    assert ops.words_to_bytes(bs).hex() == s["b_seed"]
    as_ = torch.zeros(8, dtype=torch.int32, device="cuda")
    ops.b3_root_and_seed(torch.from_numpy(A).cuda().view(-1), jk, prefix=bs, salt=ops.SALT_A.cuda(), dim=s["m"],
                         seed_out=as_)
    assert ops.words_to_bytes(as_).hex() == s["a_seed"]


def test_noise_generation_matches_reference(ops, golden):
    meta, arr = golden
    key = bytes.fromhex(meta["noise_key"])
    for rows, r, k in ((256, 128, 3072), (256, 64, 4096)):
        E = torch.empty((rows, r), dtype=torch.int8, device="cuda")
        ops.noise_uniform(E, ops.LABEL_A.cuda(), ops.words(key))
        assert np.array_equal(E.cpu().numpy(), arr[f"uniform_r{r}"])
        P = torch.empty(k, dtype=torch.int32, device="cuda")
        ops.noise_perm(P, k, r, ops.LABEL_B.cuda(), ops.words(key))
        p = P.cpu().numpy().view(np.uint32)
        want = arr[f"perm_r{r}"]
        assert np.array_equal(p & 0xFFFF, want[:, 0]) and np.array_equal(p >> 16, want[:, 1])


def test_noise_uniform_zeroes_counters(ops):
    z = torch.full((5,), 7, dtype=torch.int32, device="cuda")
    E = torch.empty((64, 64), dtype=torch.int8, device="cuda")
    ops.noise_uniform(E, ops.LABEL_A.cuda(), ops.words(bytes(32)), zero_me=z, zero_n=5)
    assert z.cpu().tolist() == [0] * 5


def test_noise_rows_noising_and_projection(ops, golden):
    meta, arr = golden
    nr = meta["noise_rows"]
    A, E, Pn, Pp = arr["nr_A"], arr["nr_E"], arr["nr_Pn"], arr["nr_Pp"]
    rows, k, r = nr["rows"], nr["k"], nr["r"]
    pack = lambda P: torch.from_numpy(O.pack_perm(P).view(np.int32)).cuda()
    dst = torch.empty((rows, k), dtype=torch.int8, device="cuda")
    L = ops.limbs_for(k)
    corr = torch.zeros((L, rows, 2 * r), dtype=torch.int8, device="cuda")
    mx = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.noise_rows(torch.from_numpy(A).cuda(), rows, k, r, E=torch.from_numpy(E).cuda(), Pn=pack(Pn), dst=dst,
                   Pp=pack(Pp), corr=corr, corr_off=0, ecopy_off=r, maxabs=mx)
    assert sha(dst.cpu().numpy()) == nr["dst_sha"]
    c = corr.cpu().numpy()
    proj = sum(c[li, :, :r].astype(np.int64) * 128 ** li for li in range(L))
    assert sha(proj) == nr["proj_sha"]
    assert int(mx.item()) == nr["maxabs"]
    for li in range(L):
        assert np.array_equal(c[li, :, r:], E)


@pytest.mark.parametrize("r", [64, 128, 256])
def test_noise_rows_ranks_against_oracle(ops, r):
    rng = np.random.default_rng(r)
    rows, k = 64, 4096
    A = rng.integers(-64, 65, size=(rows, k), dtype=np.int8)
    E = rng.integers(-32, 32, size=(rows, r), dtype=np.int8)
    Pn = O.perm_packed(O.SEED_LABEL_A, rng.bytes(32), k, r)
    Pp = O.perm_packed(O.SEED_LABEL_B, rng.bytes(32), k, r)
    L = O.limbs_for(k)
    want_corr = np.zeros((L, rows, 2 * r), np.int8)
    want_mx = np.zeros(1, np.int32)
    want_dst = O.noise_rows(A, r, E=E, Pn=Pn, want_dst=True, Pp=Pp, corr=want_corr, corr_off=0, ecopy_off=r,
                            maxabs=want_mx)
    t = lambda x: torch.from_numpy(x.view(np.int32) if x.dtype == np.uint32 else x).cuda()
    dst = torch.empty((rows, k), dtype=torch.int8, device="cuda")
    corr = torch.zeros((L, rows, 2 * r), dtype=torch.int8, device="cuda")
    mx = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.noise_rows(t(A), rows, k, r, E=t(E), Pn=t(Pn), dst=dst, Pp=t(Pp), corr=corr, corr_off=0, ecopy_off=r, maxabs=mx)
    assert np.array_equal(dst.cpu().numpy(), want_dst)
    assert np.array_equal(corr.cpu().numpy(), want_corr)
    assert int(mx.item()) == int(want_mx[0])


@pytest.mark.parametrize("rows,k,r,ecopy", [(8, 1024, 64, False), (200, 1040, 64, True), (8192, 4096, 64, False),
                                            (40000, 64, 128, True), (1776, 272, 256, True)])
def test_noise_add_against_oracle(ops, rows, k, r, ecopy):
    """The noising-only kernel (no projection): persistent CTAs with uneven row shares, shares longer
    than one staged group (40000 rows), and the E copy into every correction limb."""
    rng = np.random.default_rng(rows + k + r)
    A = rng.integers(-64, 65, size=(rows, k), dtype=np.int8)
    E = rng.integers(-32, 32, size=(rows, r), dtype=np.int8)
    Pn = O.perm_packed(O.SEED_LABEL_A, rng.bytes(32), k, r)
    L = 2 if ecopy else 0
    want_corr = np.zeros((L, rows, 2 * r), np.int8) if ecopy else None
    want_dst = O.noise_rows(A, r, E=E, Pn=Pn, want_dst=True, corr=want_corr, ecopy_off=r if ecopy else -1)
    t = lambda x: torch.from_numpy(x.view(np.int32) if x.dtype == np.uint32 else x).cuda()
    dst = torch.empty((rows, k), dtype=torch.int8, device="cuda")
    corr = torch.zeros((L, rows, 2 * r), dtype=torch.int8, device="cuda") if ecopy else None
    ops.noise_rows(t(A), rows, k, r, E=t(E), Pn=t(Pn), dst=dst, corr=corr, ecopy_off=r if ecopy else -1)
    assert np.array_equal(dst.cpu().numpy(), want_dst)
    if ecopy:
        assert np.array_equal(corr.cpu().numpy(), want_corr)


def test_proj_matrix_and_tensor_core_projection(ops):
    rng = np.random.default_rng(11)
    rows, k, r = 256, 2048, 128
    A = rng.integers(-64, 65, size=(rows, k), dtype=np.int8)
    P = O.perm_packed(O.SEED_LABEL_B, rng.bytes(32), k, r)
    Pt = torch.from_numpy(P.view(np.int32)).cuda()
    St = ops.proj_matrix(Pt, k, r)
    S = St.cpu().numpy().astype(np.int64)
    assert np.array_equal(A.astype(np.int64) @ S.T, O.projection(A, P, r))
    L = ops.limbs_for(k)
    corr = torch.zeros((L, rows, 2 * r), dtype=torch.int8, device="cuda")
    mx = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.project(torch.from_numpy(A).cuda(), St, corr, 0, mx)
    want_corr = np.zeros((L, rows, 2 * r), np.int8)
    want_mx = np.zeros(1, np.int32)
    O.noise_rows(A, r, Pp=P, corr=want_corr, corr_off=0, maxabs=want_mx)
    assert np.array_equal(corr.cpu().numpy()[:, :, :r], want_corr[:, :, :r])
    assert int(mx.item()) == int(want_mx[0])


@pytest.mark.parametrize("m,n,k", [(128, 256, 1024), (256, 512, 2048), (384, 768, 4096), (128, 256, 128),
                                   (32, 6144, 2048), (200, 320, 1040), (1, 64, 64), (4096, 256, 256)])
def test_plain_gemm_matches_oracle(ops, m, n, k):
    rng = np.random.default_rng(m + n + k)
    A = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    B = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    out = torch.full((m, n), -7, dtype=torch.int32, device="cuda")
    ops.gemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), out=out, out_mode=ops.OUT_I32)
    assert np.array_equal(out.cpu().numpy(), O.gemm_i32(A, B))


def test_published_L1_digest(ops, golden):
    """results/xc_cpu.json L1_gemm_int32 = bf9394d180bda5b0412c, on the GPU through the C ABI."""
    meta, _ = golden
    rng = np.random.default_rng(2026)
    A = rng.integers(-64, 65, size=(1024, 4096), dtype=np.int8)
    Bt = rng.integers(-64, 65, size=(3072, 4096), dtype=np.int8)
    out = torch.empty((1024, 3072), dtype=torch.int32, device="cuda")
    ops.gemm(torch.from_numpy(A).cuda(), torch.from_numpy(Bt).cuda(), out=out, out_mode=ops.OUT_I32)
    assert O.sha20(out.cpu().numpy()) == meta["xc_cpu"]["L1_gemm_int32"]


@pytest.mark.parametrize("mode", ["bf16", "f32"])
def test_scaled_epilogues(ops, mode):
    rng = np.random.default_rng(5)
    m, n, k = 256, 512, 1024
    A = rng.integers(-64, 65, size=(m, k), dtype=np.int8)
    B = rng.integers(-64, 65, size=(n, k), dtype=np.int8)
    sa = (rng.random(m, dtype=np.float32) * 0.01 + 1e-4).astype(np.float32)
    sb = (rng.random(n, dtype=np.float32) * 0.02 + 1e-4).astype(np.float32)
    acc = O.gemm_i32(A, B)
    if mode == "bf16":
        out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
        ops.gemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), a_scale=torch.from_numpy(sa).cuda(),
                 b_scale=torch.from_numpy(sb).cuda(), out=out, out_mode=ops.OUT_BF16)
        assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), O.scaled_bf16(acc, sa, sb))
    else:
        out = torch.empty((m, n), dtype=torch.float32, device="cuda")
        ops.gemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), a_scale=torch.from_numpy(sa).cuda(),
                 b_scale=torch.from_numpy(sb).cuda(), out=out, out_mode=ops.OUT_F32)
        assert np.array_equal(out.cpu().numpy().view(np.uint32), O.det_dequant(acc, sa, sb).view(np.uint32))


@pytest.mark.parametrize("m,n,k", [(32, 768, 4096), (1, 512, 1024), (7, 4096, 14336 // 2), (32, 14336, 4096),
                                   (96, 256, 128 * 3 + 16)])
@pytest.mark.parametrize("mode", ["i32", "f32", "bf16"])
def test_skinny_split_k_gemm(ops, m, n, k, mode):
    """Decode-sized GEMMs take the split-K schedule (int32 partials added into the product):
    exact int32, and the fp32 / bf16 epilogues applied once to the summed product."""
    rng = np.random.default_rng(m * 7 + n + k)
    A = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    B = rng.integers(-64, 65, size=(n, k), dtype=np.int8)
    acc = O.gemm_i32(A, B)
    sa = (rng.random(m, dtype=np.float32) * 0.01 + 1e-4).astype(np.float32)
    sb = (rng.random(n, dtype=np.float32) * 0.02 + 1e-4).astype(np.float32)
    dt = {"i32": torch.int32, "f32": torch.float32, "bf16": torch.bfloat16}[mode]
    om = {"i32": ops.OUT_I32, "f32": ops.OUT_F32, "bf16": ops.OUT_BF16}[mode]
    out = torch.full((m, n), 7, dtype=dt, device="cuda")
    ops.gemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), a_scale=torch.from_numpy(sa).cuda(),
             b_scale=torch.from_numpy(sb).cuda(), out=out, out_mode=om)
    if mode == "i32":
        assert np.array_equal(out.cpu().numpy(), acc)
    elif mode == "f32":
        assert np.array_equal(out.cpu().numpy().view(np.uint32), O.det_dequant(acc, sa, sb).view(np.uint32))
    else:
        assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), O.scaled_bf16(acc, sa, sb))
