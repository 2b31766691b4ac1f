"""Pin the CPU oracle against the reference's golden vectors before trusting it.

The vectors in tests/golden/ were produced by the reference's own reference.py
(tests/golden/make_golden.py); the L1 digest is the one the reference published in
results/xc_cpu.json (bench/crosscheck.py:66-76 inputs).
"""
import hashlib

import numpy as np
import pytest

import oracle as O


def sha(x):
    return hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest()


def test_blake3_against_package_shapes():
    blake3 = pytest.importorskip("blake3").blake3
    rng = np.random.default_rng(0)
    for n in (0, 1, 64, 1024, 1025, 4096, 70000):
        d = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        key = rng.bytes(32)
        assert O.blake3(d) == blake3(d).digest()
        assert O.keyed(key, d) == blake3(d, key=key).digest()


def test_tree_roots(golden):
    meta, _ = golden
    for nchunks, want in meta["tree_roots"]:
        rng = np.random.default_rng(nchunks)
        data = rng.integers(0, 256, size=nchunks * 1024, dtype=np.uint8)
        key = rng.bytes(32)
        assert O.tree_root(data, key).hex() == want, nchunks


def test_salts_and_seed_derivation(golden):
    meta, _ = golden
    s = meta["seeds"]
    assert O.SEED_SALT_A.hex() == s["salt_a"] and O.SEED_SALT_B.hex() == s["salt_b"]
    rng = np.random.default_rng(s["seed"])
    A = rng.integers(-64, 65, size=(s["m"], s["k"]), dtype=np.int8)
    Bt = rng.integers(-64, 65, size=(s["n"], s["k"]), dtype=np.int8)
    job_key = rng.bytes(32)
    a_seed, b_seed, ha, hb = O.commitment(job_key, A, Bt)
    assert (a_seed.hex(), b_seed.hex(), ha.hex(), hb.hex()) == (s["a_seed"], s["b_seed"], s["root_a"], s["root_b"])


def test_noise_generation(golden):
    meta, arr = golden
    key = bytes.fromhex(meta["noise_key"])
    for rows, r, k in ((256, 128, 3072), (256, 64, 4096)):
        assert np.array_equal(O.uniform_matrix(O.SEED_LABEL_A, key, rows, r), arr[f"uniform_r{r}"])
        assert np.array_equal(O.perm_matrix(O.SEED_LABEL_B, key, k, r), arr[f"perm_r{r}"])


def test_noise_rows(golden):
    meta, arr = golden
    nr = meta["noise_rows"]
    A, E, Pn, Pp = arr["nr_A"], arr["nr_E"], arr["nr_Pn"], arr["nr_Pp"]
    rows, k, r = nr["rows"], nr["k"], nr["r"]
    L = O.limbs_for(k)
    corr = np.zeros((L, rows, 2 * r), np.int8)
    mx = np.zeros(1, np.int32)
    dst = O.noise_rows(A, r, E=E, Pn=O.pack_perm(Pn), want_dst=True, Pp=O.pack_perm(Pp), corr=corr, corr_off=0,
                       ecopy_off=r, maxabs=mx)
    assert sha(dst) == nr["dst_sha"]
    proj = sum(corr[li, :, :r].astype(np.int64) * 128 ** li for li in range(L))
    assert sha(proj) == nr["proj_sha"]
    assert int(mx[0]) == nr["maxabs"]
    for li in range(L):
        assert np.array_equal(corr[li, :, r:], E)
    assert np.array_equal(O.projection(A, O.pack_perm(Pp), r), proj)


def test_limbs_for():
    # ops.py:18-24: balanced base-128 limbs covering 127 * k
    assert [O.limbs_for(k) for k in (1, 64, 4096, 8192, 1 << 20)] == [2, 3, 3, 4, 5]
    for k in (64, 1024, 4096, 16384, 1 << 20):
        L = O.limbs_for(k)
        cap = 63
        for _ in range(L - 1):
            cap = cap * 128 + 63
        assert cap >= 127 * k
        assert L == 1 or (cap - 63) // 128 < 127 * k


def test_jackpot_and_winners(golden):
    meta, arr = golden
    for c in meta["mined"]:
        m, n, k, r = c["m"], c["n"], c["k"], c["r"]
        rng = np.random.default_rng(c["seed"])
        A = rng.integers(-64, 65, size=(m, k), dtype=np.int8)
        Bt = rng.integers(-64, 65, size=(n, k), dtype=np.int8)
        job_key = rng.bytes(32)
        assert job_key.hex() == c["job_key"]
        a_seed, b_seed, wins, msgs = O.mined_reference(A, Bt, job_key, r, O.bound_words(int(c["bound"], 16)))
        assert a_seed.hex() == c["a_seed"] and b_seed.hex() == c["b_seed"]
        assert np.array_equal(msgs, arr[f"msgs_{m}_{n}_{k}_{r}"])
        assert [[a, b, h.hex()] for a, b, h in wins] == c["winners"]
        assert sha(O.gemm_i32(A, Bt)) == c["out_sha"]


def test_published_L1_digest(golden):
    """results/xc_cpu.json L1_gemm_int32: sha256[:20] of int32 A Bt^T (crosscheck.py:62-76)."""
    meta, _ = golden
    rng = np.random.default_rng(2026)
    A = rng.integers(-64, 65, size=(1024, 4096), dtype=np.int8)
    Bt = rng.integers(-64, 65, size=(3072, 4096), dtype=np.int8)
    C = O.gemm_i32_blas(A, Bt)
    assert O.sha20(C) == meta["xc_cpu"]["L1_gemm_int32"] == "bf9394d180bda5b0412c"


def test_published_L2_quantizer_digests(golden):
    """results/xc_cpu.json L2_q_bs*/L2_scale_bs*: the fused quantizer on crosscheck.py:86-97 inputs."""
    meta, _ = golden
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(2026)
    rng.integers(-64, 65, size=(1024, 4096), dtype=np.int8)
    rng.integers(-64, 65, size=(3072, 4096), dtype=np.int8)
    x = rng.standard_normal((1024, 4096)).astype(np.float32) * np.linspace(0.05, 6, 4096, dtype=np.float32)
    x[:, 7] *= 40.0
    xb = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    for bs in (0, 128, 512):
        q, s = O.quant_rows_had(xb, bs)
        assert O.sha20(q) == meta["xc_cpu"][f"L2_q_bs{bs}"], bs
        assert O.sha20(s) == meta["xc_cpu"][f"L2_scale_bs{bs}"], bs


def test_target_helpers():
    # pearl_glue.py:48-66
    assert O.nbits_to_target(0x1D00FFFF) == 0xFFFF << (8 * (0x1D - 3))
    assert O.nbits_to_target(0x03123456) == 0x123456
    assert O.nbits_to_target(0x01800000) == 0
    w = O.bound_words((1 << 256) - 1)
    assert w.dtype == np.uint32 and (w == 0xFFFFFFFF).all()
