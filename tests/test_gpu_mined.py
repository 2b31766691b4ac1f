"""The full mined path against the oracle (mirrors miner/ampere/tests/test_kernels.py:94-138,
test_proj_gemm.py and test_gemm_cfgs.py): exact output, identical winning tiles, identical
correction tensors across projection paths, CUDA-graph replay == eager."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(dev):
    from uwc_b200 import _lib, ops
    _lib.device_status(clear=True)
    yield ops
    assert _lib.device_status(clear=True) == 0, "a kernel reported a device-side timeout"


def _inputs(m, n, k, seed):
    rng = np.random.default_rng(seed)
    A = rng.integers(-64, 65, size=(m, k), dtype=np.int8)
    Bt = rng.integers(-64, 65, size=(n, k), dtype=np.int8)
    return A, Bt, rng.bytes(32)


def _expected(A, Bt, key, r, target):
    a_seed, b_seed, wins, msgs = O.mined_reference(A, Bt, key, r, target)
    return a_seed, wins


@pytest.mark.parametrize("m,n,k,r", [(256, 512, 2048, 128), (256, 512, 2048, 64), (128, 256, 1024, 64),
                                     (384, 768, 2048, 128), (128, 320, 1024, 256), (192, 256, 1024, 64)])
def test_mined_forward_exact_and_winners_match_oracle(ops, m, n, k, r):
    from uwc_b200 import glue
    A, Bt, key = _inputs(m, n, k, 7 + r)
    target = glue.target_for(m, n, 20)
    w = ops.MinedWeight(Bt=torch.from_numpy(Bt).cuda(), b_scale=torch.ones(n, device="cuda"), r=r, max_wins=4096)
    w.setup_block(key, target)
    out = w.forward(torch.from_numpy(A).cuda(), torch.ones(m, device="cuda"), out_mode=ops.OUT_I32)
    assert np.array_equal(out.cpu().numpy(), O.gemm_i32(A, Bt))
    a_seed, want = _expected(A, Bt, key, r, target)
    assert ops.words_to_bytes(w.buffers(m)["a_seed"]) == a_seed
    got = sorted(w.winners(m))
    assert want and got == want


@pytest.mark.parametrize("m,n,k,r", [(256, 512, 2048, 128), (512, 512, 1024, 64), (128, 256, 2048, 64),
                                     (384, 320, 1024, 128), (256, 256, 1024, 256)])
def test_noise_mine_winners_match_oracle(ops, m, n, k, r):
    from uwc_b200 import glue
    A, Bt, key = _inputs(m, n, k, 100 + m + r)
    target = glue.target_for(m, n, 20)
    w = ops.MinedWeight(Bt=torch.from_numpy(Bt).cuda(), b_scale=torch.ones(n, device="cuda"), r=r, max_wins=4096)
    w.setup_block(key, target)
    w.noise_mine(torch.from_numpy(A).cuda())
    _, want = _expected(A, Bt, key, r, target)
    assert want and sorted(w.winners(m)) == want


def test_golden_winners(ops, golden):
    """Winner sets produced by the reference's own reference.py (tests/golden)."""
    meta, _ = golden
    for c in meta["mined"]:
        m, n, k, r = c["m"], c["n"], c["k"], c["r"]
        rng = np.random.default_rng(c["seed"])
        A = rng.integers(-64, 65, size=(m, k), dtype=np.int8)
        Bt = rng.integers(-64, 65, size=(n, k), dtype=np.int8)
        key = rng.bytes(32)
        target = O.bound_words(int(c["bound"], 16))
        w = ops.MinedWeight(Bt=torch.from_numpy(Bt).cuda(), b_scale=torch.ones(n, device="cuda"), r=r, max_wins=4096)
        w.setup_block(key, target)
        out = w.forward(torch.from_numpy(A).cuda(), torch.ones(m, device="cuda"), out_mode=ops.OUT_I32)
        got = [[a, b, h.hex()] for a, b, h in sorted(w.winners(m))]
        assert got == c["winners"]
        assert O.sha20(out.cpu().numpy()) == c["out_sha"][:20]
        w.noise_mine(torch.from_numpy(A).cuda())
        assert [[a, b, h.hex()] for a, b, h in sorted(w.winners(m))] == c["winners"]


def test_projection_paths_identical(ops):
    """The forward's tensor-core projections (split-K GEMMs against S^T, then limbs) == the gather
    kernel of noise_rows with a projection permutation, limb for limb (test_proj_gemm.py:23-47)."""
    from uwc_b200 import glue
    for (n, k, m, r) in ((1024, 2048, 256, 128), (512, 4096, 128, 128), (512, 4096, 256, 64), (256, 2048, 128, 256)):
        A, Bt, key = _inputs(m, n, k, n + k + m)
        w = ops.MinedWeight(Bt=torch.from_numpy(Bt).cuda(), b_scale=torch.ones(n, device="cuda"), r=r)
        w.setup_block(key, glue.target_for(m, n))
        Ad = torch.from_numpy(A).cuda()
        out = w.forward(Ad, torch.ones(m, dtype=torch.float32, device="cuda"), out_mode=ops.OUT_I32)
        b = w.buffers(m)
        L = b["corrA"].shape[0]
        corrA = torch.zeros_like(b["corrA"])
        corrB = torch.zeros_like(b["corrB"])
        mx = torch.zeros(2, dtype=torch.int32, device="cuda")
        ops.noise_rows(Ad, m, k, r, E=b["EAL"], Pp=w.PB, corr=corrA, corr_off=0, ecopy_off=r, maxabs=mx[0:1])
        ops.noise_rows(w.BpEBt, n, k, r, E=w.EBRt, Pp=b["PA"], corr=corrB, corr_off=r, ecopy_off=0, maxabs=mx[1:2])
        for name, x, y in (("corrA", b["corrA"], corrA), ("corrB", b["corrB"], corrB), ("maxabs", b["maxabs"], mx)):
            assert torch.equal(x, y), (name, n, k, m, r, L)
        wins = sorted(w.winners(m))
        assert 0 < len(wins) < 64
        assert np.array_equal(out.cpu().numpy(), O.gemm_i32(A, Bt))


def test_large_projection_needs_more_limbs(ops):
    """An A aligned with P_B pushes |X| = |A P_B^T| past 8127, so the denoise must use 3 limbs."""
    m, n, k, r = 128, 256, 8192, 64
    rng = np.random.default_rng(21)
    Bt = rng.integers(-64, 65, size=(n, k), dtype=np.int8)
    key = bytes(range(32))
    b_seed = O.salted_seed(O.tree_root(Bt, key), n, O.SEED_SALT_B, key)
    PB = O.perm_matrix(O.SEED_LABEL_B, b_seed, k, r)
    A = rng.integers(-8, 9, size=(m, k), dtype=np.int8)
    A[:, PB[:, 0] == 0] = 64
    A[:, PB[:, 1] == 0] = -64
    assert O.projection(A, O.pack_perm(PB), r).max() > 8127
    w = ops.MinedWeight(Bt=torch.from_numpy(Bt).cuda(), b_scale=torch.ones(n, device="cuda"), r=r)
    w.setup_block(key, np.zeros(8, np.uint32))
    out = w.forward(torch.from_numpy(A).cuda(), torch.ones(m, device="cuda"), out_mode=ops.OUT_I32)
    assert int(w.buffers(m)["maxabs"].max().item()) > 8127
    assert np.array_equal(out.cpu().numpy(), O.gemm_i32(A, Bt))


def test_bf16_forward_matches_int_path(ops):
    """MinedWeight.forward(OUT_BF16) == RNE((float(A Bt^T) * a_scale) * b_scale) (kernels.cu:687-714)."""
    m, n, k, r = 256, 512, 2048, 128
    A, Bt, key = _inputs(m, n, k, 3)
    rng = np.random.default_rng(4)
    sa = (rng.random(m, dtype=np.float32) * 0.01).astype(np.float32)
    sb = (rng.random(n, dtype=np.float32) * 0.01).astype(np.float32)
    w = ops.MinedWeight(Bt=torch.from_numpy(Bt).cuda(), b_scale=torch.from_numpy(sb).cuda(), r=r)
    w.setup_block(key, np.zeros(8, np.uint32))
    out = w.forward(torch.from_numpy(A).cuda(), torch.from_numpy(sa).cuda())
    want = O.scaled_bf16(O.gemm_i32(A, Bt), sa, sb)
    assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), want)


def test_graphed_forward_matches_eager(ops):
    rng = np.random.default_rng(5)
    m, n, k = 256, 512, 2048
    A = torch.from_numpy(rng.integers(-64, 65, size=(m, k), dtype=np.int8)).cuda()
    Bt = torch.from_numpy(rng.integers(-64, 65, size=(n, k), dtype=np.int8)).cuda()
    w = ops.MinedWeight(Bt=Bt, b_scale=torch.ones(n, device="cuda"))
    w.setup_block(rng.bytes(32), np.zeros(8, np.uint32))
    gf = ops.GraphedForward(w, m, out_mode=ops.OUT_I32)
    gf.A.copy_(A)
    got = gf().clone()
    assert np.array_equal(got.cpu().numpy(), O.gemm_i32(A.cpu().numpy(), Bt.cpu().numpy()))


def test_win_overflow_counts_past_max(ops):
    """Every tile wins at target = 2^256-1: the count keeps counting, records stop at max_wins."""
    m, n, k, r = 128, 256, 1024, 128
    A, Bt, key = _inputs(m, n, k, 9)
    w = ops.MinedWeight(Bt=torch.from_numpy(Bt).cuda(), b_scale=torch.ones(n, device="cuda"), r=r, max_wins=16)
    w.setup_block(key, O.bound_words((1 << 256) - 1))
    w.noise_mine(torch.from_numpy(A).cuda())
    assert w.win_count(m) == m * n // 128
    assert len(w.winners(m)) == 16


def test_det_linear(ops):
    """DetLinear.int_gemm and the fused fp32 dequant (qwen3.py:106-126) at the C1 shape."""
    from uwc_b200 import det
    rng = np.random.default_rng(0)
    q = rng.integers(-127, 128, (256, 2048), dtype=np.int8)
    Wq = rng.integers(-64, 65, (6144, 2048), dtype=np.int8)
    sx = (rng.random(256, dtype=np.float32) * 0.01).astype(np.float32)
    sw = (rng.random(6144, dtype=np.float32) * 0.001).astype(np.float32)
    acc = det.int_gemm(torch.from_numpy(q).cuda(), torch.from_numpy(Wq).cuda())
    want = O.gemm_i32_blas(q, Wq)
    assert np.array_equal(acc.cpu().numpy(), want)
    y = det.linear_f32(torch.from_numpy(q).cuda(), torch.from_numpy(sx).cuda(), torch.from_numpy(Wq).cuda(),
                       torch.from_numpy(sw).cuda())
    assert np.array_equal(y.cpu().numpy().view(np.uint32), O.det_dequant(want, sx, sw).view(np.uint32))


@pytest.mark.parametrize("r", [64, 128])
def test_full_size_mining_every_tile_sampled_against_oracle(ops, r):
    """The hashed GEMM at the headline shape (8192 x 14336 x 4096): every SM processes a dozen
    units, so message-buffer reuse and the persistent schedule are exercised. With a target that
    every hash meets, each 64 x 64 block yields its 32 tiles exactly once; the tiles of sampled
    blocks (corners, edges, interior) hash exactly as the oracle's fold of that block."""
    m, n, k = 8192, 14336, 4096
    g = torch.Generator(device="cuda").manual_seed(5 + r)
    A = torch.randint(-64, 65, (m, k), dtype=torch.int8, device="cuda", generator=g)
    B = torch.randint(-64, 65, (n, k), dtype=torch.int8, device="cuda", generator=g)
    key = bytes(range(32))
    keyw = torch.from_numpy(O.words(key).view(np.int32).copy()).cuda()
    tgt = torch.full((8,), -1, dtype=torch.int32, device="cuda")
    ntiles = (m // 64) * (n // 64) * 32
    wins = torch.zeros(1 + ntiles * 10, dtype=torch.int32, device="cuda")
    ops.gemm(A, B, r=r, flags=1, key=keyw, target=tgt, wins=wins, max_wins=ntiles)
    w = wins.cpu().numpy().view(np.uint32)
    assert int(w[0]) == ntiles
    recs = w[1:].reshape(ntiles, 10)
    rows, cols = recs[:, 0].astype(np.int64), recs[:, 1].astype(np.int64)
    # tile (g, t) of block (rb, cb) is reported at row 64 rb + g, col 64 cb + 2 t
    assert np.all(rows < m) and np.all(cols < n) and np.all((rows % 64) < 8) and np.all((cols % 64) < 8)
    assert np.all(cols % 2 == 0)
    ids = rows * n + cols
    assert len(np.unique(ids)) == ntiles
    by_id = {int(i): recs[j, 2:] for j, i in enumerate(ids)}
    An, Bn = A.cpu().numpy(), B.cpu().numpy()
    rng = np.random.default_rng(r)
    blocks = [(0, 0), (m // 64 - 1, n // 64 - 1), (0, n // 64 - 1), (m // 64 - 1, 0)]
    blocks += [(int(a), int(b)) for a, b in zip(rng.integers(0, m // 64, 8), rng.integers(0, n // 64, 8))]
    for rb, cb in blocks:
        msgs = O.jackpot_msgs(An[rb * 64:(rb + 1) * 64], Bn[cb * 64:(cb + 1) * 64], r)
        for gg in range(8):
            for t in range(4):
                want = O.jackpot_hash(msgs[0, gg, 0, t], key)
                got = by_id[(rb * 64 + gg) * n + cb * 64 + 2 * t].astype("<u4").tobytes()
                assert got == want, (rb, cb, gg, t)


@pytest.mark.parametrize("mode", ["i32", "bf16", "f32"])
def test_hashed_gemm_outputs_without_denoise(ops, mode):
    """FLAG_HASH with an output and no denoise (the mining pass stores the product, a second pass
    scales it): exact / RNE outputs, and the same winning tiles as the output-free mining call."""
    rng = np.random.default_rng(77)
    m, n, k, r = 384, 640, 1024, 64
    A = rng.integers(-64, 65, size=(m, k), dtype=np.int8)
    B = rng.integers(-64, 65, size=(n, k), dtype=np.int8)
    sa = (rng.random(m, dtype=np.float32) * 0.01 + 1e-4).astype(np.float32)
    sb = (rng.random(n, dtype=np.float32) * 0.02 + 1e-4).astype(np.float32)
    key = rng.bytes(32)
    keyw = torch.from_numpy(O.words(key).view(np.int32).copy()).cuda()
    from uwc_b200 import glue
    tgt = torch.from_numpy(glue.target_for(m, n, 20).view(np.int32).copy()).cuda()
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    w0 = torch.zeros(1 + 4096 * 10, dtype=torch.int32, device="cuda")
    w1 = torch.zeros_like(w0)
    ops.gemm(Ad, Bd, r=r, flags=1, key=keyw, target=tgt, wins=w0, max_wins=4096)
    dt = {"i32": torch.int32, "bf16": torch.bfloat16, "f32": torch.float32}[mode]
    om = {"i32": ops.OUT_I32, "bf16": ops.OUT_BF16, "f32": ops.OUT_F32}[mode]
    out = torch.empty((m, n), dtype=dt, device="cuda")
    ops.gemm(Ad, Bd, r=r, flags=1, key=keyw, target=tgt, wins=w1, max_wins=4096, a_scale=torch.from_numpy(sa).cuda(),
             b_scale=torch.from_numpy(sb).cuda(), out=out, out_mode=om)

    def recs(w):
        h = w.cpu().numpy().view(np.uint32)
        return sorted(map(tuple, h[1:1 + int(h[0]) * 10].reshape(-1, 10).tolist()))
    assert int(w0[0]) > 0 and recs(w0) == recs(w1)
    acc = O.gemm_i32(A, B)
    if mode == "i32":
        assert np.array_equal(out.cpu().numpy(), acc)
    elif mode == "bf16":
        assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), O.scaled_bf16(acc, sa, sb))
    else:
        assert np.array_equal(out.cpu().numpy().view(np.uint32), O.det_dequant(acc, sa, sb).view(np.uint32))


@pytest.mark.gpu
def test_host_miner_matches_noise_mine(dev):
    """HostMiner (overlapped uploads from pinned memory) reports the same winners per attempt as
    noise_mine on device-resident inputs."""
    import torch

    from uwc_b200 import glue, ops
    m, n, k, r = 256, 512, 2048, 64
    rng = np.random.default_rng(5)
    Bt = torch.from_numpy(rng.integers(-64, 65, (n, k), dtype=np.int8)).to(dev)
    w = ops.MinedWeight(Bt=Bt, b_scale=torch.ones(n, device=dev), r=r, max_wins=4096)
    w.setup_block(rng.bytes(32), glue.target_for(m, n, 20))
    As = [rng.integers(-64, 65, (m, k), dtype=np.int8) for _ in range(4)]
    want = []
    for A in As:
        w.noise_mine(torch.from_numpy(A).to(dev))
        want.append(sorted(w.winners(m)))
    hm = ops.HostMiner(w, m, k, dev)
    hosts = [torch.from_numpy(A).pin_memory() for A in As]
    outs = [torch.empty(w.buffers(m)["wins"].numel(), dtype=torch.int32).pin_memory() for _ in As]
    for A_h, o in zip(hosts, outs):
        hm.mine(A_h, o)
    torch.cuda.synchronize()
    for o, ww in zip(outs, want):
        words = o.numpy().view(np.uint32)
        cnt = min(int(words[0]), w.max_wins)
        recs = words[1:1 + cnt * ops.WIN_WORDS].reshape(cnt, ops.WIN_WORDS)
        got = sorted((int(x[0]), int(x[1]), x[2:].astype("<u4").tobytes()) for x in recs)
        assert got == ww and ww
