"""Generate the golden vectors the oracle is pinned against, from the reference's own code.

Run in a container where the reference checkout is available (it is NOT needed on the GPU box):

    python tests/golden/make_golden.py --reference <path to useful-work-coin checkout>

It imports miner/ampere/uwc_ampere/reference.py (the reference's line-by-line port of Pearl's
rules: commitment, noise, jackpot fold, tile hash) and the `blake3` package, runs them on
seeded inputs that mirror the reference's tests (miner/ampere/tests/test_kernels.py:13-125,
test_reference_vs_pearl.py:18-40), and writes tests/golden/golden.npz plus golden.json.
Large arrays are stored as sha256 digests; small ones verbatim. The job key is a seeded
32-byte string standing in for Pearl's header hash (pearl_mining is not available here).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def sha(x) -> str:
    return hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("UWC_REFERENCE"), required="UWC_REFERENCE" not in os.environ)
    a = ap.parse_args()
    sys.path.insert(0, os.path.join(a.reference, "miner", "ampere"))
    import torch
    from blake3 import blake3
    from uwc_ampere import reference as ref  # the reference's oracle

    out, meta = {}, {}

    # 1. keyed BLAKE3 tree roots over 1 KiB-padded data (test_kernels.py:13-20 sizes, capped)
    roots = []
    for nchunks in (1, 2, 3, 63, 64, 65, 130, 1000, 4097):
        rng = np.random.default_rng(nchunks)
        data = rng.integers(0, 256, size=nchunks * 1024, dtype=np.uint8)
        key = rng.bytes(32)
        roots.append([nchunks, blake3(data.tobytes(), key=key).hexdigest()])
    meta["tree_roots"] = roots

    # 2. salted seed derivation (test_kernels.py:23-36)
    rng = np.random.default_rng(1)
    m, n, k = 256, 512, 2048
    A = rng.integers(-64, 65, size=(m, k), dtype=np.int8)
    Bt = rng.integers(-64, 65, size=(n, k), dtype=np.int8)
    job_key = rng.bytes(32)
    a_seed, b_seed, ha, hb = ref.commitment(job_key, A, Bt, salted=True)
    meta["seeds"] = dict(seed=1, m=m, n=n, k=k, a_seed=a_seed.hex(), b_seed=b_seed.hex(), root_a=ha.hex(),
                         root_b=hb.hex(), salt_a=ref.SEED_SALT_A.hex(), salt_b=ref.SEED_SALT_B.hex())

    # 3. noise generation (test_kernels.py:39-50), r = 128 and the BASELINE rank 64
    rng = np.random.default_rng(2)
    key = rng.bytes(32)
    for rows, r, kk in ((256, 128, 3072), (256, 64, 4096)):
        E = ref.uniform_matrix(ref.SEED_LABEL_A, key, rows, r)
        P = ref.perm_matrix(ref.SEED_LABEL_B, key, kk, r)
        out[f"uniform_r{r}"] = E
        out[f"perm_r{r}"] = P
    meta["noise_key"] = key.hex()

    # 4. noise_rows: noising + projection limbs + maxabs (test_kernels.py:58-81 inputs)
    rng = np.random.default_rng(3)
    rows, k, r = 128, 2048, 128
    A = rng.integers(-64, 65, size=(rows, k), dtype=np.int8)
    E = rng.integers(-32, 32, size=(rows, r), dtype=np.int8)
    Pn = ref.perm_matrix(ref.SEED_LABEL_A, b"\x01" * 32, k, r)
    Pp = ref.perm_matrix(ref.SEED_LABEL_B, b"\x02" * 32, k, r)
    noised = (A.astype(np.int16) + E[:, Pn[:, 0]] - E[:, Pn[:, 1]]).astype(np.int8)
    proj = np.zeros((rows, r), dtype=np.int64)
    for l in range(k):
        proj[:, Pp[l, 0]] += A[:, l]
        proj[:, Pp[l, 1]] -= A[:, l]
    out["nr_A"], out["nr_E"], out["nr_Pn"], out["nr_Pp"] = A, E, Pn, Pp
    meta["noise_rows"] = dict(rows=rows, k=k, r=r, dst_sha=sha(noised), proj_sha=sha(proj),
                              maxabs=int(np.abs(proj).max()))

    # 5. jackpot messages + winners on mined inputs, r = 128 (the reference default) and 64
    cases = []
    for (m, n, k, r, seed) in ((128, 256, 2048, 128, 7), (256, 256, 1024, 64, 8), (128, 128, 2048, 64, 9)):
        rng = np.random.default_rng(seed)
        A = rng.integers(-64, 65, size=(m, k), dtype=np.int8)
        Bt = rng.integers(-64, 65, size=(n, k), dtype=np.int8)
        job_key = rng.bytes(32)
        a_seed, b_seed, _, _ = ref.commitment(job_key, A, Bt, salted=True)
        nz = ref.noise(k, r, a_seed, b_seed, m, n)
        ApEA = (A.astype(np.int16) + nz["noise_a"]).astype(np.int8)
        BpEBt = (Bt.astype(np.int16) + nz["noise_bt"]).astype(np.int8)
        msgs = ref.jackpot_all_tiles(torch.from_numpy(ApEA), torch.from_numpy(BpEBt), r, None, None, 64,
                                     64).numpy().astype(np.uint32)
        # bound giving about 12 winners (the reference's own target_for, test_proj_gemm.py:17-20)
        bound = ((1 << 256) - 1) * 12 // ((m // 8) * (n // 16))
        wins = []
        for (rb, g, cb, t) in np.ndindex(msgs.shape[:4]):
            h = ref.jackpot_hash(list(msgs[rb, g, cb, t]), a_seed)
            if int.from_bytes(h, "little") <= bound:
                wins.append([rb * 64 + g, cb * 64 + 2 * t, h.hex()])
        # spot check of the batched fold against the per-tile form (test_reference_vs_pearl.py:18-27)
        rows_ = [g0 + 8 * i for g0 in (0,) for i in range(8)]
        cols_ = sorted([8 * j + e for j in range(8) for e in (0, 1)])
        want = ref.jackpot_msg_tile(ApEA[rows_].astype(np.int64), BpEBt[cols_].astype(np.int64), r)
        assert list(msgs[0, 0, 0, 0]) == want
        cases.append(dict(m=m, n=n, k=k, r=r, seed=seed, job_key=job_key.hex(), a_seed=a_seed.hex(),
                          b_seed=b_seed.hex(), bound=hex(bound), apea_sha=sha(ApEA), bpebt_sha=sha(BpEBt),
                          msgs_sha=sha(msgs), out_sha=sha((A.astype(np.int64) @ Bt.astype(np.int64).T).astype(np.int32)),
                          winners=sorted(wins)))
        out[f"msgs_{m}_{n}_{k}_{r}"] = msgs
    meta["mined"] = cases

    # 6. published digests (results/xc_cpu.json) -- the L1 int32 GEMM and the L2 quantizer
    with open(os.path.join(a.reference, "results", "xc_cpu.json")) as f:
        meta["xc_cpu"] = json.load(f)

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("wrote", sorted(out), "and golden.json")


if __name__ == "__main__":
    main()
