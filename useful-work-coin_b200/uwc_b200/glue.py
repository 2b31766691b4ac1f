"""Host-side mining glue that needs no Pearl bindings (miner/ampere/uwc_ampere/pearl_glue.py:14-66).

Header serialization, job keys, proofs and verification stay in Pearl's Rust (`pearl_mining`),
which is not part of this repository; callers keep using it for those.
"""
from __future__ import annotations

import numpy as np

# Hash-tile pattern of the kernels: rows g + 8i, cols 2t + {0,1} + 8j inside a 64 x 64 block.
AMPERE_ROWS = [8 * i for i in range(8)]
AMPERE_COLS = sorted([8 * j + e for j in range(8) for e in (0, 1)])
TILE_SIZE = len(AMPERE_ROWS) * len(AMPERE_COLS)


def nbits_to_target(nbits: int) -> int:
    exp, mant = nbits >> 24, nbits & 0xFFFFFF
    if mant == 0 or exp == 0 or mant & 0x800000:
        return 0
    return mant >> (8 * (3 - exp)) if exp <= 3 else mant << (8 * (exp - 3))


def jackpot_bound(nbits: int, k: int, r: int, penalty_base_rank: int, tile: int = TILE_SIZE) -> int:
    """min(difficulty bound, rank-penalized bound) (pearl_glue.py:55-62); penalty_base_rank is
    Pearl's PENALTY_BASE_RANK constant, passed in by the caller that has the Pearl bindings."""
    t = nbits_to_target(nbits)
    plain_b = min(t * tile * k, 2 ** 256 - 1)
    pen = min(t * tile * (k // r) * penalty_base_rank, 2 ** 256 - 1)
    return min(plain_b, pen)


def bound_words(bound: int) -> np.ndarray:
    return np.array([(bound >> (32 * i)) & 0xFFFFFFFF for i in range(8)], dtype=np.uint32)


def target_for(m: int, n: int, expected_wins: int = 12) -> np.ndarray:
    """A bound giving about `expected_wins` winning tiles per m x n GEMM (test_proj_gemm.py:17-20)."""
    return bound_words(((1 << 256) - 1) * expected_wins // ((m // 8) * (n // 16)))
