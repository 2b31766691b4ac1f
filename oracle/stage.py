"""CPU oracle of the stage-output commitments -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may import this module.

A hashlib restatement of the formats in runtime/detrt/stage.py:26-72 and runtime/agent/proto.py:24-35
(paths inside srivassid/useful-work-coin): RFC 6962 trees (leaf = sha256(0x00 || data), node =
sha256(0x01 || l || r), split at the largest power of two below n), rows as little-endian float32
bytes in 1 KiB blocks, the token leaf sha256(0x00 || "sout" || u32le t || row_root). Pinned by
tests/test_stage_oracle.py against roots the reference computed (tests/golden/make_golden_stage.py).
"""
from __future__ import annotations

import hashlib
import struct

import numpy as np

BLOCK = 1024


def leaf_hash(data: bytes) -> bytes:
    return hashlib.sha256(b"\x00" + data).digest()


def node(l: bytes, r: bytes) -> bytes:
    return hashlib.sha256(b"\x01" + l + r).digest()


def merkle_root(leaves: list[bytes]) -> bytes:
    if not leaves:
        return hashlib.sha256(b"").digest()
    if len(leaves) == 1:
        return leaves[0]
    k = 1
    while k << 1 < len(leaves):
        k <<= 1
    return node(merkle_root(leaves[:k]), merkle_root(leaves[k:]))


def merkle_root_bottom_up(leaves: list[bytes]) -> bytes:
    """Pair neighbours level by level, promoting an odd last node (the GPU kernels' order)."""
    level = list(leaves)
    while len(level) > 1:
        nxt = [node(level[i], level[i + 1]) for i in range(0, len(level) - 1, 2)]
        if len(level) & 1:
            nxt.append(level[-1])
        level = nxt
    return level[0] if level else hashlib.sha256(b"").digest()


def row_root(row: np.ndarray) -> bytes:
    b = np.ascontiguousarray(row, dtype="<f4").tobytes()
    return merkle_root([leaf_hash(b[i:i + BLOCK]) for i in range(0, max(len(b), 1), BLOCK)])


def stage_out_leaf(t: int, rroot: bytes) -> bytes:
    return leaf_hash(b"sout" + struct.pack("<I", t) + rroot)


def stage_output_root(rows: np.ndarray) -> bytes:
    return merkle_root([stage_out_leaf(t, row_root(r)) for t, r in enumerate(rows)])
