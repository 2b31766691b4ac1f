"""Stage-output commitments on the GPU, identical to runtime/agent/proto.py stage_out_leaves /
stage_output_root, with the names of runtime/detgpu/sha.py: only 32 bytes per token (sout_leaves)
or per stage (stage_roots_gpu) leave the GPU instead of the float32 rows.

A stage's T output rows are committed by the RFC 6962 Merkle root of one leaf per token,
sha256(0x00 || "sout" || u32le t || row_root), where row_root is the Merkle root of
sha256(0x00 || block) over the row's little-endian float32 bytes in 1 KiB blocks.
"""
from __future__ import annotations

import hashlib

import numpy as np
import torch

from ._lib import check, lib
from .ops import _p, _stream


def _rows(out: torch.Tensor) -> tuple[torch.Tensor, int, int, int]:
    assert out.dtype == torch.float32 and out.is_cuda and out.dim() == 3, (out.dtype, out.shape)
    out = out.contiguous()
    B, T, D = out.shape
    return out, B, T, D


def _scratch(nrows: int, D: int, device) -> torch.Tensor:
    return torch.empty(int(lib().uwc_stage_scratch_words(nrows, D)), dtype=torch.int32, device=device)


def _leaf_words(out: torch.Tensor) -> torch.Tensor:
    """(B * T, 8) int32 on the GPU: the stage-output leaves as SHA-256 state words."""
    out, B, T, D = _rows(out)
    nrows = B * T
    scratch = _scratch(nrows, D, out.device)
    res = torch.empty((nrows, 8), dtype=torch.int32, device=out.device)
    check(lib().uwc_stage_out_leaves(_p(out), nrows, D, T, _p(scratch), scratch.numel(), _p(res), _stream()),
          "stage_out_leaves")
    return res


def digest_bytes(words) -> np.ndarray:
    """(..., 8) SHA-256 state words (torch or numpy) -> (..., 32) digest bytes."""
    if isinstance(words, torch.Tensor):
        words = words.cpu().numpy()
    w = np.ascontiguousarray(words).view(np.uint32)
    return w.byteswap().view(np.uint8).reshape(*w.shape[:-1], 32)


def sout_leaves(out: torch.Tensor) -> np.ndarray:
    """The stage-output leaves of B stages: out (B, T, D) float32 on the GPU -> (B, T, 32) uint8."""
    B, T, _ = out.shape
    return digest_bytes(_leaf_words(out)).reshape(B, T, 32)


def stage_roots_gpu(out: torch.Tensor) -> torch.Tensor:
    """stage_output_root of each of the B stages in out (B, T, D), computed entirely on the GPU:
    (B, 8) int32 state words on the GPU (digest_bytes turns them into bytes)."""
    out, B, T, D = _rows(out)
    scratch = _scratch(B * T, D, out.device)
    roots = torch.empty((B, 8), dtype=torch.int32, device=out.device)
    check(lib().uwc_stage_roots(_p(out), B, T, D, _p(scratch), scratch.numel(), _p(roots), _stream()), "stage_roots")
    return roots


def _node(l: bytes, r: bytes) -> bytes:
    return hashlib.sha256(b"\x01" + l + r).digest()


def merkle_root(leaves: list[bytes]) -> bytes:
    """RFC 6962 root of already-hashed leaves (split at the largest power of two below n)."""
    if not leaves:
        return hashlib.sha256(b"").digest()
    if len(leaves) == 1:
        return leaves[0]
    k = 1
    while k << 1 < len(leaves):
        k <<= 1
    return _node(merkle_root(leaves[:k]), merkle_root(leaves[k:]))


def stage_output_roots(out: torch.Tensor) -> list[bytes]:
    """agent.proto.stage_output_root for each of the B stages in out (B, T, D)."""
    return [bytes(r) for r in digest_bytes(stage_roots_gpu(out))]
