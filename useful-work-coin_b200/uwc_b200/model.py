"""Mined integer linear layers for Hugging Face Qwen3 models on B200 (the reference's
miner/ampere/uwc_ampere/model.py surface: MinedLinear, convert_qwen3, hadamard, rotate, quant_rows).

Quantization (the reference's scheme, model.py:30-52): per output channel of the weight and per
token of the activation, a block Walsh-Hadamard rotation of size bs (the largest power of two
dividing k, capped at `hadamard_block`), then symmetric int8 in [-64, 64] with scale max|x'| / 64.
Weights and activations both go through this library's fused rotate + quantize kernel
(ops.quant_rows_had) from bf16 rows, so a layer's int8 operands are produced the same way on both
sides; the output is y = RNE_bf16((float(q_x q_W^T) * s_x) * s_w).

Modes:
  "bf16"   the original bf16 weights (F.linear), no integer math: the quality baseline;
  "int"    the exact int32 product on this library's GEMM, the dequant as separate torch
           elementwise ops: the parity baseline of the two below;
  "plain"  the same product with the dequant fused into the GEMM epilogue (bf16 out);
  "mined"  MinedWeight.forward: commit, noise, hashed GEMM, exact denoise, fused dequant. Layers
           whose shape Pearl does not accept for mining (see `mineable`) run "plain".
Every integer mode sends every shape through ops.gemm; the three give bit-identical outputs.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops

QMAX = 64
ROW_CHUNK = 8192   # weight rows quantized per kernel call (bounds the bf16 staging copy)


def hadamard(n: int, device, dtype=torch.float32) -> torch.Tensor:
    """The orthonormal n x n Sylvester Hadamard matrix: H[i, j] = (-1)^popcount(i & j) / sqrt(n)."""
    assert n > 0 and n & (n - 1) == 0
    idx = torch.arange(n)
    parity = torch.zeros(n, n, dtype=torch.int64)
    b = idx[:, None] & idx[None, :]
    while bool(b.any()):
        parity ^= b & 1
        b = b >> 1
    return ((1 - 2 * parity).to(torch.float64) / math.sqrt(n)).to(device=device, dtype=dtype)


def rotate(x: torch.Tensor, H: torch.Tensor | None) -> torch.Tensor:
    """x multiplied by the block-diagonal matrix diag(H, H, ...) along its last dimension."""
    if H is None:
        return x
    bs = H.shape[0]
    blocks = x.to(H.dtype).unflatten(-1, (x.shape[-1] // bs, bs))
    return torch.matmul(blocks, H).flatten(-2)


def quant_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric int8 per row: q = round_half_even(x / s) clamped to [-64, 64], s = max|x| / 64
    (at least 1e-8 / 64). Returns (q int8, s float32 per row)."""
    xf = x.float()
    s = torch.clamp(xf.abs().amax(dim=-1), min=1e-8) / QMAX
    q = torch.clamp(torch.round(xf / s.unsqueeze(-1)), -QMAX, QMAX).to(torch.int8)
    return q, s


def _block_size(k: int, hadamard_block: int) -> int:
    return min(hadamard_block, k & -k) if hadamard_block else 0


class MinedLinear(nn.Module):
    """nn.Linear layers that read the same input, concatenated along the output dimension and
    computed as one integer GEMM (one mined weight when mode is "mined")."""

    def __init__(self, linears: list[nn.Linear], device, mode: str = "mined", hadamard_block: int = 512,
                 r: int = 128, cfg: str | None = None):
        super().__init__()
        if mode not in ("bf16", "int", "plain", "mined"):
            raise ValueError(f"mode {mode!r}")
        self.mode, self.r, self.cfg = mode, r, cfg
        self.splits = [lin.out_features for lin in linears]
        self.k = linears[0].in_features
        self.n = sum(self.splits)
        self.bs = _block_size(self.k, hadamard_block)
        self.H = hadamard(self.bs, device) if self.bs > 1 else None
        biases = [lin.bias.detach() if lin.bias is not None else None for lin in linears]
        self.bias = None
        if any(b is not None for b in biases):
            self.bias = torch.cat([b if b is not None else torch.zeros(n) for b, n in zip(biases, self.splits)]).to(
                device=device, dtype=torch.bfloat16)
        if mode == "bf16":
            self.W = torch.cat([lin.weight.detach() for lin in linears]).to(device=device, dtype=torch.bfloat16)
        else:
            self.Wq = torch.empty((self.n, self.k), dtype=torch.int8, device=device)
            self.sw = torch.empty(self.n, dtype=torch.float32, device=device)
            row = 0
            for lin in linears:
                for r0 in range(0, lin.out_features, ROW_CHUNK):
                    w = lin.weight.detach()[r0:r0 + ROW_CHUNK].to(device=device, dtype=torch.bfloat16).contiguous()
                    ops.quant_rows_had(w, self.bs, q=self.Wq[row:row + w.shape[0]], scale=self.sw[row:row + w.shape[0]])
                    row += w.shape[0]
        self.mw: ops.MinedWeight | None = None
        self.hashed_macs = 0   # padded rows x n x k over the calls that took the mined path
        self.useful_macs = 0   # rows x n x k over all calls

    @property
    def mineable(self) -> bool:
        """Pearl's shape rules for a mined weight (k at least max(1024, 16 r), at most 4 r^2, a
        multiple of r; miner/ampere/uwc_ampere/model.py:95-98) and this kernel's 64-alignment."""
        k, n, r = self.k, self.n, self.r
        return max(1024, 16 * r) <= k <= 4 * r * r and k % r == 0 and k % 64 == 0 and n % 64 == 0

    def setup_block(self, job_key_for_k, bound_for_k):
        """Prepare the mined weight for a block: job_key_for_k(k) -> 32-byte key, bound_for_k(k) ->
        8 target words. A no-op unless this layer mines."""
        if self.mode != "mined" or not self.mineable:
            return
        if self.mw is None:
            self.mw = ops.MinedWeight(Bt=self.Wq, b_scale=self.sw, r=self.r)
        self.mw.setup_block(job_key_for_k(self.k), bound_for_k(self.k))

    def _integer(self, xq: torch.Tensor, sx: torch.Tensor) -> torch.Tensor:
        m = xq.shape[0]
        if self.mode == "mined" and self.mw is not None:
            self.hashed_macs += m * self.n * self.k
            return self.mw.forward(xq, sx)
        if self.n % 8 == 0 and self.mode != "int":        # "plain", and "mined" layers that do not mine
            y = torch.empty((m, self.n), dtype=torch.bfloat16, device=xq.device)
            ops.gemm(xq, self.Wq, a_scale=sx, b_scale=self.sw, out=y, out_mode=ops.OUT_BF16)
            return y
        acc = torch.empty((m, self.n), dtype=torch.int32, device=xq.device)
        ops.gemm(xq, self.Wq, out=acc, out_mode=ops.OUT_I32)
        return ((acc.float() * sx.unsqueeze(1)) * self.sw.unsqueeze(0)).to(torch.bfloat16)

    @torch.compiler.disable
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        xb = x.reshape(-1, self.k).to(torch.bfloat16)
        m = xb.shape[0]
        if self.mode == "bf16":
            y = F.linear(xb, self.W)
        else:
            mined = self.mode == "mined" and self.mw is not None
            rows = -(-m // 64) * 64 if mined else m     # the mined GEMM works on 64-row multiples
            if rows != m:
                xb = torch.cat([xb, xb.new_zeros(rows - m, self.k)])
            xq, sx = ops.quant_rows_had(xb.contiguous(), self.bs)
            y = self._integer(xq, sx)[:m]
        self.useful_macs += m * self.n * self.k
        if self.bias is not None:
            y = y + self.bias
        return y.reshape(*lead, self.n)


class _SharedInput:
    """One fused MinedLinear serving the stand-ins of several projections that read the same input
    (q/k/v, or gate/up). A stand-in called with a new input tensor runs the fused layer; the others
    then take their parts of that result. The input is held (and compared by identity) only until
    every stand-in has taken its part, so no stale result can match a later tensor."""

    def __init__(self, fused: MinedLinear):
        self.fused = fused
        self.x = None
        self.parts: tuple[torch.Tensor, ...] = ()
        self.waiting: set[int] = set()

    def part(self, x: torch.Tensor, idx: int) -> torch.Tensor:
        if x is not self.x or idx not in self.waiting:
            self.parts = torch.split(self.fused(x), self.fused.splits, dim=-1)
            self.x, self.waiting = x, set(range(len(self.parts)))
        self.waiting.discard(idx)
        y = self.parts[idx]
        if not self.waiting:
            self.x, self.parts = None, ()
        return y


class _Part(nn.Module):
    """Stand-in for one of the fused projections."""

    def __init__(self, shared: _SharedInput, idx: int):
        super().__init__()
        self.shared, self.idx = shared, idx
        if idx == 0:
            self.fused = shared.fused       # registered once, so .to() / state_dict see it

    @torch.compiler.disable
    def forward(self, x):
        return self.shared.part(x, self.idx)


def _fuse(owner: nn.Module, names: list[str], device, mode, hadamard_block, cfg) -> MinedLinear:
    ml = MinedLinear([getattr(owner, nm) for nm in names], device, mode, hadamard_block, cfg=cfg)
    if len(names) == 1:
        setattr(owner, names[0], ml)
        return ml
    shared = _SharedInput(ml)
    for i, nm in enumerate(names):
        setattr(owner, nm, _Part(shared, i))
    return ml


def convert_qwen3(model, device, mode="mined", hadamard_block=512, mine_lm_head=True, cfg=None) -> list[MinedLinear]:
    """Replace every linear layer of a Hugging Face Qwen3 model by MinedLinear: q/k/v fused into one,
    o alone, gate/up fused, down alone, and the LM head (if mine_lm_head). Returns the new layers,
    four per decoder layer in that order, then the head."""
    layers = []
    body = getattr(model, "model", model)
    for block in body.layers:
        attn, mlp = block.self_attn, block.mlp
        layers.append(_fuse(attn, ["q_proj", "k_proj", "v_proj"], device, mode, hadamard_block, cfg))
        layers.append(_fuse(attn, ["o_proj"], device, mode, hadamard_block, cfg))
        layers.append(_fuse(mlp, ["gate_proj", "up_proj"], device, mode, hadamard_block, cfg))
        layers.append(_fuse(mlp, ["down_proj"], device, mode, hadamard_block, cfg))
    if mine_lm_head and hasattr(model, "lm_head"):
        layers.append(_fuse(model, ["lm_head"], device, mode, hadamard_block, cfg))
    return layers
