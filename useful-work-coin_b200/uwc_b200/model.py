"""Integer linear layers for Hugging Face Qwen3 models, mined on B200 (miner/ampere/uwc_ampere/model.py).

Same quantization and modes as the reference module, so provider code switches by import:
  weights      per output channel, W' = W H (H: block Walsh-Hadamard, orthonormal), s_w = max|W'| / 64
  activations  per token, x' = x H, s_x = max|x'| / 64 (ops.quant_rows_had: rotate + quantize fused)
  y = (q(x') q(W')^T) * s_x * s_w, bf16 out

Modes: "bf16" (original weights), "int" (the integer math through cuBLAS int8: the quality and
parity reference), "plain" (this library's tcgen05 GEMM with the bf16 dequant fused, no mining),
"mined" (MinedWeight.forward: commit, noise, hashed GEMM, exact denoise; bit-identical to "int").
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops

QMAX = 64


def hadamard(n: int, device, dtype=torch.float32) -> torch.Tensor:
    """The n x n Sylvester Hadamard matrix scaled to be orthonormal (model.py:30-36)."""
    assert n > 0 and n & (n - 1) == 0
    H = torch.ones(1, 1)
    while H.shape[0] < n:
        H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
    return (H / math.sqrt(n)).to(device=device, dtype=dtype)


def rotate(x: torch.Tensor, H: torch.Tensor | None) -> torch.Tensor:
    """x times the block-diagonal H along the last dim (model.py:39-44)."""
    if H is None:
        return x
    bs = H.shape[0]
    shp = x.shape
    return (x.reshape(*shp[:-1], shp[-1] // bs, bs).to(H.dtype) @ H).reshape(shp)


def quant_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric per-row quantization to int8 values in [-64, 64] (model.py:47-52)."""
    xf = x.float()
    s = xf.abs().amax(dim=-1, keepdim=True).clamp_min(1e-8) / QMAX
    q = torch.round(xf / s).clamp_(-QMAX, QMAX).to(torch.int8)
    return q, s.squeeze(-1)


class MinedLinear(nn.Module):
    """One or more nn.Linear layers that share an input, fused along n (model.py:55-141)."""

    def __init__(self, linears: list[nn.Linear], device, mode: str = "mined", hadamard_block: int = 512,
                 r: int = 128, cfg: str | None = None):
        super().__init__()
        if mode not in ("bf16", "int", "plain", "mined"):
            raise ValueError(f"mode {mode!r}")
        self.mode = mode
        self.splits = [l.out_features for l in linears]
        W = torch.cat([l.weight.detach() for l in linears], 0)
        bias = [l.bias for l in linears]
        self.bias = None if all(b is None for b in bias) else torch.cat(
            [b.detach() if b is not None else torch.zeros(l.out_features) for b, l in zip(bias, linears)]).to(
                device, torch.bfloat16)
        self.n, self.k = W.shape
        self.H = hadamard(min(hadamard_block, self.k & -self.k), device) if hadamard_block else None
        if mode == "bf16":
            self.W = W.to(device=device, dtype=torch.bfloat16)
        else:
            # row chunks, so a huge layer (lm_head) never needs a full float32 copy on the GPU
            qs, ss = [], []
            for s0 in range(0, self.n, 16384):
                q, sc = quant_rows(rotate(W[s0:s0 + 16384].to(device=device, dtype=torch.float32), self.H))
                qs.append(q)
                ss.append(sc)
            self.Wq, self.sw = torch.cat(qs).contiguous(), torch.cat(ss).contiguous()
        del W
        self.r = r
        self.cfg = cfg or ops.DEFAULT_CFG
        self.mw: ops.MinedWeight | None = None
        self.hashed_macs = 0   # m_pad * n * k summed over mined calls
        self.useful_macs = 0   # m * n * k summed over calls

    @property
    def mineable(self) -> bool:
        """Pearl's shape rules for a mined weight (model.py:95-98) and this kernel's tile alignment."""
        k, n, r = self.k, self.n, self.r
        return k >= max(1024, 16 * r) and k % r == 0 and k % 64 == 0 and k <= 4 * r * r and n % 64 == 0

    def setup_block(self, job_key_for_k, bound_for_k):
        """job_key_for_k(k) -> 32-byte job key; bound_for_k(k) -> 8 target words (model.py:100-107)."""
        if self.mode != "mined" or not self.mineable:
            return
        if self.mw is None:
            self.mw = ops.MinedWeight(Bt=self.Wq, b_scale=self.sw, r=self.r)
        self.mw.setup_block(job_key_for_k(self.k), bound_for_k(self.k))

    def _int_forward(self, xq, sx):
        y = torch._int_mm(xq, self.Wq.t()).float() * sx[:, None] * self.sw[None, :]
        return y.to(torch.bfloat16)

    @torch.compiler.disable
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shp = x.shape
        x2 = x.reshape(-1, self.k)
        m = x2.shape[0]
        if self.mode == "bf16":
            y = F.linear(x2.to(torch.bfloat16), self.W)
        else:
            bs = self.H.shape[0] if self.H is not None else 0
            kernel_path = self.mode in ("mined", "plain") and self.mineable
            mp = -(-m // ops.BM) * ops.BM if kernel_path else m
            xb = x2.to(torch.bfloat16)
            if mp != m:
                xb = F.pad(xb, (0, 0, 0, mp - m))
            xq, sx = ops.quant_rows_had(xb.contiguous(), bs)          # fused rotate + quantize
            if self.mode == "mined" and self.mineable:
                y = self.mw.forward(xq, sx)[:m]
                self.hashed_macs += mp * self.n * self.k
            elif self.mode == "plain" and self.mineable:
                y = torch.empty((mp, self.n), dtype=torch.bfloat16, device=xq.device)
                ops.gemm(xq, self.Wq, a_scale=sx, b_scale=self.sw, out=y, out_mode=ops.OUT_BF16)
                y = y[:m]
            elif m < 17:                                              # cuBLAS int8 needs m > 16
                y = (xq.float() @ self.Wq.float().t() * sx[:, None] * self.sw[None, :]).to(torch.bfloat16)
            else:
                y = self._int_forward(xq.contiguous(), sx)
        self.useful_macs += m * self.n * self.k
        if self.bias is not None:
            y = y + self.bias
        return y.reshape(*shp[:-1], self.n)


class _Slice(nn.Module):
    """k_proj / v_proj / up_proj stand-in: its slice of the fused output the head layer computed."""

    def __init__(self, head: "_FusedHead", idx: int):
        super().__init__()
        self.head, self.idx = head, idx

    @torch.compiler.disable
    def forward(self, x):
        assert self.head.last_input is x, "fused layers must be called with the same input tensor, in order"
        y = self.head.outputs[self.idx]
        if self.idx == len(self.head.outputs) - 1:    # the last consumer drops the references
            self.head.outputs = self.head.last_input = None
        return y


class _FusedHead(nn.Module):
    def __init__(self, ml: MinedLinear):
        super().__init__()
        self.ml = ml
        self.last_input = None
        self.outputs = None

    @torch.compiler.disable
    def forward(self, x):
        y = self.ml(x)
        self.last_input = x
        self.outputs = torch.split(y, self.ml.splits, dim=-1)
        return self.outputs[0]


def convert_qwen3(model, device, mode="mined", hadamard_block=512, mine_lm_head=True, cfg=None) -> list[MinedLinear]:
    """Swap every linear of a HF Qwen3 model (q/k/v fused, gate/up fused); returns the MinedLinears
    (model.py:171-197)."""
    mls = []
    base = model.model if hasattr(model, "model") else model
    for layer in base.layers:
        at, mlp = layer.self_attn, layer.mlp
        qkv = MinedLinear([at.q_proj, at.k_proj, at.v_proj], device, mode, hadamard_block, cfg=cfg)
        head = _FusedHead(qkv)
        at.q_proj, at.k_proj, at.v_proj = head, _Slice(head, 1), _Slice(head, 2)
        o = MinedLinear([at.o_proj], device, mode, hadamard_block, cfg=cfg)
        at.o_proj = o
        gu = MinedLinear([mlp.gate_proj, mlp.up_proj], device, mode, hadamard_block, cfg=cfg)
        head2 = _FusedHead(gu)
        mlp.gate_proj, mlp.up_proj = head2, _Slice(head2, 1)
        d = MinedLinear([mlp.down_proj], device, mode, hadamard_block, cfg=cfg)
        mlp.down_proj = d
        mls += [qkv, o, gu, d]
    if mine_lm_head and hasattr(model, "lm_head"):
        lm = MinedLinear([model.lm_head], device, mode, hadamard_block, cfg=cfg)
        model.lm_head = lm
        mls.append(lm)
    return mls
