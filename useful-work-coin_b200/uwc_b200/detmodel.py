"""runtime/detrt/qwen3.py's deterministic Qwen3 / Llama forward on B200, bit-identical to detrt.

`DetQwen3` keeps the reference class's name, constructor arguments and methods (new_cache,
forward, logprobs, generate_greedy; qwen3.py:137-329), so provider code and the reference's own
determinism tests can switch by import. Every op runs on this library's kernels:

  embedding row gather                       torch indexing (a copy)
  det_rmsnorm + quant_act                    rmsnorm_quant            qwen3.py:294 + DetLinear
  q / k / v linear                           tcgen05 int8 GEMM        DetLinear.int_gemm
  dequant, q/k head norm, rope, quant127     qkv_post                 qwen3.py:240-252
  attention (cache, causal, exact P V)       attention_cache          qwen3.py:253-283
  o linear + residual                        quant_act, GEMM, dequant_residual
  MLP + residual                             detgpu.mlp_residual      qwen3.py:295-297
  final norm                                 rmsnorm                  qwen3.py:299
  lm_head, log-softmax, greedy argmax        GEMM (dequant fused), logprobs   qwen3.py:302-329

Weights are quantized on the GPU with quant_act, which is DetLinear's own quantization
(fwht(bs), quant_sym(64), the 1/sqrt(bs) fold; qwen3.py:73-88) evaluated bit for bit.
"""
from __future__ import annotations

import hashlib

import numpy as np
import torch

from . import det, detgpu, ops

MAX_KEYS = 1 << 20          # qwen3.py:33, the attention row sum's length bound (kernel constant)
ARCH_QWEN3, ARCH_LLAMA = 0, 1
ARCHS = {"qwen3": ARCH_QWEN3, "llama": ARCH_LLAMA, "mistral": ARCH_LLAMA}


def llama3_inv_freq(inv: np.ndarray, factor: float, low: float, high: float, orig: int) -> np.ndarray:
    """Llama 3.1+ rotary frequency scaling (the published rule transformers implements, which
    runtime/detrt/qwen3.py:38-47 pins): for each inverse frequency f with wavelength w = 2 pi / f,
    w above orig / low -> f / factor; w below orig / high -> f; in between the blend
    ((1 - s) f) / factor + s f with s = (orig / w - low) / (high - low). Every value is one float64
    expression evaluated in that order, so the table is the same bit for bit."""
    out = np.empty_like(inv)
    long_w, short_w = orig / low, orig / high
    for i, f in enumerate(inv.tolist()):
        w = 2 * np.pi / f
        if w > long_w:
            out[i] = f / factor
        elif w < short_w:
            out[i] = f
        else:
            s = (orig / w - low) / (high - low)
            out[i] = (1 - s) * f / factor + s * f
    return out


def rope_table(theta: float, head_dim: int, max_pos: int = 8192, scaling: dict | None = None):
    """float32 cos / sin rows for positions 0..max_pos-1 (qwen3.py:50-68): angles in float64,
    emb = [ang, ang], rounded once to float32. Returns (cos, sin, sha256 of cos||sin)."""
    inv = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim))
    if scaling:
        inv = llama3_inv_freq(inv, float(scaling["factor"]), float(scaling["low_freq_factor"]),
                              float(scaling["high_freq_factor"]), int(scaling["original_max_position_embeddings"]))
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
    emb = np.concatenate([ang, ang], axis=1)
    cos, sin = np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)
    return cos, sin, hashlib.sha256(cos.tobytes() + sin.tobytes()).hexdigest()


LLAMA3_SCALING_KEYS = ("factor", "low_freq_factor", "high_freq_factor", "original_max_position_embeddings")


def rope_config(cfg) -> tuple[float, dict | None]:
    """(rope theta, Llama 3 scaling parameters or None) of a transformers config. transformers 5
    keeps theta and the rope type together in `rope_parameters`; transformers 4 has `rope_theta`
    and an optional `rope_scaling` dict (type under "rope_type" or "type"). Defaults: theta 1e6,
    no scaling. Scalings other than llama3 are refused (qwen3.py:133-148 accepts the same set)."""
    v5 = dict(getattr(cfg, "rope_parameters", None) or {})
    v4 = dict(getattr(cfg, "rope_scaling", None) or {})
    theta = float(getattr(cfg, "rope_theta", None) or v5.get("rope_theta") or 1e6)
    if v5.get("rope_type"):
        kind, params = v5["rope_type"], v5
    else:
        kind, params = v4.get("rope_type") or v4.get("type") or "default", v4
    if kind == "default":
        return theta, None
    if kind == "llama3":
        return theta, {key: params[key] for key in LLAMA3_SCALING_KEYS}
    raise ValueError(f"unsupported rotary scaling {kind!r}: the deterministic forward knows the default and llama3")


class Linear:
    """A deterministic int8 linear (DetLinear, qwen3.py:71-126): Wq (n x k int8), sw (n float32),
    bs (Hadamard block). `int_gemm(q)` is the exact int32 q @ Wq^T; calling it on float32 rows
    quantizes them (quant_act) and returns the dequantized product."""

    def __init__(self, W: torch.Tensor, device, hadamard_block: int):
        n, k = W.shape
        self.n, self.k = n, k
        self.bs = min(hadamard_block, k & -k) if hadamard_block else 0
        Wq, sw = [], []
        for r0 in range(0, n, 16384):                      # bound the float32 staging copy
            q, s = detgpu.quant_act(W[r0:r0 + 16384].to(device=device, dtype=torch.float32), self.bs)
            Wq.append(q)
            sw.append(s)
        self.Wq = torch.cat(Wq).contiguous()
        self.sw = torch.cat(sw).contiguous()

    def int_gemm(self, q: torch.Tensor) -> torch.Tensor:
        return det.int_gemm(q, self.Wq, static_weights=True)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        q, s = detgpu.quant_act(x, self.bs)
        return det.linear_f32(q, s, self.Wq, self.sw, static_weights=True)


class DetQwen3:
    """Qwen3, Llama and Mistral checkpoints on one B200 (qwen3.py:151-329): the same outputs, bit
    for bit, as the reference's DetQwen3 on any device. hf_model: a transformers causal LM (its
    weights are read once and quantized on the GPU)."""

    def __init__(self, hf_model, device="cuda", hadamard_block: int = 512, mine: bool = False, max_pos: int = 8192):
        cfg = hf_model.config
        if mine:
            raise ValueError("the mined GEMM path of DetQwen3 is MinedWeight (ops.py); this runtime is the plain one")
        if cfg.model_type not in ARCHS:
            raise ValueError(f"model type {cfg.model_type!r} is not supported (supported: {sorted(ARCHS)})")
        if getattr(cfg, "attention_bias", False) or getattr(cfg, "mlp_bias", False):
            raise ValueError("biased attention or MLP projections are not supported")
        if getattr(cfg, "hidden_act", "silu") != "silu":
            raise ValueError(f"activation {cfg.hidden_act!r} is not supported")
        sw_ = getattr(cfg, "sliding_window", None)
        if ARCHS[cfg.model_type] == ARCH_LLAMA and sw_ is not None and sw_ < max_pos:
            raise ValueError(f"sliding-window attention ({sw_} < MaxPos {max_pos}) is not supported")
        self.device = torch.device(device)
        base = hf_model.model
        W = lambda mod: mod.weight.detach()
        hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        layers = []
        for lay in base.layers:
            at, mlp = lay.self_attn, lay.mlp
            layers.append(dict(
                in_norm=W(lay.input_layernorm), post_norm=W(lay.post_attention_layernorm),
                q_norm=W(at.q_norm) if hasattr(at, "q_norm") else None,
                k_norm=W(at.k_norm) if hasattr(at, "k_norm") else None,
                qkv=torch.cat([W(at.q_proj), W(at.k_proj), W(at.v_proj)]), o=W(at.o_proj),
                gu=torch.cat([W(mlp.gate_proj), W(mlp.up_proj)]), down=W(mlp.down_proj)))
        self._build(cfg.model_type, cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads, hd,
                    cfg.rms_norm_eps, rope_config(cfg), W(base.embed_tokens), layers, W(base.norm),
                    W(hf_model.lm_head), hadamard_block, max_pos)

    @classmethod
    def from_weights(cls, model_type: str, D: int, H: int, Hkv: int, hd: int, eps: float, rope, embed, layers,
                     norm, lm_head, device="cuda", hadamard_block: int = 512, max_pos: int = 8192) -> "DetQwen3":
        """The same model from raw float weights (layers: dicts with in_norm, post_norm, q_norm,
        k_norm, qkv = [q; k; v], o, gu = [gate; up], down), e.g. random-initialized on the GPU."""
        self = cls.__new__(cls)
        self.device = torch.device(device)
        self._build(model_type, D, H, Hkv, hd, eps, rope, embed, layers, norm, lm_head, hadamard_block, max_pos)
        return self

    def _build(self, model_type, D, H, Hkv, hd, eps, rope, embed, layers, norm, lm_head, hb, max_pos):
        if hd != 128:
            raise ValueError(f"head_dim {hd}: the attention kernel is built for head_dim 128")
        dev = self.device
        f32 = lambda t: t.to(device=dev, dtype=torch.float32).contiguous()
        self.arch = ARCHS[model_type]
        self.qk_norm = self.arch == ARCH_QWEN3
        self.D, self.H, self.Hkv, self.hd, self.eps = D, H, Hkv, hd, eps
        self.hadamard_block = hb
        cos, sin, self.rope_sha = rope_table(rope[0], hd, max_pos, rope[1])
        self.cos, self.sin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
        self.embed = f32(embed)
        ones = torch.ones(hd, dtype=torch.float32, device=dev)   # Llama / Mistral: q/k norms never read
        self.layers = []
        for L in layers:
            self.layers.append(dict(
                in_norm=f32(L["in_norm"]), post_norm=f32(L["post_norm"]),
                q_norm=f32(L["q_norm"]) if self.qk_norm else ones, k_norm=f32(L["k_norm"]) if self.qk_norm else ones,
                **{nm: L[nm] if isinstance(L[nm], Linear) else Linear(L[nm], dev, hb)
                   for nm in ("qkv", "o", "gu", "down")}))
        self.norm = f32(norm)
        self.lm_head = Linear(lm_head, dev, hb)
        # float(torch.tensor(1 / sqrt(hd)).to(F32)): the float64 value rounded once to float32
        self.inv_sqrt_hd = float(np.float32(1.0 / np.sqrt(hd)))

    def linears(self):
        for L in self.layers:
            yield from (L["qkv"], L["o"], L["gu"], L["down"])
        yield self.lm_head

    # ---------------------------------------------------------------- cache (qwen3.py:216-221)
    def new_cache(self, B: int, max_len: int):
        dev = self.device
        z = lambda *s, dt=torch.int8: torch.zeros(*s, dtype=dt, device=dev)
        return [dict(k=z(B, self.Hkv, max_len, self.hd), sk=z(B, self.Hkv, max_len, 1, dt=torch.float32),
                     v=z(B, self.Hkv, max_len, self.hd), sv=z(B, self.Hkv, max_len, 1, dt=torch.float32))
                for _ in self.layers]

    # ---------------------------------------------------------------- forward (qwen3.py:286-299)
    def _layer(self, L, x, cache, B: int, T: int, start: int, cos_t, sin_t) -> torch.Tensor:
        H, Hkv, hd = self.H, self.Hkv, self.hd
        q1, s1 = detgpu.rmsnorm_quant(x, L["in_norm"], self.eps, L["qkv"].bs)
        qq, qs, kq, ks, vq, vs = detgpu.qkv_post(L["qkv"].int_gemm(q1), s1, L["qkv"].sw, L["q_norm"], L["k_norm"],
                                                 cos_t, sin_t, T, H, Hkv, self.eps, self.qk_norm)
        end = start + T
        cache["k"][:, :, start:end] = kq.view(B, T, Hkv, hd).transpose(1, 2)
        cache["v"][:, :, start:end] = vq.view(B, T, Hkv, hd).transpose(1, 2)
        cache["sk"][:, :, start:end] = ks.view(B, T, Hkv, 1).transpose(1, 2)
        cache["sv"][:, :, start:end] = vs.view(B, T, Hkv, 1).transpose(1, 2)
        o = detgpu.attention_cache(qq, qs, cache, B, T, start, H, Hkv, self.inv_sqrt_hd)
        q2, s2 = detgpu.quant_act(o, L["o"].bs)
        r1 = detgpu.linear_resid(L["o"], q2, s2, x)
        return detgpu.mlp_residual(L["gu"], L["down"], L["post_norm"], r1, self.eps)

    @torch.no_grad()
    def forward(self, ids: torch.Tensor, cache, start: int = 0, layer_hashes: list | None = None) -> torch.Tensor:
        """ids: (B, T) tokens at positions start..start+T-1. Returns the final-norm hidden (B, T, D) fp32."""
        B, T = ids.shape
        x = self.embed[ids.to(self.device).reshape(-1)]
        cos_t = self.cos[start:start + T].contiguous()
        sin_t = self.sin[start:start + T].contiguous()
        for L, c in zip(self.layers, cache):
            x = self._layer(L, x, c, B, T, start, cos_t, sin_t)
            if layer_hashes is not None:
                layer_hashes.append(sha(x.reshape(B, T, self.D)))
        return detgpu.rmsnorm(x, self.norm, self.eps).reshape(B, T, self.D)

    @torch.no_grad()
    def logprobs(self, hidden: torch.Tensor, chunk: int = 256) -> torch.Tensor:
        """log_softmax(lm_head(hidden)) rows, deterministic (qwen3.py:302-312)."""
        flat = hidden.reshape(-1, self.D).to(self.device)
        out = [detgpu.logprobs(self.lm_head(flat[s0:s0 + chunk]))[0] for s0 in range(0, flat.shape[0], chunk)]
        return torch.cat(out).reshape(*hidden.shape[:-1], -1)

    @torch.no_grad()
    def next_tokens(self, last: torch.Tensor) -> torch.Tensor:
        """Greedy tokens of hidden rows (B, D): argmax of logprobs, first maximum (qwen3.py:322-323)."""
        return detgpu.logprobs(self.lm_head(last.reshape(-1, self.D)), want_lp=False)[1]

    def _decode_step(self, tok: torch.Tensor, cache, pos: torch.Tensor, max_start: int):
        """One decode step for B sequences with the position in device memory (int32 `pos`): the
        token embedding, every layer, the final norm and the greedy next token. The same
        arithmetic as forward(tok[:, None], cache, pos) + next_tokens; capturable as one graph."""
        B = tok.shape[0]
        H, Hkv, hd = self.H, self.Hkv, self.hd
        x = self.embed[tok]
        for L, c in zip(self.layers, cache):
            q1, s1 = detgpu.rmsnorm_quant(x, L["in_norm"], self.eps, L["qkv"].bs)
            qq, qs = detgpu.qkv_post_kv(L["qkv"].int_gemm(q1), s1, L["qkv"].sw, L["q_norm"], L["k_norm"], self.cos,
                                        self.sin, pos, 1, H, Hkv, self.eps, c, self.qk_norm)
            o = detgpu.attention_cache_at(qq, qs, c, B, 1, pos, max_start, H, Hkv, self.inv_sqrt_hd)
            q2, s2 = detgpu.quant_act(o, L["o"].bs)
            r1 = detgpu.linear_resid(L["o"], q2, s2, x)
            x = detgpu.mlp_residual(L["gu"], L["down"], L["post_norm"], r1, self.eps)
        h = detgpu.rmsnorm(x, self.norm, self.eps)
        return h, self.next_tokens(h)

    @torch.no_grad()
    def generate_greedy(self, prompt: torch.Tensor, n_new: int, graph: bool = True):
        """Prefill the prompt, then decode n_new tokens one at a time (qwen3.py:315-329).
        Returns (tokens (B, n_new), step hiddens (B, n_new, D)).

        graph=True replays the decode step as one CUDA graph (decode_graph: captured once per batch
        size and length, then reused by every call); the step reads its position from device
        memory, so one capture serves every step. The outputs are the same bits as the eager loop."""
        B, T0 = prompt.shape
        if graph and n_new >= 2:
            return self.decode_graph(B, T0 + n_new).run(prompt, n_new)
        cache = self.new_cache(B, T0 + n_new)
        last = self.forward(prompt, cache, 0)[:, -1]
        if n_new == 0:
            return torch.empty((B, 0), dtype=torch.int64, device=self.device), last[:, None][:, :0]
        toks, hs = [self.next_tokens(last)], [last]
        for i in range(1, n_new):
            last = self.forward(toks[-1][:, None], cache, T0 + i - 1)[:, 0]
            toks.append(self.next_tokens(last))
            hs.append(last)
        return torch.stack(toks, 1), torch.stack(hs, 1)

    def decode_graph(self, B: int, max_len: int) -> "DecodeGraph":
        """The captured decode step for B sequences of up to max_len positions (kept for the last
        (B, max_len) asked for; a new shape replaces it)."""
        dg = getattr(self, "_decode_graph", None)
        if dg is None or (dg.B, dg.max_len) != (B, max_len):
            self._decode_graph = None
            dg = self._decode_graph = DecodeGraph(self, B, max_len)
        return dg


class DecodeGraph:
    """One greedy decode step of DetQwen3 captured as a CUDA graph over a persistent KV cache and
    static token / position buffers: run() prefills a prompt into the cache and replays the step
    per token. The first step runs eagerly once before the capture (kernel attributes and
    workspaces), at position 0 of the zeroed cache."""

    def __init__(self, model: DetQwen3, B: int, max_len: int):
        self.model, self.B, self.max_len = model, B, max_len
        dev = model.device
        self.cache = model.new_cache(B, max_len)
        self.max_start = max_len - 2
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.tok = torch.zeros(B, dtype=torch.int64, device=dev)
        model._decode_step(self.tok, self.cache, self.pos, self.max_start)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        c0 = ops.launches()
        with torch.cuda.graph(self.graph):
            self.h, self.nxt = model._decode_step(self.tok, self.cache, self.pos, self.max_start)
            self.tok.copy_(self.nxt)
            self.pos.add_(1)
        self.launches_per_step = ops.launches() - c0   # this library's kernels in one replay
        ops.note_graph(-self.launches_per_step)        # captured, not launched

    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        """Prompt (B, T0) into the cache; returns the final-norm hidden of the last position."""
        assert prompt.shape[0] == self.B and prompt.shape[1] + 1 < self.max_len
        return self.model.forward(prompt, self.cache, 0)[:, -1]

    @torch.no_grad()
    def decode(self, last: torch.Tensor, T0: int, n_new: int):
        """n_new greedy tokens after a prefill of T0 positions whose last hidden is `last`."""
        assert T0 + n_new <= self.max_len
        nxt = self.model.next_tokens(last)
        toks, hs = [nxt], [last]
        self.tok.copy_(nxt)
        self.pos.fill_(T0)
        for _ in range(1, n_new):
            self.graph.replay()
            toks.append(self.nxt.clone())
            hs.append(self.h.clone())
        ops.note_graph(self.launches_per_step * (n_new - 1))
        return torch.stack(toks, 1), torch.stack(hs, 1)

    def run(self, prompt: torch.Tensor, n_new: int):
        return self.decode(self.prefill(prompt), prompt.shape[1], n_new)


def sha(t: torch.Tensor) -> str:
    """sha256[:20] of a tensor's bytes (qwen3.py:332-334)."""
    return hashlib.sha256(t.detach().contiguous().cpu().numpy().tobytes()).hexdigest()[:20]


QWEN3_1P7B = dict(model_type="qwen3", D=2048, H=16, Hkv=8, hd=128, I=6144, layers=28, vocab=151936, eps=1e-6,
                  theta=1e6, tied=True)


def random_model(shape: dict = QWEN3_1P7B, device="cuda", seed: int = 0, std: float = 0.02,
                 hadamard_block: int = 512, max_pos: int = 8192) -> DetQwen3:
    """A random-initialized model of the given shape, generated and quantized on the GPU one layer
    at a time (linear weights and the embedding N(0, std), norm weights 1 + N(0, 0.1))."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    D, H, Hkv, hd, I = shape["D"], shape["H"], shape["Hkv"], shape["hd"], shape["I"]
    rnd = lambda *s: torch.randn(*s, device=dev, generator=g) * std
    nrm = lambda n: 1 + 0.1 * torch.randn(n, device=dev, generator=g)
    self = DetQwen3.__new__(DetQwen3)
    self.device = dev
    embed = rnd(shape["vocab"], D)
    lm_head = embed if shape.get("tied") else rnd(shape["vocab"], D)
    layers = []
    for _ in range(shape["layers"]):
        # one layer's float weights at a time: quantized right away, then freed
        L = dict(in_norm=nrm(D), post_norm=nrm(D), q_norm=nrm(hd), k_norm=nrm(hd),
                 qkv=rnd((H + 2 * Hkv) * hd, D), o=rnd(D, H * hd), gu=rnd(2 * I, D), down=rnd(D, I))
        layers.append(_QuantizedLayer(L, dev, hadamard_block))
    self._build(shape["model_type"], D, H, Hkv, hd, shape["eps"], (shape["theta"], None), embed, layers,
                nrm(D), lm_head, hadamard_block, max_pos)
    return self


class _QuantizedLayer(dict):
    """A layer's weights with its linears already quantized (so random_model never holds more
    than one layer of float weights)."""

    def __init__(self, L: dict, dev, hb: int):
        super().__init__({k: (Linear(v, dev, hb) if k in ("qkv", "o", "gu", "down") else v) for k, v in L.items()})
