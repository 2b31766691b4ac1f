"""B200 drop-in for `uwc_ampere.ops` (miner/ampere/uwc_ampere/ops.py): the NoisyGEMM launchers,
`MinedWeight` and `GraphedForward`, on torch tensors and torch's current CUDA stream.

Same names, argument meanings and error behaviour as the reference module, so miner, provider
and verifier code can switch with `from uwc_b200 import ops`. The work runs in libuwcb200.so
(sm_100a kernels behind the C ABI in include/uwc_b200.h); this module only owns workspaces and
passes pointers, sizes and the stream.

Differences from the reference, all additive:
  * one tcgen05 kernel family replaces the mma.sync tile configs: `cfg` is accepted and ignored,
    CONFIGS / DEFAULT_CFG keep their names for callers that read them;
  * OUT_F32 (the detrt dequant epilogue) joins OUT_NONE / OUT_I32 / OUT_BF16;
  * the rank-r projections default to the tensor-core path (`project`), which the reference
    offers as UWC_PROJ_GEMM; set UWC_PROJ_GEMM=0 for the shared-memory-atomics path. Both are
    bit-identical (tests/test_gpu_mined.py checks it, as the reference's test_proj_gemm.py does).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from ._lib import check, lib

BM, BN, BK = 128, 256, 128          # unit rows, unit columns, K bytes per pipeline stage
WIN_WORDS = 10
CHUNKS_PER_CTA = 128
FLAG_HASH, FLAG_DENOISE = 1, 2
OUT_NONE, OUT_I32, OUT_BF16, OUT_F32 = 0, 1, 2, 3
CONFIGS = {"sm100": (256, 3, 1)}
DEFAULT_CFG = "sm100"
PROJ_GEMM = os.environ.get("UWC_PROJ_GEMM", "1") != "0"
LAUNCHES = 0   # kernels this module has launched (all of them this library's own)


def _count(n: int = 1) -> None:
    global LAUNCHES
    LAUNCHES += n


def limbs_for(k: int) -> int:
    """Balanced base-128 limbs that always cover |projection| <= 127 * k (ops.py:18-24)."""
    bound, L, cap = 127 * k, 1, 63
    while cap < bound:
        L += 1
        cap = cap * 128 + 63
    return L


# Pearl cert-v3 constants (reference.py:22-25): labels are ASCII names padded to 32 bytes, salts are
# BLAKE3("pearl/cert-v3/noise-seed/A|B") (checked against the blake3 package in tests/test_host.py).
SEED_LABEL_A = b"A_tensor" + b"\x00" * 24
SEED_LABEL_B = b"B_tensor" + b"\x00" * 24
SEED_SALT_A = bytes.fromhex("8249406ca0ed15169616f692fcf076f892dbdb2a7023b852f0d47719c390017b")
SEED_SALT_B = bytes.fromhex("11300632ec6301ca2be2af718b3f4d4f1ae9c63988e8cc044844301d71b89aa9")


def words(b: bytes, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.frombuffer(b, dtype="<u4").view(np.int32).copy()).to(device)


def words_to_bytes(t: torch.Tensor) -> bytes:
    return t.detach().cpu().numpy().view(np.uint32).astype("<u4").tobytes()


LABEL_A = words(SEED_LABEL_A, "cpu")
LABEL_B = words(SEED_LABEL_B, "cpu")
SALT_A = words(SEED_SALT_A, "cpu")
SALT_B = words(SEED_SALT_B, "cpu")
_CONSTS: dict = {}


def consts(device) -> dict:
    """Device copies of the label/salt constants (made once; forward() must not copy H2D)."""
    key = str(torch.device(device))
    c = _CONSTS.get(key)
    if c is None:
        c = _CONSTS[key] = {n: t.to(device) for n, t in
                            dict(LABEL_A=LABEL_A, LABEL_B=LABEL_B, SALT_A=SALT_A, SALT_B=SALT_B).items()}
    return c


def _p(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    assert t.is_cuda, "uwc_b200 operates on CUDA tensors only"
    return t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


# ------------------------------------------------------------------ BLAKE3
def b3_scratch_words(nbytes: int) -> int:
    return int(lib().uwc_b3_scratch_words(nbytes))


def b3_root_and_seed(data: torch.Tensor, key: torch.Tensor, *, prefix=None, salt=None, dim: int = 0,
                     root_out=None, seed_out=None, scratch=None):
    """Keyed BLAKE3 of `data` (length a multiple of 1024) -> root, optional salted seed (ops.py:99-118)."""
    nbytes = _nbytes(data)
    assert nbytes % 1024 == 0 and nbytes > 0
    need = b3_scratch_words(nbytes)
    if scratch is None or scratch.numel() < need:
        scratch = torch.empty(need, dtype=torch.int32, device=data.device)
    check(lib().uwc_b3_root_and_seed(_p(data), nbytes, _p(key), _p(prefix), _p(salt), dim, _p(root_out),
                                     _p(seed_out), _p(scratch), scratch.numel(), _stream()), "b3_root_and_seed")
    cnt, launches = -(-(nbytes // 1024) // CHUNKS_PER_CTA), 2
    while cnt > 1024:
        cnt, launches = -(-cnt // 1024), launches + 1
    _count(launches)
    return scratch


# ------------------------------------------------------------------ noise
def noise_uniform(out: torch.Tensor, label: torch.Tensor, key: torch.Tensor, zero_me=None, zero_n: int = 0):
    check(lib().uwc_noise_uniform(_p(out), _nbytes(out), _p(label), _p(key), _p(zero_me), zero_n, _stream()),
          "noise_uniform")
    _count()


def noise_perm(out: torch.Tensor, k: int, r: int, label: torch.Tensor, key: torch.Tensor):
    check(lib().uwc_noise_perm(_p(out), k, r, _p(label), _p(key), _stream()), "noise_perm")
    _count()


def noise_rows(src, rows, k, r, *, E=None, Pn=None, dst=None, Pp=None, corr=None, corr_off=-1, ecopy_off=-1,
               maxabs=None, lmax=None):
    lmax = corr.shape[0] if corr is not None else 0
    assert rows % 8 == 0 and k % 4 == 0
    check(lib().uwc_noise_rows(_p(src), rows, k, r, _p(E), _p(Pn), _p(dst), _p(Pp), _p(corr), corr_off, ecopy_off,
                               _p(maxabs), lmax, _stream()), "noise_rows")
    _count()


# ------------------------------------------------------------------ projections as int8 GEMMs
def proj_matrix(P: torch.Tensor, k: int, r: int, St: torch.Tensor | None = None) -> torch.Tensor:
    """S^T for a noise permutation P: r x k int8 with S^T[lo(l), l] += 1 and S^T[hi(l), l] -= 1."""
    if St is None:
        St = torch.empty((r, k), dtype=torch.int8, device=P.device)
    check(lib().uwc_proj_matrix(_p(P), k, r, _p(St), _stream()), "proj_matrix")
    _count()
    return St


def project(src: torch.Tensor, St: torch.Tensor, corr: torch.Tensor, corr_off: int, maxabs: torch.Tensor,
            proj: torch.Tensor | None = None):
    """noise_rows' projection (limbs at corr_off, maxabs) with the sum on the tensor cores: src @ S
    is an exact int8 GEMM (int32 accumulate) on this library's own tcgen05 kernel."""
    rows, r = src.shape[0], St.shape[0]
    if proj is None:
        proj = torch.empty((rows, r), dtype=torch.int32, device=src.device)
    gemm(src, St, out=proj, out_mode=OUT_I32)
    check(lib().uwc_proj_corr(_p(proj), rows, r, _p(corr), corr_off, _p(maxabs), corr.shape[0], _stream()),
          "proj_corr")
    _count()


# ------------------------------------------------------------------ GEMM
_GEMM_WS: dict = {}


def quant_rows_had(x: torch.Tensor, bs: int, q: torch.Tensor | None = None, scale: torch.Tensor | None = None):
    """ops.py:172-181: bf16 rows (m x k) -> block Walsh-Hadamard (size bs, 0 = none), then per-row
    int8 in [-64, 64] with float32 scale max|x'| / 64 folded with 1/sqrt(bs)."""
    assert x.dtype == torch.bfloat16 and x.is_contiguous() and x.dim() == 2
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=x.device) if q is None else q
    scale = torch.empty(m, dtype=torch.float32, device=x.device) if scale is None else scale
    check(lib().uwc_quant_rows_had(_p(x), m, k, bs, _p(q), _p(scale), _stream()), "quant_rows_had")
    _count()
    return q, scale


def gemm_workspace(device, m: int, n: int, flags: int, out_mode: int) -> torch.Tensor | None:
    """Per-device workspace of the hashed GEMM (tile messages; the int32 product of a denoised bf16
    forward), grown on demand. Callers serialize on one stream per device (like the reference's
    shared workspace, ops.py:258-277)."""
    nbytes = int(lib().uwc_gemm_workspace_bytes(m, n, flags, out_mode))
    if nbytes == 0:
        return None
    key = str(torch.device(device))
    ws = _GEMM_WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = _GEMM_WS[key] = torch.empty(nbytes, dtype=torch.uint8, device=device)
    return ws


def gemm(A, B, *, r=128, flags=0, corrA=None, corrB=None, maxabs=None, key=None, target=None, wins=None,
         max_wins=0, a_scale=None, b_scale=None, out=None, out_mode=OUT_NONE, cfg=None):
    """C = A B^T (ops.py:185-198) with hashing / denoising / scaled output, see uwc_gemm."""
    m, k = A.shape
    n = B.shape[0]
    assert A.dtype == torch.int8 and B.dtype == torch.int8 and A.is_contiguous() and B.is_contiguous()
    if flags:
        assert m % 64 == 0 and n % 64 == 0 and k % 64 == 0 and r % 64 == 0 and k % r == 0, (m, n, k, r)
    lmax = corrA.shape[0] if corrA is not None else 0
    ws = gemm_workspace(A.device, m, n, flags, out_mode)
    check(lib().uwc_gemm(_p(A), _p(B), m, n, k, r, flags, _p(corrA), _p(corrB), _p(maxabs), lmax, _p(key), _p(target),
                         _p(wins), max_wins, _p(a_scale), _p(b_scale), _p(out), out_mode, _p(ws),
                         0 if ws is None else ws.numel(), _stream()), "gemm")
    _count()


# ------------------------------------------------------------------ one mined linear layer
_WORKSPACE: dict = {}


@dataclass
class MinedWeight:
    """A weight B^T (n x k int8, values in [-64, 64]) prepared for mining under one block template.

    setup_block() runs once per (block header, k); forward() runs per call and needs no host sync
    (ops.py:205-371)."""
    Bt: torch.Tensor            # n x k int8 (GPU, or pinned CPU: only BpEBt lives on the GPU)
    b_scale: torch.Tensor       # n float32, on the mining GPU
    r: int = 128
    max_wins: int = 64
    # per block
    job_key: torch.Tensor | None = None
    b_seed: torch.Tensor | None = None
    target: torch.Tensor | None = None
    BpEBt: torch.Tensor | None = None
    PB: torch.Tensor | None = None
    EBRt: torch.Tensor | None = None
    corrB: torch.Tensor | None = None
    SBt: torch.Tensor | None = None
    _bufs: dict = field(default_factory=dict)

    @property
    def n(self):
        return self.Bt.shape[0]

    @property
    def k(self):
        return self.Bt.shape[1]

    @property
    def device(self):
        return self.b_scale.device

    def setup_block(self, job_key: bytes, target_words: np.ndarray):
        dev = self.device
        n, k, r = self.n, self.k, self.r
        Bt = self.Bt if self.Bt.device == dev else self.Bt.to(dev, non_blocking=True)
        self.job_key = words(job_key, dev)
        self.target = torch.from_numpy(np.asarray(target_words).astype(np.uint32).view(np.int32).copy()).to(dev)
        self.b_seed = torch.empty(8, dtype=torch.int32, device=dev)
        c = consts(dev)
        b3_root_and_seed(Bt.view(-1), self.job_key, prefix=self.job_key, salt=c["SALT_B"], dim=n,
                         seed_out=self.b_seed)
        self.EBRt = torch.empty((n, r), dtype=torch.int8, device=dev)
        noise_uniform(self.EBRt, c["LABEL_B"], self.b_seed)
        self.PB = torch.empty(k, dtype=torch.int32, device=dev)
        noise_perm(self.PB, k, r, c["LABEL_B"], self.b_seed)
        if self.BpEBt is None:
            self.BpEBt = torch.empty((n, k), dtype=torch.int8, device=dev)
            self.corrB = torch.zeros((limbs_for(k), n, 2 * r), dtype=torch.int8, device=dev)
        noise_rows(Bt, n, k, r, E=self.EBRt, Pn=self.PB, dst=self.BpEBt, corr=self.corrB, ecopy_off=0)
        self.SBt = proj_matrix(self.PB, k, r)
        del Bt

    def _buf(self, m: int):
        """Per-call buffers. The large ones are a workspace shared by every weight with the same
        (m, k, r): layers run one after another on one stream. Win records are per weight."""
        dev, k, r = self.device, self.k, self.r
        key = (str(dev), m, k, r)
        ws = _WORKSPACE.get(key)
        if ws is None:
            n_max = max(m, 1)
            ws = _WORKSPACE[key] = dict(
                a_seed=torch.empty(8, dtype=torch.int32, device=dev),
                EAL=torch.empty((m, r), dtype=torch.int8, device=dev),
                PA=torch.empty(k, dtype=torch.int32, device=dev),
                SAt=torch.empty((r, k), dtype=torch.int8, device=dev),
                ApEA=torch.empty((m, k), dtype=torch.int8, device=dev),
                corrA=torch.zeros((limbs_for(k), m, 2 * r), dtype=torch.int8, device=dev),
                maxabs=torch.zeros(2, dtype=torch.int32, device=dev),
                projA=torch.empty((n_max, r), dtype=torch.int32, device=dev),
                scratch=torch.empty(b3_scratch_words(m * k), dtype=torch.int32, device=dev),
            )
        wins = self._bufs.get(m)
        if wins is None:
            wins = self._bufs[m] = torch.zeros(1 + self.max_wins * WIN_WORDS, dtype=torch.int32, device=dev)
        return {**ws, "wins": wins}

    def _projB(self):
        if self._bufs.get("projB") is None:
            self._bufs["projB"] = torch.empty((self.n, self.r), dtype=torch.int32, device=self.device)
        return self._bufs["projB"]

    def forward(self, A: torch.Tensor, a_scale: torch.Tensor, out: torch.Tensor | None = None,
                out_mode: int = OUT_BF16, hash_tiles: bool = True) -> torch.Tensor:
        """A: m x k int8 (values in [-64, 64]). Returns A @ Bt^T scaled (bf16), exact int32, or the
        detrt fp32 dequant (OUT_F32). Every path gives bit-identical outputs and winning tiles."""
        return self._forward(A, a_scale, out, out_mode, hash_tiles, DEFAULT_CFG, PROJ_GEMM)

    def _forward(self, A, a_scale, out, out_mode, hash_tiles, cfg, proj):
        m, k = A.shape
        n, r = self.n, self.r
        dev = A.device
        b = self._buf(m)
        c = consts(dev)
        if out is None and out_mode != OUT_NONE:
            dt = {OUT_BF16: torch.bfloat16, OUT_I32: torch.int32, OUT_F32: torch.float32}[out_mode]
            out = torch.empty((m, n), dtype=dt, device=dev)
        # 1. commit to A, derive a_seed = H(b_seed || bind_a(root_A, m))
        b3_root_and_seed(A.view(-1), self.job_key, prefix=self.b_seed, salt=c["SALT_A"], dim=m,
                         seed_out=b["a_seed"], scratch=b["scratch"])
        # 2. A-side noise (also zeroes maxabs and the win counter)
        noise_uniform(b["EAL"], c["LABEL_A"], b["a_seed"], zero_me=b["maxabs"], zero_n=2)
        b["wins"][:1].zero_()
        noise_perm(b["PA"], k, r, c["LABEL_A"], b["a_seed"])
        # 3. ApEA = A + EAL*P_A ; X = A * P_B^T (limbs) ; EAL copy ; 4. Y = BpEBt * P_A^T (limbs)
        if proj:
            noise_rows(A, m, k, r, E=b["EAL"], Pn=b["PA"], dst=b["ApEA"], corr=b["corrA"], ecopy_off=r)
            project(A, self.SBt, b["corrA"], 0, b["maxabs"][0:1], proj=b["projA"][:m])
            project(self.BpEBt, proj_matrix(b["PA"], k, r, b["SAt"]), self.corrB, r, b["maxabs"][1:2],
                    proj=self._projB())
        else:
            noise_rows(A, m, k, r, E=b["EAL"], Pn=b["PA"], dst=b["ApEA"], Pp=self.PB, corr=b["corrA"], corr_off=0,
                       ecopy_off=r, maxabs=b["maxabs"][0:1])
            noise_rows(self.BpEBt, n, k, r, Pp=b["PA"], corr=self.corrB, corr_off=r, maxabs=b["maxabs"][1:2])
        # 5. noisy GEMM: hash every tile, denoise exactly, scale
        gemm(b["ApEA"], self.BpEBt, r=r, flags=(FLAG_HASH if hash_tiles else 0) | FLAG_DENOISE,
             corrA=b["corrA"], corrB=self.corrB, maxabs=b["maxabs"], key=b["a_seed"], target=self.target,
             wins=b["wins"], max_wins=self.max_wins, a_scale=a_scale, b_scale=self.b_scale, out=out,
             out_mode=out_mode)
        return out

    def noise_mine(self, A: torch.Tensor):
        """What a pure noise miner runs per attempt batch: commit A, noise it, hashed GEMM, no output.

        No projections (X, Y) and no denoise, since nobody needs C (ops.py:349-364)."""
        b = self._buf(A.shape[0])
        self.mine_prepare(A, b["a_seed"], b["ApEA"], b["wins"], b["EAL"], b["PA"], b["scratch"])
        self.mine_gemm(b["ApEA"], b["a_seed"], b["wins"])

    def mine_prepare(self, A, a_seed, ApEA, wins, EAL, PA, scratch):
        """The first half of noise_mine: commit to A (a_seed), its noise EAL and P_A, ApEA = A + noise,
        and the win counter zeroed. Writes only the given buffers."""
        m, k = A.shape
        c = consts(A.device)
        b3_root_and_seed(A.view(-1), self.job_key, prefix=self.b_seed, salt=c["SALT_A"], dim=m, seed_out=a_seed,
                         scratch=scratch)
        noise_uniform(EAL, c["LABEL_A"], a_seed, zero_me=wins, zero_n=1)
        noise_perm(PA, k, self.r, c["LABEL_A"], a_seed)
        noise_rows(A, m, k, self.r, E=EAL, Pn=PA, dst=ApEA)

    def mine_gemm(self, ApEA, a_seed, wins):
        """The second half of noise_mine: the hashed GEMM of a prepared attempt."""
        gemm(ApEA, self.BpEBt, r=self.r, flags=FLAG_HASH, key=a_seed, target=self.target, wins=wins,
             max_wins=self.max_wins)

    def win_count(self, m: int) -> int:
        """Winning tiles of the last call with this m, including any beyond max_wins (syncs)."""
        return int(self._buf(m)["wins"][0].item())

    def winners(self, m: int) -> list[tuple[int, int, bytes]]:
        """(row_offset, col_offset, hash) for winning tiles of the last forward with this m (syncs).
        Raises if a kernel reported a device-side timeout since the last check."""
        w = self._buf(m)["wins"].cpu().numpy().view(np.uint32)
        st = _lib.device_status(clear=True)
        if st:
            raise _lib.UWCError(f"device status {st:#x}: a kernel wait timed out; results are invalid")
        cnt = min(int(w[0]), self.max_wins)
        recs = w[1:1 + cnt * WIN_WORDS].reshape(cnt, WIN_WORDS)
        return [(int(x[0]), int(x[1]), x[2:].astype("<u4").tobytes()) for x in recs]


class HostMiner:
    """Noise mining from nonce matrices in pinned host memory, the way a miner fed by another
    process or machine runs miner_loop.py:109-111: the upload of attempt i + 1 (a copy stream, two
    device buffers) overlaps the commit, noise and hashed GEMM of attempt i, and every attempt's
    win records come back to pinned host memory. Results equal noise_mine + winners per attempt."""

    def __init__(self, w: "MinedWeight", m: int, k: int, device):
        self.w, self.m, self.k = w, m, k
        dev = torch.device(device)
        self.A = [torch.empty((m, k), dtype=torch.int8, device=dev) for _ in range(2)]
        self.copy_stream = torch.cuda.Stream(dev)
        self.uploaded = [torch.cuda.Event() for _ in range(2)]
        self.consumed = [torch.cuda.Event() for _ in range(2)]
        self.wins_dev = w._buf(m)["wins"]
        self.i = 0

    def mine(self, A_host: torch.Tensor, wins_host: torch.Tensor) -> None:
        """Enqueue one attempt: A_host (m x k int8, pinned), its win records (the device wins
        buffer's words) copied into wins_host (pinned int32) when the attempt is done. Asynchronous."""
        assert A_host.is_pinned() and A_host.shape == (self.m, self.k) and wins_host.is_pinned()
        s = self.i & 1
        main = torch.cuda.current_stream()
        with torch.cuda.stream(self.copy_stream):
            if self.i >= 2:
                self.copy_stream.wait_event(self.consumed[s])     # the attempt two back read this buffer
            self.A[s].copy_(A_host, non_blocking=True)
            self.uploaded[s].record(self.copy_stream)
        main.wait_event(self.uploaded[s])
        self.w.noise_mine(self.A[s])
        self.consumed[s].record(main)
        wins_host.copy_(self.wins_dev, non_blocking=True)
        self.i += 1


class GraphedForward:
    """MinedWeight.forward captured as one CUDA graph for a fixed m (static input/output buffers)."""

    def __init__(self, w: MinedWeight, m: int, out_mode: int = OUT_BF16):
        dev = w.device
        self.w, self.m = w, m
        self.A = torch.zeros((m, w.k), dtype=torch.int8, device=dev)
        self.a_scale = torch.ones(m, dtype=torch.float32, device=dev)
        dt = {OUT_BF16: torch.bfloat16, OUT_I32: torch.int32, OUT_F32: torch.float32}[out_mode]
        self.out = torch.empty((m, w.n), dtype=dt, device=dev)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                w.forward(self.A, self.a_scale, out=self.out, out_mode=out_mode)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            w.forward(self.A, self.a_scale, out=self.out, out_mode=out_mode)

    def __call__(self):
        self.graph.replay()
        return self.out
