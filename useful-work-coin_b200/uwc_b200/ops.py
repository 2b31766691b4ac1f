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
  * MinedWeight's per-block and per-call sequences are single library calls
    (uwc_mined_setup_block, uwc_mined_forward, uwc_mine_attempt) over a block buffer and a
    shared workspace; the rank-r projections run on the tensor cores (the reference's opt-in
    UWC_PROJ_GEMM path). noise_rows with a projection permutation runs a gather kernel instead;
    both give the same integers (tests/test_gpu_mined.py, as the reference's test_proj_gemm.py).
"""
from __future__ import annotations

import ctypes

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

_REPLAYED = 0   # kernels run by graph replays, net of the ones recorded (captured, not run) by captures


def launches() -> int:
    """Kernels of this library launched in this process: the library's own counter of host-side
    launches, adjusted by note_graph() for kernels captured into CUDA graphs and run by replays."""
    return _lib.launch_count() + _REPLAYED


def note_graph(kernels: int) -> None:
    """Adjust launches() by `kernels`: minus a capture's kernels (recorded, not run), plus a replay's."""
    global _REPLAYED
    _REPLAYED += kernels


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
    return scratch


# ------------------------------------------------------------------ noise
def noise_uniform(out: torch.Tensor, label: torch.Tensor, key: torch.Tensor, zero_me=None, zero_n: int = 0):
    check(lib().uwc_noise_uniform(_p(out), _nbytes(out), _p(label), _p(key), _p(zero_me), zero_n, _stream()),
          "noise_uniform")


def noise_perm(out: torch.Tensor, k: int, r: int, label: torch.Tensor, key: torch.Tensor):
    check(lib().uwc_noise_perm(_p(out), k, r, _p(label), _p(key), _stream()), "noise_perm")


def noise_rows(src, rows, k, r, *, E=None, Pn=None, dst=None, Pp=None, corr=None, corr_off=-1, ecopy_off=-1,
               maxabs=None, lmax=None):
    lmax = corr.shape[0] if corr is not None else 0
    assert rows % 8 == 0 and k % 4 == 0
    check(lib().uwc_noise_rows(_p(src), rows, k, r, _p(E), _p(Pn), _p(dst), _p(Pp), _p(corr), corr_off, ecopy_off,
                               _p(maxabs), lmax, _stream()), "noise_rows")


# ------------------------------------------------------------------ projections as int8 GEMMs
def proj_matrix(P: torch.Tensor, k: int, r: int, St: torch.Tensor | None = None) -> torch.Tensor:
    """S^T for a noise permutation P: r x k int8 with S^T[lo(l), l] += 1 and S^T[hi(l), l] -= 1."""
    if St is None:
        St = torch.empty((r, k), dtype=torch.int8, device=P.device)
    check(lib().uwc_proj_matrix(_p(P), k, r, _p(St), _stream()), "proj_matrix")
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


SEPI_I32, SEPI_F32, SEPI_BF16, SEPI_RESID, SEPI_SWIGLU = range(5)
SEPI_EARLY_W = 0x100
STREAM_MAX_M = 64


def gemm_stream(X, W, epi=SEPI_I32, *, x_scale=None, w_scale=None, resid=None, out=None, early_w=False):
    """out = X W^T on the weight-streaming GEMM (m <= 64), with the epilogue `epi` (uwc_gemm_stream):
    SEPI_I32 int32; SEPI_F32 / SEPI_BF16 the dequant fmul(fmul(float(acc), x_scale), w_scale);
    SEPI_RESID that plus `resid` (fp32 m x n); SEPI_SWIGLU det_silu(gate) * up for W = [gate; up]
    (n / 2 rows each), m x n/2 fp32. early_w: W is a static weight (not written by the kernel
    launched just before), so the call may stream it while that kernel finishes."""
    m, k = X.shape
    n = W.shape[0]
    assert X.dtype == torch.int8 and W.dtype == torch.int8 and X.is_contiguous() and W.is_contiguous()
    if out is None:
        dt = {SEPI_I32: torch.int32, SEPI_BF16: torch.bfloat16}.get(epi, torch.float32)
        out = torch.empty((m, n // 2 if epi == SEPI_SWIGLU else n), dtype=dt, device=X.device)
    f32 = (lambda t: None if t is None else t.contiguous().float())
    check(lib().uwc_gemm_stream(_p(X), _p(W), m, n, k, _p(f32(x_scale)), _p(f32(w_scale)),
                                _p(None if resid is None else resid.contiguous()), _p(out),
                                epi | (SEPI_EARLY_W if early_w else 0), _stream()),
          "gemm_stream")
    return out


def gemm_epi(X, W, epi=SEPI_I32, *, x_scale=None, w_scale=None, resid=None, out=None, early_w=False):
    """gemm_stream's epilogues at any m (uwc_gemm_epi): m <= 64 streams W; larger m runs the tcgen05
    GEMM with the output step (dequant, + resid, SwiGLU of W = [gate; up]) in its epilogue, so no
    int32 product goes through HBM."""
    m, k = X.shape
    n = W.shape[0]
    assert X.dtype == torch.int8 and W.dtype == torch.int8 and X.is_contiguous() and W.is_contiguous()
    if out is None:
        dt = {SEPI_I32: torch.int32, SEPI_BF16: torch.bfloat16}.get(epi, torch.float32)
        out = torch.empty((m, n // 2 if epi == SEPI_SWIGLU else n), dtype=dt, device=X.device)
    f32 = (lambda t: None if t is None else t.contiguous().float())
    flags = epi | (SEPI_EARLY_W if early_w else 0)
    nbytes = int(lib().uwc_gemm_epi_workspace_bytes(m, n, epi))
    ws = None
    if nbytes:
        key = str(torch.device(X.device))
        ws = _GEMM_WS.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = _GEMM_WS[key] = torch.empty(nbytes, dtype=torch.uint8, device=X.device)
    check(lib().uwc_gemm_epi(_p(X), _p(W), m, n, k, _p(f32(x_scale)), _p(f32(w_scale)),
                             _p(None if resid is None else resid.contiguous()), _p(out), flags, _p(ws),
                             0 if ws is None else ws.numel(), _stream()), "gemm_epi")
    return out


# ------------------------------------------------------------------ one mined linear layer
MB_CONSTS, MB_EBRT, MB_PB, MB_SBT, MB_BPEBT, MB_BYTES = range(6)
MW_A_SEED, MW_MAXABS, MW_EAL, MW_PA, MW_APEA, MW_B3, MW_GEMM, MW_SAT, MW_CORRA, MW_CORRB, MW_PROJA, MW_PROJB, \
    MW_BYTES = range(13)
_SHARED_WS: dict = {}   # device -> one uint8 workspace, grown on demand, shared by every weight


def _offsets(fn, *args, count: int) -> list[int]:
    arr = (ctypes.c_uint64 * (count + 1))()
    check(fn(*args, arr), fn.__name__)
    return list(arr)


def shared_workspace(device, nbytes: int) -> torch.Tensor:
    """The per-device call workspace of MinedWeight: layers run one after another on one stream, so
    they share it (as the reference shares its per-(device, m, k, r) buffers, ops.py:258-277)."""
    key = str(torch.device(device))
    ws = _SHARED_WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = _SHARED_WS[key] = torch.empty(nbytes, dtype=torch.uint8, device=device)
    return ws


class MinedWeight:
    """B^T (n x k int8, values in [-64, 64]) prepared for mining under one block template, with the
    reference's call surface (ops.py:205-371): setup_block() once per block key, then forward() /
    noise_mine() per call and winners() to read the win records.

    The block state lives in one device buffer written by uwc_mined_setup_block; a call is a single
    library call (uwc_mined_forward / uwc_mine_attempt) over a workspace shared by every weight on
    the device. Attribute views (BpEBt, target, ...) and buffers(m) expose the parts by the
    library's layout, for tests and benchmarks."""

    def __init__(self, Bt: torch.Tensor, b_scale: torch.Tensor, r: int = 128, max_wins: int = 64):
        self.Bt, self.b_scale, self.r, self.max_wins = Bt, b_scale, r, max_wins
        self.block: torch.Tensor | None = None
        self._wins: dict[int, torch.Tensor] = {}
        self._last_ws: dict[int, tuple[torch.Tensor, list[int]]] = {}

    n = property(lambda self: self.Bt.shape[0])
    k = property(lambda self: self.Bt.shape[1])
    device = property(lambda self: self.b_scale.device)

    # -------------------------------------------------------- per block
    def setup_block(self, job_key: bytes, target_words) -> None:
        n, k, r, dev = self.n, self.k, self.r, self.device
        assert len(job_key) == 32
        self._bo = _offsets(lib().uwc_mined_block_layout, n, k, r, count=MB_BYTES)
        if self.block is None:
            self.block = torch.empty(self._bo[MB_BYTES], dtype=torch.uint8, device=dev)
        Bt = self.Bt if self.Bt.device == dev else self.Bt.to(dev, non_blocking=True)
        scratch = shared_workspace(dev, 4 * b3_scratch_words(n * k))
        key = (ctypes.c_uint8 * 32).from_buffer_copy(job_key)
        tgt = (ctypes.c_uint32 * 8)(*[int(x) for x in np.asarray(target_words, dtype=np.uint64)])
        check(lib().uwc_mined_setup_block(_p(Bt.contiguous()), n, k, r, key, tgt, _p(self.block), self.block.numel(),
                                          _p(scratch), scratch.numel(), _stream()), "mined_setup_block")
        del Bt

    def _block_part(self, idx: int, shape, dtype) -> torch.Tensor:
        assert self.block is not None, "setup_block() first"
        nbytes = int(np.prod(shape)) * torch.tensor([], dtype=dtype).element_size()
        return self.block[self._bo[idx]:self._bo[idx] + nbytes].view(dtype).view(shape)

    BpEBt = property(lambda self: self._block_part(MB_BPEBT, (self.n, self.k), torch.int8))
    EBRt = property(lambda self: self._block_part(MB_EBRT, (self.n, self.r), torch.int8))
    PB = property(lambda self: self._block_part(MB_PB, (self.k,), torch.int32))
    SBt = property(lambda self: self._block_part(MB_SBT, (self.r, self.k), torch.int8))
    job_key = property(lambda self: self._block_part(MB_CONSTS, (64,), torch.int32)[0:8])
    b_seed = property(lambda self: self._block_part(MB_CONSTS, (64,), torch.int32)[8:16])
    target = property(lambda self: self._block_part(MB_CONSTS, (64,), torch.int32)[16:24])

    # -------------------------------------------------------- per call
    def _wins_for(self, m: int) -> torch.Tensor:
        w = self._wins.get(m)
        if w is None:
            w = self._wins[m] = torch.zeros(1 + self.max_wins * WIN_WORDS, dtype=torch.int32, device=self.device)
        return w

    def _workspace(self, m: int, forward: bool, hash_tiles: bool, out_mode: int):
        wo = _offsets(lib().uwc_mined_workspace_layout, m, self.n, self.k, self.r, int(forward), int(hash_tiles),
                      out_mode, count=MW_BYTES)
        ws = shared_workspace(self.device, wo[MW_BYTES])
        self._last_ws[m] = (ws, wo)
        return ws, wo

    def forward(self, A: torch.Tensor, a_scale: torch.Tensor, out: torch.Tensor | None = None,
                out_mode: int = OUT_BF16, hash_tiles: bool = True) -> torch.Tensor:
        """A: m x k int8 (values in [-64, 64]). Returns A @ Bt^T exactly, scaled to bf16 (default),
        int32 (OUT_I32) or the detrt fp32 dequant (OUT_F32); with hash_tiles every tile of the
        noisy product is hashed and checked against the block target (winners())."""
        m, k = A.shape
        assert A.dtype == torch.int8 and A.is_contiguous() and k == self.k
        if out is None and out_mode != OUT_NONE:
            dt = {OUT_BF16: torch.bfloat16, OUT_I32: torch.int32, OUT_F32: torch.float32}[out_mode]
            out = torch.empty((m, self.n), dtype=dt, device=A.device)
        ws, wo = self._workspace(m, True, hash_tiles, out_mode)
        wins = self._wins_for(m)
        check(lib().uwc_mined_forward(_p(A), m, self.n, k, self.r, _p(a_scale), _p(self.b_scale), _p(self.block),
                                      int(hash_tiles), _p(wins), self.max_wins, _p(out), out_mode, _p(ws), ws.numel(),
                                      _stream()), "mined_forward")
        return out

    def noise_mine(self, A: torch.Tensor) -> None:
        """One noise-mining attempt on A: commit, noise, hashed GEMM, no output (ops.py:349-364)."""
        m, k = A.shape
        assert A.dtype == torch.int8 and A.is_contiguous() and k == self.k
        ws, _ = self._workspace(m, False, True, OUT_NONE)
        check(lib().uwc_mine_attempt(_p(A), m, self.n, k, self.r, _p(self.block), _p(self._wins_for(m)),
                                     self.max_wins, _p(ws), ws.numel(), _stream()), "mine_attempt")

    def buffers(self, m: int) -> dict:
        """Views of the last call's workspace parts for this m (a_seed, EAL, PA, ApEA, maxabs and,
        after a forward, corrA, corrB) and the win buffer."""
        ws, wo = self._last_ws[m]
        L, r, n, k = limbs_for(self.k), self.r, self.n, self.k

        def part(idx, shape, dtype):
            nbytes = int(np.prod(shape)) * torch.tensor([], dtype=dtype).element_size()
            return ws[wo[idx]:wo[idx] + nbytes].view(dtype).view(shape)
        views = dict(a_seed=part(MW_A_SEED, (8,), torch.int32), maxabs=part(MW_MAXABS, (2,), torch.int32),
                     EAL=part(MW_EAL, (m, r), torch.int8), PA=part(MW_PA, (k,), torch.int32),
                     ApEA=part(MW_APEA, (m, k), torch.int8), wins=self._wins_for(m))
        if wo[MW_CORRB] > wo[MW_CORRA]:
            views.update(corrA=part(MW_CORRA, (L, m, 2 * r), torch.int8),
                         corrB=part(MW_CORRB, (L, n, 2 * r), torch.int8))
        return views

    def win_count(self, m: int) -> int:
        """Winning tiles of the last call with this m, including any beyond max_wins (syncs)."""
        return int(self._wins_for(m)[0].item())

    def winners(self, m: int) -> list[tuple[int, int, bytes]]:
        """(row_offset, col_offset, hash) of the winning tiles of the last call with this m (syncs).
        Raises if a kernel reported a device-side timeout since the last check."""
        words_ = self._wins_for(m).cpu().numpy().view(np.uint32)
        st = _lib.device_status(clear=True)
        if st:
            raise _lib.UWCError(f"device status {st:#x}: a kernel wait timed out; results are invalid")
        cnt = min(int(words_[0]), self.max_wins)
        return [(int(rec[0]), int(rec[1]), rec[2:].astype("<u4").tobytes())
                for rec in words_[1:1 + cnt * WIN_WORDS].reshape(cnt, WIN_WORDS)]


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
        self.wins_dev = w._wins_for(m)
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
    """A MinedWeight's forward for one m as a replayable CUDA graph over static buffers: write the
    nonce matrix into .A (and scales into .a_scale), call the object, read .out. The forward is a
    single library call, so the graph holds exactly its kernels; the first (uncaptured) call sets
    the library's per-device launch state, which capture must not do."""

    def __init__(self, w: MinedWeight, m: int, out_mode: int = OUT_BF16, hash_tiles: bool = True):
        dev = w.device
        dt = {OUT_BF16: torch.bfloat16, OUT_I32: torch.int32, OUT_F32: torch.float32}[out_mode]
        self.A = torch.zeros((m, w.k), dtype=torch.int8, device=dev)
        self.a_scale = torch.ones(m, dtype=torch.float32, device=dev)
        self.out = torch.empty((m, w.n), dtype=dt, device=dev)
        call = lambda: w.forward(self.A, self.a_scale, out=self.out, out_mode=out_mode, hash_tiles=hash_tiles)
        call()
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            call()

    def __call__(self) -> torch.Tensor:
        self.graph.replay()
        return self.out
