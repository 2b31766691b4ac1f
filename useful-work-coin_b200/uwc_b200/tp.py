"""Tensor-parallel deterministic int8 linears over torch.distributed (NCCL over NVLink on B200s).

New: the reference splits a model only into pipeline stages of whole layers
(runtime/detrt/qwen3.py:151-158); these layers split single linears across GPUs and stay
bit-identical to one device:

  ColumnParallelLinear  rows of W (output features) split across ranks; each rank computes its
                        output columns with the dequant fused into the GEMM; `gather` concatenates.
  RowParallelLinear     columns of W (input features) split on Hadamard-block boundaries. Each rank
                        transforms its activation shard, the row absmax is all-reduced with MAX
                        (exact), every rank quantizes with the full row's scale (so q is the full
                        row's q, sliced), multiplies its shard, and the int32 partial products are
                        all-reduced with SUM -- exact, since integer addition is associative --
                        before the dequant (+ residual).
  TPMLP                 the MLP block of runtime/detrt/fast.py:182-189: rmsnorm_quant on the
                        replicated input, gate/up column-parallel on the down projection's k shards,
                        fp32 SwiGLU, row-parallel down projection with the residual add.

`kernels` is the device backend: by default this library's CUDA kernels (GPUKernels); tests pass
a CPU stand-in built from the oracle to check the sharding and collectives with gloo ranks. A
backend with `fused = True` also offers quant_act, linear_resid and swiglu_linear: the output step
then runs inside the GEMM's epilogue (the row-parallel layer on one rank, and the gate/up SwiGLU on
any number; the weight-streaming GEMM for decode-sized calls), with the same bits as the separate
kernels. Given a
PeerExchange, a row-parallel layer on several ranks runs its two all-reduces (the row absmax and
the int32 partial products) inside its quantizer and GEMM over NVLink peer memory instead of NCCL.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist


def _all_reduce(t: torch.Tensor, op, group) -> None:
    """all_reduce over `group`; a no-op for a single rank (no process group needed)."""
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=op, group=group)


class _UwcTP(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int), ("world", ctypes.c_int), ("max_m", ctypes.c_int), ("max_n", ctypes.c_int),
                ("base", ctypes.c_void_p * 8)]


class PeerExchange:
    """The NVLink peer exchange of the fused tensor-parallel decode kernels (uwc_quant_act_tp,
    uwc_gemm_stream_tp): one zero-filled buffer per rank, every peer's buffer mapped here through CUDA
    IPC. Collective over `group`: every rank constructs it with the same max_m / max_n and makes the
    same sequence of fused calls; close() (also collective) releases it."""

    def __init__(self, max_m: int, max_n: int, rank: int, world: int, device, group=None):
        from ._lib import check, lib
        L = lib()
        self.rank, self.world, self.group, self.device = rank, world, group, torch.device(device)
        self._own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(L.uwc_tp_alloc(max_m, max_n, ctypes.byref(self._own)), "tp_alloc")
            handle = (ctypes.c_uint8 * 64)()
            check(L.uwc_ipc_handle(self._own, handle), "ipc_handle")
            mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
            handles = [torch.empty_like(mine) for _ in range(world)]
            if world > 1:
                dist.all_gather(handles, mine, group=group)
            else:
                handles = [mine]
            self.peers = []
            self.tp = _UwcTP(rank, world, max_m, max_n)
            for r in range(world):
                if r == rank:
                    self.tp.base[r] = self._own.value
                    continue
                hb = (ctypes.c_uint8 * 64)(*handles[r].cpu().tolist())
                ptr = ctypes.c_void_p()
                check(L.uwc_ipc_open(hb, ctypes.byref(ptr)), "ipc_open")
                self.peers.append(ptr)
                self.tp.base[r] = ptr.value

    def barrier(self) -> None:
        """Device-side barrier of the ranks on the current stream (uwc_tp_barrier): the streams
        leave it within about one NVLink write latency of each other."""
        from ._lib import check, lib
        from .ops import _stream
        check(lib().uwc_tp_barrier(ctypes.byref(self.tp), _stream()), "tp_barrier")

    def close(self) -> None:
        from ._lib import lib
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)          # no peer writes into this buffer any more
        L = lib()
        for ptr in self.peers:
            L.uwc_ipc_close(ptr)
        if self.world > 1:
            dist.barrier(group=self.group)          # every peer has unmapped it
        L.uwc_tp_free(self._own)
        self._own, self.peers = None, []


def even_bounds(n: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """[lo, hi) of `rank`'s share of n items cut on multiples of `align` (n % align == 0), as even
    as the alignment allows; earlier ranks take the remainder."""
    assert n % align == 0, (n, align)
    units = n // align
    base, extra = divmod(units, world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo * align, hi * align


class GPUKernels:
    """The CUDA backend (uwc_b200.detgpu / uwc_b200.det / uwc_b200.ops)."""

    fused = True

    @staticmethod
    def _mods():
        from . import det, detgpu
        return det, detgpu

    def linear_f32(self, q, s, Wq, sw):
        return self._mods()[0].linear_f32(q, s, Wq, sw, static_weights=True)

    def int_gemm(self, q, Wq):
        return self._mods()[0].int_gemm(q, Wq, static_weights=True)

    def fwht_absmax(self, x, bs):
        return self._mods()[1].fwht_absmax(x, bs)

    def quant_act_global(self, x, bs, amax):
        return self._mods()[1].quant_act_global(x, bs, amax)

    def rmsnorm_quant(self, x, w, eps, bs):
        return self._mods()[1].rmsnorm_quant(x, w, eps, bs)

    def swiglu(self, acc, s3, sw):
        return self._mods()[1].swiglu(acc, s3, sw)

    def dequant_residual(self, acc, s, sw, x):
        return self._mods()[1].dequant_residual(acc, s, sw, x)

    def quant_act(self, x, bs):
        return self._mods()[1].quant_act(x, bs)

    def linear_resid(self, q, s, Wq, sw, x):
        """fadd(x, deq(q Wq^T)) (x None: deq alone), the output step in the GEMM's epilogue."""
        from . import ops
        return ops.gemm_epi(q, Wq, ops.SEPI_RESID, x_scale=s, w_scale=sw, resid=x, early_w=True)

    def quant_act_tp(self, x, bs, exchange):
        """quant_act of a row-parallel shard with the whole row's absmax, exchanged in the kernel."""
        from . import ops
        from ._lib import check, lib
        x = x.contiguous().float()
        m, k = x.shape
        q = torch.empty((m, k), dtype=torch.int8, device=x.device)
        sc = torch.empty(m, dtype=torch.float32, device=x.device)
        check(lib().uwc_quant_act_tp(ops._p(x), m, k, bs, ops._p(q), ops._p(sc), ctypes.byref(exchange.tp),
                                     ops._stream()), "quant_act_tp")
        return q, sc

    def linear_resid_tp(self, q, s, Wq, sw, x, exchange):
        """fadd(x, deq(sum over the ranks of q Wq^T)), the sum exchanged in the GEMM's epilogue."""
        from . import ops
        from ._lib import check, lib
        m, n = q.shape[0], Wq.shape[0]
        out = torch.empty((m, n), dtype=torch.float32, device=q.device)
        f32 = s.contiguous().float(), sw.contiguous().float()
        check(lib().uwc_gemm_stream_tp(ops._p(q.contiguous()), ops._p(Wq), m, n, q.shape[1], ops._p(f32[0]),
                                       ops._p(f32[1]), ops._p(None if x is None else x.contiguous()), ops._p(out),
                                       ops.SEPI_RESID | ops.SEPI_EARLY_W, ctypes.byref(exchange.tp), ops._stream()),
              "gemm_stream_tp")
        return out

    def swiglu_linear(self, q, s, Wq, sw):
        """det_silu(deq(gate)) * deq(up) of q [gate; up]^T, computed in the GEMM's epilogue."""
        from . import ops
        if Wq.shape[0] % 8:
            return self.swiglu(self.int_gemm(q, Wq), s, sw)
        return ops.gemm_epi(q, Wq, ops.SEPI_SWIGLU, x_scale=s, w_scale=sw, early_w=True)


def _default(kernels):
    return GPUKernels() if kernels is None else kernels


class ColumnParallelLinear:
    """W (n x k int8, per-row scales sw) split by output rows; forward(q, s) -> this rank's columns."""

    def __init__(self, Wq: torch.Tensor, sw: torch.Tensor, bs: int, rank: int, world: int, device, kernels=None,
                 group=None):
        n = Wq.shape[0]
        self.n, self.bs, self.group, self.world = n, bs, group, world
        self.lo, self.hi = even_bounds(n, world, rank, 4 if n % 4 == 0 else 1)
        self.Wq = Wq[self.lo:self.hi].contiguous().to(device)
        self.sw = sw[self.lo:self.hi].contiguous().to(device)
        self.K = _default(kernels)

    def forward(self, q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
        return self.K.linear_f32(q, s, self.Wq, self.sw)

    def gather(self, y_local: torch.Tensor) -> torch.Tensor:
        """The full output (m x n) on every rank: all_gather of the column shards (exact copies)."""
        parts = [torch.empty((y_local.shape[0], hi - lo), dtype=y_local.dtype, device=y_local.device)
                 for lo, hi in (even_bounds(self.n, self.world, r, 4 if self.n % 4 == 0 else 1)
                                for r in range(self.world))]
        if self.world == 1:
            return y_local
        dist.all_gather(parts, y_local.contiguous(), group=self.group)
        return torch.cat(parts, dim=1)


class RowParallelLinear:
    """W (n x k) split by input columns on Hadamard-block boundaries; forward(x_shard) -> full output."""

    def __init__(self, Wq: torch.Tensor, sw: torch.Tensor, bs: int, rank: int, world: int, device, kernels=None,
                 group=None, bounds: tuple[int, int] | None = None, exchange: PeerExchange | None = None):
        n, k = Wq.shape
        self.n, self.k, self.bs, self.group, self.exchange = n, k, bs, group, exchange
        align = max(bs, 16)
        self.lo, self.hi = bounds if bounds is not None else even_bounds(k, world, rank, align)
        assert self.lo % align == 0 and self.hi % align == 0, "shards must hold whole Hadamard blocks"
        self.Wq = Wq[:, self.lo:self.hi].contiguous().to(device)
        self.sw = sw.contiguous().to(device)
        self.K = _default(kernels)

    def _solo(self) -> bool:
        return not (dist.is_available() and dist.is_initialized() and dist.get_world_size(self.group) > 1)

    def forward(self, x_shard: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        K = self.K
        if getattr(K, "fused", False) and self._solo():
            # one rank: the shard is the whole row, so its own absmax is the row's
            q, s = K.quant_act(x_shard, self.bs)
            return K.linear_resid(q, s, self.Wq, self.sw, residual)
        ex = self.exchange
        if ex is not None and getattr(K, "fused", False) and x_shard.shape[0] <= min(64, ex.tp.max_m) \
                and self.n <= ex.tp.max_n:
            # decode over NVLink: both all-reduces inside the kernels
            q, s = K.quant_act_tp(x_shard, self.bs, ex)
            return K.linear_resid_tp(q, s, self.Wq, self.sw, residual, ex)
        amax = K.fwht_absmax(x_shard, self.bs)
        _all_reduce(amax, dist.ReduceOp.MAX, self.group)
        q, s = K.quant_act_global(x_shard, self.bs, amax)
        acc = K.int_gemm(q, self.Wq)
        _all_reduce(acc, dist.ReduceOp.SUM, self.group)
        return K.dequant_residual(acc, s, self.sw, residual)


class TPMLP:
    """gate/up (2I x D, gate rows then up rows) and down (D x I) split over the ranks of `group`."""

    def __init__(self, gu_Wq, gu_sw, gu_bs: int, down_Wq, down_sw, down_bs: int, rank: int, world: int, device,
                 kernels=None, group=None, exchange: PeerExchange | None = None):
        I = down_Wq.shape[1]
        assert gu_Wq.shape[0] == 2 * I
        lo, hi = even_bounds(I, world, rank, max(down_bs, 16))
        self.gu_bs = gu_bs
        self.gu_Wq = torch.cat([gu_Wq[lo:hi], gu_Wq[I + lo:I + hi]]).contiguous().to(device)
        self.gu_sw = torch.cat([gu_sw[lo:hi], gu_sw[I + lo:I + hi]]).contiguous().to(device)
        self.down = RowParallelLinear(down_Wq, down_sw, down_bs, rank, world, device, kernels, group, (lo, hi),
                                      exchange)
        self.K = _default(kernels)

    def forward(self, r1: torch.Tensor, w_norm: torch.Tensor, eps: float) -> torch.Tensor:
        K = self.K
        q3, s3 = K.rmsnorm_quant(r1, w_norm, eps, self.gu_bs)
        if getattr(K, "fused", False):
            h = K.swiglu_linear(q3, s3, self.gu_Wq, self.gu_sw)
        else:
            h = K.swiglu(K.int_gemm(q3, self.gu_Wq), s3, self.gu_sw)
        return self.down.forward(h, residual=r1)
