"""Tensor-parallel linears (uwc_b200/tp.py) on two gloo ranks on the CPU: the sharding, the MAX
all-reduce of the quantizer's row absmax and the int32 SUM all-reduce of the partial products give
bit-identical results to one device. The device kernels are replaced by the oracle (CPU) here; the
same classes run on NCCL with the CUDA kernels in tests/test_gpu_tp.py."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


class CPUKernels:
    """The tp backend interface implemented with the oracle (numpy)."""

    def __init__(self):
        import detq as D
        import oracle as O
        self.D, self.O = D, O

    @staticmethod
    def _n(t):
        return t.detach().cpu().numpy()

    def linear_f32(self, q, s, Wq, sw):
        return torch.from_numpy(self.O.det_dequant(self.O.gemm_i32(self._n(q), self._n(Wq)), self._n(s), self._n(sw)))

    def int_gemm(self, q, Wq):
        return torch.from_numpy(self.O.gemm_i32(self._n(q), self._n(Wq)))

    def fwht_absmax(self, x, bs):
        return torch.from_numpy(self.D.fwht_absmax(self._n(x), bs).astype(np.float32))

    def quant_act_global(self, x, bs, amax):
        q, s = self.D.quant_act_global(self._n(x), bs, self._n(amax))
        return torch.from_numpy(q), torch.from_numpy(s)

    def rmsnorm_quant(self, x, w, eps, bs):
        q, s = self.D.rmsnorm_quant(self._n(x), self._n(w), eps, bs)
        return torch.from_numpy(q), torch.from_numpy(s)

    def swiglu(self, acc, s3, sw):
        a = self._n(acc)
        I = a.shape[1] // 2
        gu = self.D.deq(a, self._n(s3), self._n(sw))
        return torch.from_numpy(self.D.fmul(self.D.det_silu(gu[:, :I]), gu[:, I:]))

    def dequant_residual(self, acc, s, sw, x):
        if x is None:
            return torch.from_numpy(self.D.deq(self._n(acc), self._n(s), self._n(sw)))
        return torch.from_numpy(self.D.dequant_residual(self._n(acc), self._n(s), self._n(sw), self._n(x)))


def _problem():
    import detq as D
    rng = np.random.default_rng(31)
    Dm, I, m = 256, 1536, 9
    W_gu = (rng.standard_normal((2 * I, Dm)) * 0.02).astype(np.float32)
    W_dn = (rng.standard_normal((Dm, I)) * 0.02).astype(np.float32)
    gq, gs = D.quant_act(W_gu, 128)
    dq, ds = D.quant_act(W_dn, 512)
    r1 = (rng.standard_normal((m, Dm)) * 3).astype(np.float32)
    wn = (1 + 0.1 * rng.standard_normal(Dm)).astype(np.float32)
    x = (rng.standard_normal((m, I)) * 0.7).astype(np.float32)
    return dict(gq=gq, gs=gs, dq=dq, ds=ds, r1=r1, wn=wn, x=x)


def _worker(rank, world, port, outdir):
    for p in (os.path.join(HERE, ".."), os.path.join(HERE, "..", "useful-work-coin_b200"),
              os.path.join(HERE, "..", "oracle"), HERE):
        sys.path.insert(0, os.path.abspath(p))
    import torch.distributed as dist
    from uwc_b200 import tp
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        P = _problem()
        K = CPUKernels()
        t = torch.from_numpy
        mlp = tp.TPMLP(t(P["gq"]), t(P["gs"]), 128, t(P["dq"]), t(P["ds"]), 512, rank, world, "cpu", K)
        y = mlp.forward(t(P["r1"]), t(P["wn"]), 1e-6)
        # row-parallel down alone on an uneven split (3 Hadamard blocks of 512 over 2 ranks)
        row = tp.RowParallelLinear(t(P["dq"]), t(P["ds"]), 512, rank, world, "cpu", K)
        z = row.forward(t(P["x"][:, row.lo:row.hi]).contiguous())
        # column-parallel gate/up, gathered
        col = tp.ColumnParallelLinear(t(P["gq"]), t(P["gs"]), 128, rank, world, "cpu", K)
        q, s = K.rmsnorm_quant(t(P["r1"]), t(P["wn"]), 1e-6, 128)
        g = col.gather(col.forward(q, s))
        np.savez(os.path.join(outdir, f"rank{rank}.npz"), y=y.numpy(), z=z.numpy(), g=g.numpy(),
                 lo=row.lo, hi=row.hi)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tensor_parallel_layers_bit_identical_on_gloo(tmp_path):
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    import detq as D
    import oracle as O
    P = _problem()
    q3, s3 = D.rmsnorm_quant(P["r1"], P["wn"], 1e-6, 128)
    q4, s4 = D.swiglu_quant(O.gemm_i32(q3, P["gq"]), s3, P["gs"], 512)
    y_ref = D.dequant_residual(O.gemm_i32(q4, P["dq"]), s4, P["ds"], P["r1"])
    qx, sx = D.quant_act(P["x"], 512)
    z_ref = D.deq(O.gemm_i32(qx, P["dq"]), sx, P["ds"])
    g_ref = O.det_dequant(O.gemm_i32(q3, P["gq"]), s3, P["gs"])
    outs = [dict(np.load(os.path.join(tmp_path, f"rank{r}.npz"))) for r in range(2)]
    assert (int(outs[0]["lo"]), int(outs[0]["hi"]), int(outs[1]["hi"])) == (0, 1024, 1536)
    for o in outs:
        for name, ref in (("y", y_ref), ("z", z_ref), ("g", g_ref)):
            assert np.array_equal(o[name].view(np.uint32), ref.view(np.uint32)), name


@pytest.mark.parametrize("n,world,align", [(28672, 8, 1), (14336, 8, 512), (1536, 2, 512), (100, 3, 4)])
def test_even_bounds_cover_and_align(n, world, align):
    from uwc_b200 import tp
    b = [tp.even_bounds(n, world, r, align) for r in range(world)]
    assert b[0][0] == 0 and b[-1][1] == n
    assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))
    assert all(lo % align == 0 and hi % align == 0 for lo, hi in b)
    sizes = [hi - lo for lo, hi in b]
    assert max(sizes) - min(sizes) <= align
