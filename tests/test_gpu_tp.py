"""Tensor-parallel linears on 2+ GPUs with this library's CUDA kernels: the MLP block at
Llama-3.1-8B widths (hidden 4096, MLP 14336), at decode (M = 32) and prefill-like M, with the
all-reduces over NCCL and (decode) inside the kernels over NVLink peer memory, eager and as a
replayed CUDA graph: bit-identical to the same layer on one GPU. Skipped with fewer than 2 GPUs."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _weights(Dm, I):
    g = torch.Generator().manual_seed(8)
    gq = torch.randint(-64, 65, (2 * I, Dm), dtype=torch.int8, generator=g)
    dq = torch.randint(-64, 65, (Dm, I), dtype=torch.int8, generator=g)
    gs = torch.rand(2 * I, generator=g) * 1e-3 + 1e-5
    ds = torch.rand(Dm, generator=g) * 1e-3 + 1e-5
    wn = 1 + 0.1 * torch.randn(Dm, generator=g)
    return gq, gs, dq, ds, wn


def _worker(rank, world, port, outdir, Dm, I, ms):
    for p in (os.path.join(HERE, ".."), os.path.join(HERE, "..", "useful-work-coin_b200")):
        sys.path.insert(0, os.path.abspath(p))
    import torch.distributed as dist
    from uwc_b200 import tp
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        gq, gs, dq, ds, wn = _weights(Dm, I)
        mlp = tp.TPMLP(gq, gs, 512, dq, ds, 512, rank, world, dev)
        res = {}
        for m in ms:
            r1 = (torch.randn(m, Dm, generator=torch.Generator().manual_seed(m)) * 2).to(dev)
            res[f"y{m}"] = mlp.forward(r1, wn.to(dev), 1e-5).cpu().numpy()
        # the same block with both all-reduces inside the kernels (NVLink peer exchange): eager calls,
        # then a CUDA graph replayed several times (the exchange's epochs advance on the device)
        ex = tp.PeerExchange(64, Dm, rank, world, dev)
        try:
            mlpx = tp.TPMLP(gq, gs, 512, dq, ds, 512, rank, world, dev, exchange=ex)
            for m in ms:
                r1 = (torch.randn(m, Dm, generator=torch.Generator().manual_seed(m)) * 2).to(dev)
                res[f"x{m}"] = mlpx.forward(r1, wn.to(dev), 1e-5).cpu().numpy()
            # the GEMM's exchange in its other form (reduce-scatter + all-gather below 8 ranks,
            # one-shot at 8), same bits
            from uwc_b200 import _lib
            _lib.lib().uwc_test_hook(_lib.HOOK_TP_TWO_PHASE, world if world < 8 else 9)
            m = ms[0]
            r1 = (torch.randn(m, Dm, generator=torch.Generator().manual_seed(m)) * 2).to(dev)
            res[f"p{m}"] = mlpx.forward(r1, wn.to(dev), 1e-5).cpu().numpy()
            _lib.lib().uwc_test_hook(_lib.HOOK_TP_TWO_PHASE, 8)
            m = ms[0]
            r1 = (torch.randn(m, Dm, generator=torch.Generator().manual_seed(m)) * 2).to(dev)
            wnd = wn.to(dev)
            st = torch.cuda.Stream()
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                mlpx.forward(r1, wnd, 1e-5)
            torch.cuda.current_stream().wait_stream(st)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                yg = mlpx.forward(r1, wnd, 1e-5)
            for i in range(5):
                graph.replay()
            torch.cuda.synchronize()
            res[f"g{m}"] = yg.cpu().numpy()
            del graph
            from uwc_b200 import _lib
            res["status"] = np.array([_lib.device_status(clear=True)])
        finally:
            ex.close()
        torch.cuda.synchronize()
        np.savez(os.path.join(outdir, f"rank{rank}.npz"), **res)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_mlp_nccl_matches_one_gpu(tmp_path):
    world = min(torch.cuda.device_count(), 8)
    Dm, I, ms = 4096, 14336, (32, 300)
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), Dm, I, ms), nprocs=world, join=True)
    from uwc_b200 import detgpu

    class Lin:
        def __init__(self, Wq, sw, bs):
            self.Wq, self.sw, self.bs = Wq.cuda(), sw.cuda(), bs
    gq, gs, dq, ds, wn = _weights(Dm, I)
    gu, down = Lin(gq, gs, 512), Lin(dq, ds, 512)
    for m in ms:
        r1 = (torch.randn(m, Dm, generator=torch.Generator().manual_seed(m)) * 2).cuda()
        ref = detgpu.mlp_residual(gu, down, wn.cuda(), r1, 1e-5).cpu().numpy()
        for r in range(world):
            got = np.load(os.path.join(tmp_path, f"rank{r}.npz"))
            assert int(got["status"][0]) == 0, r
            for key in (f"y{m}", f"x{m}") + ((f"g{m}", f"p{m}") if m == ms[0] else ()):
                assert np.array_equal(got[key].view(np.uint32), ref.view(np.uint32)), (key, r)
