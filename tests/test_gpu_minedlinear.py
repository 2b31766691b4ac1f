"""GPU: uwc_b200.model.MinedLinear, the mined bf16 linear of miner/ampere/uwc_ampere/model.py, in
'mined' and 'plain' mode is bit-identical to the same integer math through cuBLAS ('int'), as the
reference's tests/test_model.py requires, and the fused quantizer tracks the torch rotation."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_mined_and_plain_equal_int_path(dev):
    import torch
    import torch.nn as nn

    from uwc_b200 import model as M
    torch.manual_seed(0)
    lins = [nn.Linear(2560, 4096, bias=False), nn.Linear(2560, 1024, bias=False)]
    a = M.MinedLinear(lins, "cuda", mode="int")
    b = M.MinedLinear(lins, "cuda", mode="mined")
    c = M.MinedLinear(lins, "cuda", mode="plain")
    assert b.mineable
    b.setup_block(lambda k: bytes(32), lambda k: np.zeros(8, np.uint32))
    x = torch.randn(3, 333, 2560, device="cuda", dtype=torch.bfloat16)      # m = 999, padded to 1024
    ya, yb, yc = a(x), b(x), c(x)
    assert ya.shape == yb.shape == yc.shape == (3, 333, 5120)
    assert torch.equal(ya, yb) and torch.equal(ya, yc)
    # independent of the library's GEMM: the int8 operands' exact product on the host
    import oracle as O
    from uwc_b200 import ops
    xq, sx = ops.quant_rows_had(x.reshape(-1, 2560).contiguous(), a.bs)
    acc = torch.from_numpy(O.gemm_i32(xq.cpu().numpy(), a.Wq.cpu().numpy()))
    want = ((acc.float() * sx.cpu().unsqueeze(1)) * a.sw.cpu().unsqueeze(0)).to(torch.bfloat16)
    assert torch.equal(ya.reshape(-1, 5120).cpu(), want)
    ref = x.float() @ torch.cat([l.weight for l in lins]).cuda().t()
    assert ((ya.float() - ref).norm() / ref.norm()).item() < 0.03


def test_fused_quantizer_matches_torch_rotation(dev):
    import torch

    from uwc_b200 import model as M
    from uwc_b200 import ops
    torch.manual_seed(1)
    x = (torch.randn(300, 2560, device="cuda") * torch.linspace(0.1, 8, 2560, device="cuda")).to(torch.bfloat16)
    for bs in (0, 128, 512):
        q, s = ops.quant_rows_had(x, bs)
        H = M.hadamard(bs, "cuda") if bs else None
        qr, sr = M.quant_rows(M.rotate(x.float(), H))
        assert torch.allclose(s, sr, rtol=1e-5)
        assert (q.int() - qr.int()).abs().max().item() <= 1          # only float rounding ties differ
        assert (q != qr).float().mean().item() < 1e-3


def test_convert_tiny_qwen3_mined_equals_int(dev):
    """convert_qwen3 on a whole model: mined logits == int logits bit for bit."""
    pytest.importorskip("transformers")
    import copy

    import torch

    import model_fixture as mf
    from uwc_b200 import model as M
    from transformers import Qwen3Config, Qwen3ForCausalLM
    torch.manual_seed(0)
    cfg = Qwen3Config(**dict(mf.CFG, hidden_size=2048, intermediate_size=4096))
    hf = Qwen3ForCausalLM(cfg).eval()
    hi, hm = copy.deepcopy(hf).cuda(), copy.deepcopy(hf).cuda()
    M.convert_qwen3(hi, "cuda", mode="int", hadamard_block=256)
    mined = M.convert_qwen3(hm, "cuda", mode="mined", hadamard_block=256)
    for ml in mined:
        ml.setup_block(lambda k: bytes(range(32)), lambda k: np.zeros(8, np.uint32))
    ids = torch.randint(0, 1024, (2, 64), device="cuda")
    with torch.no_grad():
        li, lm = hi(ids).logits, hm(ids).logits
    assert torch.equal(li, lm)
    assert sum(ml.hashed_macs for ml in mined) > 0, "no layer took the mined path"
