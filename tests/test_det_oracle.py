"""oracle/detq.py (the deterministic-linear producers and consumers) against vectors produced by
the reference's own runtime/detrt (tests/golden/make_golden_det.py): every array bit-identical."""
import numpy as np
import pytest

import detq as D


def _bits(a):
    a = np.asarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a


def _eq(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape or a.size == b.size
    assert np.array_equal(_bits(a.reshape(b.shape).astype(b.dtype)), _bits(b)), np.flatnonzero(a.reshape(b.shape) != b)[:10]


@pytest.mark.parametrize("bs", [0, 64, 512])
def test_quant_act(det_golden, bs):
    g = det_golden
    q, s = D.quant_act(g[f"qa{bs}_x"], bs)
    _eq(q, g[f"qa{bs}_q"])
    _eq(s, g[f"qa{bs}_s"])


def test_quant_act_global_equals_full_row(det_golden):
    """The row-parallel form: column shards quantized with the max over shards give the full row's q and scale."""
    x = det_golden["qa64_x"]
    q, s = D.quant_act(x, 64)
    amax = np.max([D.fwht_absmax(x[:, i * 256:(i + 1) * 256], 64) for i in range(4)], axis=0)
    parts = [D.quant_act_global(x[:, i * 256:(i + 1) * 256], 64, amax) for i in range(4)]
    _eq(np.concatenate([p[0] for p in parts], axis=1), q)
    for p in parts:
        _eq(p[1], s)


def test_rmsnorm_quant(det_golden):
    g = det_golden
    q, s = D.rmsnorm_quant(g["rq_x"], g["rq_w"], 1e-6, 128)
    _eq(q, g["rq_q"])
    _eq(s, g["rq_s"])


def test_swiglu_quant(det_golden):
    g = det_golden
    q, s = D.swiglu_quant(g["sg_acc"], g["sg_s3"], g["sg_sw"], 256)
    _eq(q, g["sg_q"])
    _eq(s, g["sg_s"])


def test_dequant_residual(det_golden):
    g = det_golden
    _eq(D.dequant_residual(g["dr_acc"], g["dr_s"], g["dr_sw"], g["dr_x"]), g["dr_out"])


@pytest.mark.parametrize("qk", [1, 0])
def test_qkv_post(det_golden, qk):
    g = det_golden
    res = D.qkv_post(g["qp_acc"], g["qp_s1"], g["qp_sw"], g["qp_qnw"], g["qp_knw"], g["qp_cos"], g["qp_sin"],
                     3, 2, 1, 1e-6, bool(qk))
    for name, a in zip(("qq", "qs", "kq", "ks", "vq", "vs"), res):
        _eq(a, g[f"qp{qk}_{name}"])


def test_det_exp_and_exact_rowsum(det_golden):
    g = det_golden
    _eq(D.det_exp(g["ex_z"]), g["ex_out"])
    _eq(D.exact_rowsum(g["rs_x"], 512), g["rs_out"])
