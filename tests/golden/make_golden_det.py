"""Generate tests/golden/det_golden.npz from the reference's own deterministic runtime (detrt).

Run in a checkout that has the reference next to it (not needed by the tests themselves):
    python tests/golden/make_golden_det.py <path to srivassid/useful-work-coin>

Every output comes from runtime/detrt/core.py (quant_act, det_rmsnorm, det_silu, det_exp,
exact_rowsum, quant_sym) composed the way runtime/detrt/fast.py:108-190 composes them, on seeded
inputs. The fixtures pin oracle/detq.py (tests/test_det_oracle.py) and the GPU kernels
(tests/test_gpu_det.py).
"""
from __future__ import annotations

import os
import sys

import numpy as np


def main(ref: str) -> None:
    sys.path.insert(0, os.path.join(ref, "runtime"))
    import torch
    from detrt import core
    from detrt.core import F32, fadd, fmul

    rng = np.random.default_rng(20261201)
    out: dict[str, np.ndarray] = {}
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))

    def deq(acc, s, sw):
        return fmul(fmul(t(acc).to(F32), t(s)[:, None]), t(sw)[None, :])

    # quant_act at several Hadamard block sizes (0 = none), rows with very different ranges
    for bs in (0, 64, 512):
        x = (rng.standard_normal((6, 1024)) * rng.choice([1e-3, 0.05, 3.0, 40.0], (6, 1))).astype(np.float32)
        x[2, :7] = 0.0
        q, s = core.quant_act(t(x), bs)
        out[f"qa{bs}_x"], out[f"qa{bs}_q"], out[f"qa{bs}_s"] = x, q.numpy(), s.numpy()

    # det_rmsnorm + quant_act (detgpu rmsnorm_quant)
    x = (rng.standard_normal((5, 768)) * rng.choice([1e-2, 1.0, 25.0], (5, 1))).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(768)).astype(np.float32)
    q, s = core.quant_act(core.det_rmsnorm(t(x), t(w), 1e-6), 128)
    out.update(rq_x=x, rq_w=w, rq_q=q.numpy(), rq_s=s.numpy())

    # swiglu_quant: quant_act(fmul(det_silu(gate), up)) of the dequantized gate/up GEMM output
    I = 512
    acc = rng.integers(-(1 << 21), 1 << 21, size=(4, 2 * I), dtype=np.int32)
    s3 = (rng.random(4) * 1e-4 + 1e-6).astype(np.float32)
    sw = (rng.random(2 * I) * 1e-2 + 1e-4).astype(np.float32)
    gu = deq(acc, s3, sw)
    q, s = core.quant_act(fmul(core.det_silu(gu[:, :I]), gu[:, I:]), 256)
    out.update(sg_acc=acc, sg_s3=s3, sg_sw=sw, sg_q=q.numpy(), sg_s=s.numpy())

    # dequant_residual: fadd(x, deq(acc))
    acc = rng.integers(-(1 << 24), 1 << 24, size=(3, 384), dtype=np.int32)
    s = (rng.random(3) * 1e-4).astype(np.float32)
    sw = (rng.random(384) * 1e-2).astype(np.float32)
    x = rng.standard_normal((3, 384)).astype(np.float32)
    out.update(dr_acc=acc, dr_s=s, dr_sw=sw, dr_x=x, dr_out=fadd(t(x), deq(acc, s, sw)).numpy())

    # qkv_post: dequant, split, per-head RMSNorm (Qwen3) or none (Llama), rope, quant_sym(127)
    T, B, H, Hkv, hd = 3, 2, 2, 1, 128
    N = B * T
    acc = rng.integers(-(1 << 20), 1 << 20, size=(N, (H + 2 * Hkv) * hd), dtype=np.int32)
    s1 = (rng.random(N) * 1e-4 + 1e-6).astype(np.float32)
    sw = (rng.random((H + 2 * Hkv) * hd) * 1e-2 + 1e-4).astype(np.float32)
    qnw = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    knw = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    ang = np.arange(T)[:, None] * (1.0 / (1e6 ** (np.arange(0, hd, 2) / hd)))[None, :]
    emb = np.concatenate([ang, ang], axis=1)
    cos, sin = np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)
    out.update(qp_acc=acc, qp_s1=s1, qp_sw=sw, qp_qnw=qnw, qp_knw=knw, qp_cos=cos, qp_sin=sin)
    qkv = deq(acc, s1, sw)
    pos = torch.arange(T).repeat(B)
    cs, sn = t(cos)[pos][:, None, :], t(sin)[pos][:, None, :]
    half = hd // 2
    rope = lambda z: fadd(fmul(z, cs), fmul(torch.cat([-z[..., half:], z[..., :half]], -1), sn))
    for qk in (1, 0):
        q, k, v = torch.split(qkv, [H * hd, Hkv * hd, Hkv * hd], dim=-1)
        qn, kn = q.reshape(N, H, hd), k.reshape(N, Hkv, hd)
        if qk:
            qn, kn = core.det_rmsnorm(qn, t(qnw), 1e-6), core.det_rmsnorm(kn, t(knw), 1e-6)
        qq, qs = core.quant_sym(rope(qn), 127)
        kq, ks = core.quant_sym(rope(kn), 127)
        vq, vs = core.quant_sym(v.reshape(N, Hkv, hd), 127)
        for name, a in (("qq", qq), ("qs", qs), ("kq", kq), ("ks", ks), ("vq", vq), ("vs", vs)):
            a = a.numpy()
            out[f"qp{qk}_{name}"] = a.astype(np.int8) if name.endswith("q") else a.astype(np.float32)

    # det_exp / exact_rowsum edge cases
    z = np.concatenate([rng.standard_normal(64) * 30, [0.0, -0.0, -87.0, -88.0, -104.0, 88.0, 88.8, 89.0, 1e-30,
                                                      -1e-30, np.inf, -np.inf, np.nan]]).astype(np.float32)
    out.update(ex_z=z, ex_out=core.det_exp(t(z)).numpy())
    rs = (rng.standard_normal((4, 300)) * rng.choice([1e-20, 1.0, 1e20], (4, 1))).astype(np.float32)
    out.update(rs_x=rs, rs_out=core.exact_rowsum(t(rs), 512).numpy())

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "det_golden.npz")
    np.savez_compressed(path, **out)
    print(path, sum(a.nbytes for a in out.values()), "bytes")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("UWC_REFERENCE", "../useful-work-coin"))
