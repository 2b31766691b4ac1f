"""CPU-side checks of the boundary: the C-ABI library loads and exports every symbol that
include/uwc_b200.h declares, argument validation rejects bad shapes before touching a device,
and the host constants match the reference's definitions. No kernel runs here."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "uwc_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(uwc_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from uwc_b200 import _lib
    L = _lib.lib()
    names = declared_functions()
    assert len(names) >= 10, names
    for name in names:
        assert hasattr(L, name), f"{name} declared in uwc_b200.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_library_has_no_driver_link_dependency():
    """The .so must load on a host without libcuda (static cudart, driver entry points at run time)."""
    import shutil
    import subprocess
    from uwc_b200 import _lib
    if shutil.which("readelf"):
        dyn = subprocess.run(["readelf", "-d", _lib.LIB_PATH], capture_output=True, text=True).stdout
        needed = re.findall(r"\(NEEDED\).*\[(.+?)\]", dyn)
        assert needed and not any(n.startswith(("libcuda.", "libcudart.")) for n in needed), needed
    _lib.lib()  # loads without a driver on a CPU-only host


def test_status_strings_and_version():
    from uwc_b200 import _lib
    L = _lib.lib()
    assert L.uwc_version() >= 100
    for code in range(7):
        assert L.uwc_status_string(code)
    assert L.uwc_status_string(0) == b"ok"


def test_shape_validation_needs_no_device():
    from uwc_b200 import _lib
    L = _lib.lib()
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: validation fails first
    # hashed GEMM with m % 64 != 0
    rc = L.uwc_gemm(fake, fake, 100, 256, 1024, 128, 1, None, None, None, 0, fake, fake, fake, 4, None, None, None, 0,
                    fake, 1 << 30, None)
    assert rc == _lib.ERR_SHAPE
    # k % r != 0
    rc = L.uwc_gemm(fake, fake, 128, 256, 1000, 128, 1, None, None, None, 0, fake, fake, fake, 4, None, None, None, 0,
                    fake, 1 << 30, None)
    assert rc == _lib.ERR_SHAPE
    # bad out_mode / flags
    assert L.uwc_gemm(fake, fake, 128, 256, 1024, 128, 8, None, None, None, 0, None, None, None, 0, None, None, None, 0,
                      None, 0, None) == _lib.ERR_ARG
    # unaligned operand
    bad = ctypes.c_void_p(0x1001)
    assert L.uwc_gemm(bad, fake, 128, 256, 1024, 128, 0, None, None, None, 0, None, None, None, 0, None, None, fake, 1,
                      None, 0, None) == _lib.ERR_ALIGN
    # BLAKE3 input not a multiple of 1 KiB
    assert L.uwc_b3_root_and_seed(fake, 1000, fake, None, None, 0, None, None, fake, 64, None) == _lib.ERR_SHAPE
    # noise_rows rank must be 64/128/256
    assert L.uwc_noise_rows(fake, 8, 1024, 96, None, None, None, None, None, -1, -1, None, 0, None) == _lib.ERR_SHAPE
    # perm rank must be a power of two
    assert L.uwc_noise_perm(fake, 1024, 96, fake, fake, None) == _lib.ERR_SHAPE


def test_scratch_words():
    from uwc_b200 import ops
    assert ops.b3_scratch_words(1024) == 8
    assert ops.b3_scratch_words(128 * 1024) == 8
    assert ops.b3_scratch_words(129 * 1024) == 16
    n = 1024 * 128 * 1024 + 1024  # more than 1024 CTA values -> an extra reduce level
    assert ops.b3_scratch_words(n) == 8 * 1025 + 8 * 2


def test_constants_match_reference_definitions():
    blake3 = pytest.importorskip("blake3").blake3
    from uwc_b200 import ops
    assert ops.SEED_SALT_A == blake3(b"pearl/cert-v3/noise-seed/A").digest()
    assert ops.SEED_SALT_B == blake3(b"pearl/cert-v3/noise-seed/B").digest()
    import oracle as O
    for k in (64, 1024, 2048, 4096, 8192, 1 << 20):
        assert ops.limbs_for(k) == O.limbs_for(k)
    assert (ops.FLAG_HASH, ops.FLAG_DENOISE, ops.OUT_NONE, ops.OUT_I32, ops.OUT_BF16, ops.WIN_WORDS) == (1, 2, 0, 1, 2,
                                                                                                      10)


def test_glue_helpers():
    import oracle as O
    from uwc_b200 import glue
    for nbits in (0x1D00FFFF, 0x1E00FFFF, 0x03123456, 0x01800000, 0x207FFFFF):
        assert glue.nbits_to_target(nbits) == O.nbits_to_target(nbits)
    b = ((1 << 256) - 1) // 12345
    assert np.array_equal(glue.bound_words(b), O.bound_words(b))
    assert glue.AMPERE_ROWS == [0, 8, 16, 24, 32, 40, 48, 56]
    assert glue.AMPERE_COLS[:4] == [0, 1, 8, 9] and len(glue.AMPERE_COLS) == 16
    # penalized bound picks the smaller of the two (pearl_glue.py:55-62)
    t = glue.nbits_to_target(0x1E00FFFF)
    assert glue.jackpot_bound(0x1E00FFFF, 2048, 128, 4) == min(t * 128 * 2048, t * 128 * 16 * 4)


def test_attention_and_batched_gemm_validation_needs_no_device():
    from uwc_b200 import _lib
    L = _lib.lib()
    f = ctypes.c_void_p(0x1000)
    gb = lambda *a: L.uwc_gemm_batched(f, f, *a, f, None)
    assert gb(128, 258, 128, 2, 128, 258, 1, 0, 0, 0) == _lib.ERR_SHAPE      # n % 4
    assert gb(128, 256, 120, 2, 128, 256, 1, 0, 0, 0) == _lib.ERR_SHAPE      # k % 16
    assert gb(128, 256, 128, 2, 100, 256, 1, 0, 0, 0) == _lib.ERR_SHAPE      # a_brows < m
    assert gb(256, 128, 256, 2, 256, 128, 1, 2, 0, 100) == _lib.ERR_SHAPE    # qrows % 128
    assert gb(128, 256, 128, 2, 128, 256, 0, 0, 0, 0) == _lib.ERR_ARG        # b_bdiv
    assert gb(128, 256, 128, 2, 128, 256, 1, 3, 0, 0) == _lib.ERR_ARG        # causal mode
    at = lambda B, Tq, start, H, Hkv, ws: L.uwc_attention_tc(f, f, f, f, f, f, B, Tq, start, H, Hkv, 1 << 20, 128, 1 << 16,
                                                             1 << 13, 1, 1 << 9, 0.088, f, f, ws, None)
    assert at(2, 256, 0, 6, 4, 1 << 40) == _lib.ERR_SHAPE                   # H % Hkv
    assert at(1, 1024, 131000, 2, 2, 1 << 40) == _lib.ERR_SHAPE             # start + Tq > 2^17
    need = L.uwc_attention_tc_workspace_bytes(2, 256, 0, 4, 2)
    assert need > 0 and at(2, 256, 0, 4, 2, need - 1) == _lib.ERR_SCRATCH


def test_attention_tc_workspace_and_path_selection():
    """The tensor-core attention's workspace (query / key / transposed value gathers, key and
    value scales, int32 scores, P limbs, int32 P V rows, P scales, each 256-byte aligned) and the
    automatic choice between it and the SIMT kernel."""
    from uwc_b200 import detgpu
    from uwc_b200._lib import lib
    up = lambda x, a: (x + a - 1) // a * a
    for B, Tq, start, H, Hkv in ((8, 2048, 0, 16, 8), (2, 300, 40, 4, 2), (1, 129, 1000, 8, 1)):
        nb, nkv, Tp, S = B * H, B * Hkv, up(Tq, 128), start + Tq
        Sp, Sn = up(S, 128), up(S, 4)
        parts = [nb * Tp * 128, nkv * Sp * 128, nkv * 128 * Sp, nkv * Sp * 4, nkv * Sp * 4, nb * Tp * Sn * 4,
                 nb * 2 * Tp * Sp, nb * 2 * Tp * 128 * 4, nb * Tp * 4]
        assert lib().uwc_attention_tc_workspace_bytes(B, Tq, start, H, Hkv) == sum(up(p, 256) for p in parts)
    assert detgpu.use_tensor_cores(8, 2048, 0, 16, 8)                       # the C4 prefill
    assert not detgpu.use_tensor_cores(8, 127, 0, 16, 8)                    # short prefills
    assert not detgpu.use_tensor_cores(8, 1, 2100, 16, 8)                   # decode
    assert not detgpu.use_tensor_cores(1, 13000, 0, 16, 8)                  # scores beyond shared memory
    assert not detgpu.use_tensor_cores(64, 8192, 0, 32, 8)                  # workspace above the cap
    assert detgpu.use_tensor_cores(1, 1, 0, 2, 2, "tc") and not detgpu.use_tensor_cores(8, 2048, 0, 16, 8, "simt")
    with pytest.raises(ValueError):
        detgpu.use_tensor_cores(1, 1, 0, 2, 2, "fast")
