"""CPU: the integer-rounding identities the deterministic kernels use instead of conversion
instructions (det_math.cuh floor_small / rint_small / int_of_small / float_of_small) give the same
values as floorf, rintf and the int <-> float conversions over the ranges the kernels feed them.
IEEE single-precision addition and subtraction round identically on the host and the GPU, so a
host check in C (with the rounding mode set explicitly) stands for the device code. Every float in
the ranges is visited with a stride; the small-integer conversion is checked for every integer."""
import ctypes
import os
import shutil
import subprocess
import tempfile

import pytest

SRC = r"""
#include <fenv.h>
#include <math.h>
#include <stdint.h>
#include <string.h>
#pragma STDC FENV_ACCESS ON
static float fi(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t uf(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static const float M = 12582912.0f;          /* 1.5 * 2^23 */
static const uint32_t MB = 0x4B400000u;      /* its bits */

/* returns the number of mismatches over every stride-th float in [lo, hi) */
long check_floor(float lo, float hi, uint32_t stride) {
  long bad = 0;
  for (uint64_t u = 0; u < 0x100000000ull; u += stride) {
    float t = fi((uint32_t)u);
    if (!(t >= lo && t < hi)) continue;
    fesetround(FE_DOWNWARD);
    volatile float s = t + M;
    fesetround(FE_TONEAREST);
    volatile float f = s - M;
    if (f != floorf(t) || (int)(uf(s) - MB) != (int)floorf(t)) bad++;
  }
  return bad;
}
long check_rint(float lo, float hi, uint32_t stride) {
  long bad = 0;
  for (uint64_t u = 0; u < 0x100000000ull; u += stride) {
    float x = fi((uint32_t)u);
    if (!(x >= lo && x <= hi)) continue;
    volatile float s = x + M;
    volatile float r = s - M;
    float y = rintf(x);
    volatile float s2 = y + M;
    if (r != y || (int)(uf(s2) - MB) != (int)y) bad++;
  }
  return bad;
}
long check_i2f(void) {
  long bad = 0;
  for (int d = -(1 << 22) + 1; d < (1 << 22); d++) {
    volatile float f = fi(MB + (uint32_t)d) - M;
    if (f != (float)d) bad++;
  }
  return bad;
}
"""


@pytest.fixture(scope="module")
def lib():
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    d = tempfile.mkdtemp()
    src, so = os.path.join(d, "r.c"), os.path.join(d, "r.so")
    open(src, "w").write(SRC)
    subprocess.check_call([cc, "-O2", "-frounding-math", "-shared", "-fPIC", src, "-o", so, "-lm"])
    L = ctypes.CDLL(so)
    for f in ("check_floor", "check_rint"):
        getattr(L, f).argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_uint32]
        getattr(L, f).restype = ctypes.c_long
    L.check_i2f.restype = ctypes.c_long
    yield L
    shutil.rmtree(d, ignore_errors=True)


def test_floor_for_det_exp(lib):
    # det_exp clamps t = z log2(e) to [-126, 128) before taking its floor
    assert lib.check_floor(-126.0, 128.0, 97) == 0


def test_rint_for_the_quantizers(lib):
    # quant_sym(64) rounds |x| <= 64 (1 + 2^-22); the attention's 14-bit P rounds x in [0, 16383 (1 + 2^-22)]
    assert lib.check_rint(-70.0, 16400.0, 97) == 0


def test_small_int_to_float(lib):
    # the attention dots: |q . k| <= 127 * 127 * 128 < 2^22
    assert lib.check_i2f() == 0
