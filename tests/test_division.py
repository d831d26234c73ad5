"""The bulk encoder's group normalisation divides every element of a group by the group
norm through one reciprocal (csrc/encode.cu, phase 2 of encode_tile_kernel):

    y = RN(1/n), q0 = RN(x*y), r = x - n*q0 (one FMA, exact), q = RN(q0 + r*y) (one FMA)

which must equal the IEEE quotient RN(x/n) that the oracle and the reference's encoder
(src/reference/production_math.py:4-24) compute, or codes would differ.  The identity is
IEEE arithmetic, so the host's correctly rounded operations check it: every finite FP16
numerator x (the encoder promotes FP16 keys) against divisors n >= |x| spread over the
norms' range, with all-ones significands among them.  Negative numerators are compared as
values: the quotient of -0 comes out +0, and no output of the encoder depends on the sign of
a zero (it only meets FMA chains, the code LUT's clamp and sums of squares).
"""
import ctypes
import shutil
import subprocess

import pytest

_SRC = r"""
#include <math.h>
#include <stdint.h>
#include <string.h>
static float bits(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }
static uint32_t ubits(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static float half_to_float(uint16_t h) {
    const uint32_t e = (h >> 10) & 31u, m = h & 1023u;
    if (e == 0) return ldexpf((float)m, -24);
    return bits(((e + 112u) << 23) | (m << 13));
}
long long check(int n_div, unsigned long long seed) {
    uint64_t s = seed | 1u;
    long long bad = 0;
    for (int ib = 0; ib < n_div; ++ib) {
        s ^= s << 13; s ^= s >> 7; s ^= s << 17;
        uint32_t mb = (uint32_t)(s & 0x7fffffu);
        if ((ib & 3) == 0) mb = 0x7fffffu - (uint32_t)(s >> 61);
        const uint32_t eb = 127u - 34u + (uint32_t)((s >> 23) % 55u);   /* n in [2^-34, 2^21) */
        const float n = bits((eb << 23) | mb);
        const float y = 1.0f / n;
        for (uint32_t h = 0; h < 0x7c00u; ++h) {
            const float x = half_to_float((uint16_t)h);
            if (!(x <= n)) break;
            volatile float q0 = x * y;
            const float r = fmaf(-n, q0, x);
            const float q = fmaf(r, y, q0);
            volatile float ref = x / n;
            if (ubits(q) != ubits(ref)) ++bad;
            volatile float xm = -x, q0m = xm * y;
            const float qm = fmaf(fmaf(-n, q0m, xm), y, q0m);
            volatile float refm = xm / n;
            if (qm != refm) ++bad;
        }
    }
    return bad;
}
"""


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    d = tmp_path_factory.mktemp("division")
    (d / "div.c").write_text(_SRC)
    so = d / "div.so"
    subprocess.run([gcc, "-O2", "-ffp-contract=off", "-fno-fast-math", "-shared", "-fPIC", "-o", str(so),
                    str(d / "div.c"), "-lm"], check=True)
    lib = ctypes.CDLL(str(so))
    lib.check.restype = ctypes.c_longlong
    lib.check.argtypes = [ctypes.c_int, ctypes.c_ulonglong]
    return lib


@pytest.mark.parametrize("seed", [1, 0x9E3779B97F4A7C15])
def test_reciprocal_division_equals_ieee_quotient(checker, seed):
    assert checker.check(1500, seed) == 0
