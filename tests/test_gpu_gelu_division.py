"""The GELU vector body divides by the erf denominator with an FMA-refined
reciprocal instead of an IEEE division (exactmath.cuh div_erf). The quotient
depends on the clamped t alone and reaches the output only through 1 + erf, so
checking 1 + quotient for every float t in [-4, 4] against the IEEE quotient
proves the GeGLU epilogue keeps the reference's VDIVPS result
(linalg/gelu_amd64.s:165-225) for every input."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_division_equals_ieee_for_every_t(igdev):
    from indecis_b200 import _capi
    L = _capi.load()
    bad = (C.c_int64 * 2)(-1, -1)
    first = C.c_uint32(0)
    hist = np.zeros((2, 256), np.int64)
    _capi.check(L.ig_check_gelu_division(bad, C.byref(first), hist.ctypes.data))
    where = {int(e): int(hist[1, e]) for e in np.nonzero(hist[1])[0]}
    raw = {int(e): int(hist[0, e]) for e in np.nonzero(hist[0])[0]}
    print("quotients differing by exponent of t:", raw)
    assert bad[1] == 0, f"{bad[1]} values of 1 + erf differ (first |t| bits {first.value:#010x}); by exponent {where}"
