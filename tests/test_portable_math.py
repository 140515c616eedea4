"""The exp / erf shared by the CPU oracle and the reference-arithmetic kernels
(crispembed_b200/csrc/ceb_portable_math.h) round correctly: against the double
results of Python's math module rounded once to float, on seeded arguments over
the ranges the encoder meets (softmax and attention exponents, GELU inputs), and
they stay within one ulp of the C library's expf / erff they stand in for."""
import ctypes
import ctypes.util
import math

import numpy as np
import pytest


@pytest.fixture(scope="module")
def lib(oracle):
    return oracle.lib()


def _args(rng, lo, hi, n):
    return rng.uniform(lo, hi, n).astype(np.float32)


def _ulps(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(a - b)


@pytest.mark.parametrize("lo,hi", [(-104.0, 0.0), (-20.0, 20.0), (-1e-3, 1e-3), (0.0, 88.7)])
def test_expf_correctly_rounded(lib, lo, hi):
    rng = np.random.default_rng(11)
    xs = _args(rng, lo, hi, 20000)
    mine = np.array([lib.ceo_expf(float(x)) for x in xs], np.float32)
    ref = np.array([math.exp(float(x)) for x in xs], np.float64).astype(np.float32)
    assert int((mine != ref).sum()) == 0


@pytest.mark.parametrize("lo,hi", [(-6.0, 6.0), (-2.01, -1.99), (-1e-4, 1e-4), (3.0, 5.0)])
def test_erff_correctly_rounded(lib, lo, hi):
    rng = np.random.default_rng(12)
    xs = _args(rng, lo, hi, 20000)
    mine = np.array([lib.ceo_erff(float(x)) for x in xs], np.float32)
    ref = np.array([math.erf(float(x)) for x in xs], np.float64).astype(np.float32)
    assert int((mine != ref).sum()) == 0


def test_special_values(lib):
    assert lib.ceo_expf(float("-inf")) == 0.0
    assert lib.ceo_expf(0.0) == 1.0
    assert math.isinf(lib.ceo_expf(89.5))
    assert lib.ceo_expf(-110.0) == 0.0
    assert math.isnan(lib.ceo_expf(float("nan")))
    assert lib.ceo_erff(0.0) == 0.0
    assert lib.ceo_erff(10.0) == 1.0 and lib.ceo_erff(-10.0) == -1.0


def test_within_one_ulp_of_libm(lib):
    libm = ctypes.CDLL(ctypes.util.find_library("m"))
    for f in (libm.expf, libm.erff):
        f.argtypes = [ctypes.c_float]
        f.restype = ctypes.c_float
    rng = np.random.default_rng(13)
    xs = _args(rng, -30.0, 30.0, 20000)
    assert _ulps([lib.ceo_expf(float(x)) for x in xs], [libm.expf(float(x)) for x in xs]).max() <= 1
    xs = _args(rng, -6.0, 6.0, 20000)
    assert _ulps([lib.ceo_erff(float(x)) for x in xs], [libm.erff(float(x)) for x in xs]).max() <= 1
