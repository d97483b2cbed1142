"""Arithmetic primitives of ta_math.h (host build), CPU only.

* Philox4x32-10 against the known-answer vectors published with the
  algorithm (Random123 distribution, kat_vectors);
* ta_logf / ta_expf max error < 1 ulp over strided scans of the binary32
  range plus special values (the full exhaustive scan is in
  test_math_exhaustive, marked slow);
* fp32 -> fp16 round-to-nearest-even against numpy.
"""
import os

import numpy as np
import pytest


@pytest.mark.parametrize(
    "ctr,key,expect",
    [
        ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
        ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
        ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
         (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
    ],
)
def test_philox_kat(oracle, ctr, key, expect):
    out = oracle.philox(ctr, key)
    assert tuple(int(x) for x in out) == expect


def test_log_exp_special_values(oracle):
    x = np.array([1.0, 2.0, 0.5, 1e-38, 1e-45, 3.4e38, np.inf], np.float32)
    y = oracle.logf(x)
    ref = np.log(x.astype(np.float64))
    assert np.isinf(y[-1])
    ulp = np.spacing(np.abs(ref[:-1]).astype(np.float32)).astype(np.float64)
    assert (np.abs(y[:-1] - ref[:-1]) < ulp).all()
    assert y[0] == 0.0
    e = oracle.expf(np.array([0.0, -200.0, 200.0, np.nan], np.float32))
    assert e[0] == 1.0 and e[1] == 0.0 and np.isinf(e[2]) and np.isnan(e[3])


def test_log_strided_scan(oracle):
    # every 97th positive binary32 pattern: ~22M inputs incl. subnormals
    worst, bad = 0.0, 0
    for lo in range(1, 0x7F800000, 0x04000000):
        hi = min(lo + 0x04000000, 0x7F800000)
        m, b = oracle.scan_log(lo, lo + (hi - lo) // 97)
        worst, bad = max(worst, m), bad + b
    assert bad == 0 and worst < 1.0


def test_exp_strided_scan(oracle):
    worst, bad = 0.0, 0
    # [-110, 100] in both signs, sampled in slices
    for lo in list(range(0x00000000, 0x42C80000, 0x02000000)) + list(
            range(0x80000000, 0xC2DC0000, 0x02000000)):
        m, b = oracle.scan_exp(lo, lo + 0x00100000)
        worst, bad = max(worst, m), bad + b
    assert bad == 0 and worst < 1.0


@pytest.mark.skipif(not os.environ.get("TA_EXHAUSTIVE"), reason="set TA_EXHAUSTIVE=1 (minutes)")
def test_math_exhaustive(oracle):
    m, b = oracle.scan_log(1, 0x7F800000)
    assert b == 0 and m < 1.0
    m1, b1 = oracle.scan_exp(0, 0x42C80000)
    m2, b2 = oracle.scan_exp(0x80000000, 0xC2DC0001)
    assert b1 == 0 and b2 == 0 and max(m1, m2) < 1.0


def test_fp16_conversion(oracle):
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * 10.0 ** rng.uniform(-9, 5, 200000),
        np.array([65504, 65519.99, 65520, 65536, 1e-8, 2.0 ** -25, 2.0 ** -24, 5.96e-8,
                  -0.0, np.inf, -np.inf], np.float32),
        rng.uniform(-90, 90, 100000).astype(np.float32),
    ]).astype(np.float32)
    got = oracle.f32_to_f16_bits(x)
    ref = x.astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(got, ref)


FAST_V_MIN = np.float32(2.0 ** -99)  # ta_kernels.cuh: blocks with a smaller v_new take the exact path


def test_fast_range_lies_inside_the_certified_log_domain(oracle):
    """Unflagged blocks have v_new >= 2^-99, so every log the fast paths take
    (approximate per element, exact for the block extremes) is >= -69.3: the
    domain over which the lg2 error bound of the certified re-quantisation is
    measured (ta_selftest_fast_math)."""
    assert oracle.logf(np.array([FAST_V_MIN], np.float32))[0] > -69.3
    # and everything below the flag -- zero, subnormals, tiny normals -- is flagged
    assert not np.any(np.arange(0, 1 << 23, dtype=np.uint32).view(np.float32) >= FAST_V_MIN)


def test_fast_log_equals_exact_log_in_range(oracle):
    """The paired log of the block extremes is ta_logf bit for bit on every
    input the fast path gives it (normal, >= 2^-99, finite)."""
    bits = np.arange(FAST_V_MIN.view(np.uint32), 0x7F800000, 61, dtype=np.uint32)
    x = bits.view(np.float32)
    np.testing.assert_array_equal(oracle.logf_fast(x).view(np.uint32),
                                  oracle.logf(x).view(np.uint32))
