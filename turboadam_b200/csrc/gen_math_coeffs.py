"""Generate the polynomial coefficients used by ta_math.h.

Run: python turboadam_b200/csrc/gen_math_coeffs.py
Prints C initialisers (float32, exact hex-float) for

  * log1p kernel  Q(f) = (log1p(f) - f) / f^2   on f in [-1/3, 1/3]   (degree 9)
  * exp kernel    P(r) = (e^r - 1 - r) / r^2     on |r| <= ln(2)/2     (degree 5)

The fits are Chebyshev (near-minimax) approximations computed with mpmath at
40 digits and then rounded to binary32. The resulting functions are checked
exhaustively for max-ulp error by tests/test_math.py through the oracle build.
"""
import mpmath as mp

mp.mp.dps = 40


def _q(f):
    f = mp.mpf(f)
    if abs(f) < mp.mpf("1e-25"):
        return mp.mpf(-0.5) + f / 3
    return (mp.log1p(f) - f) / (f * f)


def _p(r):
    r = mp.mpf(r)
    if abs(r) < mp.mpf("1e-25"):
        return mp.mpf(0.5) + r / 6
    return (mp.exp(r) - 1 - r) / (r * r)


def _fit(fn, lo, hi, deg):
    coeffs, err = mp.chebyfit(fn, [lo, hi], deg + 1, error=True)
    # chebyfit returns highest degree first
    return [float(mp.mpf(c)) for c in coeffs], err


def _f32_hex(x):
    import numpy as np
    return float(np.float32(x)).hex()


def main():
    third = mp.mpf(1) / 3
    qc, qe = _fit(_q, -third, third, 9)
    half_ln2 = mp.log(2) / 2 + mp.mpf("0.002")
    pc, pe = _fit(_p, -half_ln2, half_ln2, 5)
    print("/* log1p kernel Q(f), degree 9, highest first; fit error %s */" % mp.nstr(qe, 4))
    print("static const float TA_LOG_Q[10] = {%s};" % ", ".join(_f32_hex(c) + "f" for c in qc))
    print("/* exp kernel P(r), degree 5, highest first; fit error %s */" % mp.nstr(pe, 4))
    print("static const float TA_EXP_P[6] = {%s};" % ", ".join(_f32_hex(c) + "f" for c in pc))


if __name__ == "__main__":
    main()
