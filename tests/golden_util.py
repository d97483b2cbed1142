"""Helpers to replay the golden fixtures (tests/golden/*.npz)."""
import importlib.util
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def load_module(name):
    """A module of tests/golden/ (make_golden.py: its tables, without running
    the generator, which needs the reference checkout)."""
    spec = importlib.util.spec_from_file_location(
        "_golden_" + name.replace(".py", ""), os.path.join(GOLDEN, name))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def runs():
    """RUNS table of make_golden.py."""
    return load_module("make_golden.py").RUNS


def bf16_to_f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def p_close(ours, ref, update_scale, rtol=1e-6):
    """Parameter agreement: |ours - ref| <= rtol * (|ref| + update_scale).

    ``update_scale`` is the largest per-element update the reference applied
    so far, so elements where p crosses zero are compared against the update
    size, not against |p| ~ 0.
    """
    ours = np.asarray(ours, np.float64)
    ref = np.asarray(ref, np.float64)
    tol = rtol * (np.abs(ref) + np.asarray(update_scale, np.float64))
    return np.abs(ours - ref) <= tol


def bf16_p_close(ours_bits, ref_bits, before, wdf, rtol=1e-6):
    """bf16 parameter agreement: the fp32 results before the final rounding
    agree as p_close says (rtol of |ref| plus the update), and rounding each
    to bf16 adds at most one ulp, so |ours - ref| <= ulp(ref) + rtol *
    (|ref| + |ref - before * wdf|). The update term matters where the update
    cancels the decayed parameter (the result is then tiny and an ulp of it
    says nothing about the update's accuracy)."""
    o = bf16_to_f32(ours_bits).astype(np.float64)
    r = bf16_to_f32(ref_bits).astype(np.float64)
    t = np.abs(r - np.asarray(before, np.float64) * float(wdf))
    return np.abs(o - r) <= np.abs(r) * 2.0 ** -7 + rtol * (np.abs(r) + t) + 1e-38
