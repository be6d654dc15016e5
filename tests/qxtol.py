"""Tolerances used by the parity tests.

The reference accumulates every dot product in double.  The engine forms exact
integer block sums on the tensor cores (int8 weights times a 56-bit fixed-point
activation) and folds them into double accumulators, so its floats normally
equal the reference's bit for bit; the tests still allow the stated bound.
Float vectors (logits, residuals, projections) must agree to 1e-4 relative in
the infinity norm:
    max|gpu - ref| <= REL * max|ref|.
Indices (top-8 experts, argmax tokens) must match exactly.
"""
import numpy as np

REL = 1e-4


def rel_err(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    scale = np.max(np.abs(want))
    return float(np.max(np.abs(got - want)) / (scale if scale > 0 else 1.0))


def assert_close(got, want, rel=REL, what="vector"):
    e = rel_err(got, want)
    assert e <= rel, "%s: relative error %.3g exceeds %.1g" % (what, e, rel)
