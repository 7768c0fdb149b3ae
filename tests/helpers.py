"""Shared comparison helpers for the parity tests."""
import numpy as np


def rms(x):
    x = np.asarray(x, np.float64)
    return float(np.sqrt(np.mean(x * x))) if x.size else 0.0


def assert_close(got, ref, rtol, atol_frac, what=""):
    """|got - ref| <= rtol*|ref| + atol_frac*rms(ref), element-wise."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    atol = atol_frac * rms(ref)
    err = np.abs(got - ref)
    bad = err > rtol * np.abs(ref) + atol
    if bad.any():
        i = np.unravel_index(np.argmax(err - rtol * np.abs(ref)), err.shape)
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{bad.size} elements out of tolerance "
            f"(rtol={rtol}, atol={atol:.3g}); worst at {i}: got {got[i]}, ref {ref[i]}")


def rel_fro(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(got - ref) / (np.linalg.norm(ref) + 1e-30))
