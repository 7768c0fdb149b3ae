"""Shared comparison helpers for the parity tests."""
import numpy as np

# GLA forward (o and the final state) against the fp32 oracle:
# |gpu - ref| <= GLA_RTOL |ref| + GLA_ATOL_FRAC rms(ref) element-wise and a
# relative Frobenius error below GLA_FRO.  The absolute term holds the
# reference template's own bf16 operand roundings, which a CPU emulation of
# every one of its casts measures at up to 3.2 % of rms on the inputs of
# tests/test_oracle_gla.py::test_reference_bf16_casts_stay_within_the_kernel_tolerance.
GLA_RTOL, GLA_ATOL_FRAC, GLA_FRO = 2e-2, 4e-2, 1e-2


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
