"""Shared checks for the parity tests."""
import numpy as np

# Tolerance for fp32 attention outputs against the reference's CPU attention:
# max-abs 1e-4 and rel 1e-3.
ATOL = 1e-4
RTOL = 1e-3


def assert_attn_close(out, ref, what=""):
    out = np.asarray(out, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    assert out.shape == ref.shape, (what, out.shape, ref.shape)
    assert np.isfinite(out).all(), f"{what}: non-finite output"
    err = np.abs(out.astype(np.float64) - ref.astype(np.float64))
    max_abs = float(err.max()) if err.size else 0.0
    assert max_abs <= ATOL, f"{what}: max-abs error {max_abs:.3e} > {ATOL}"
    np.testing.assert_allclose(out, ref, rtol=RTOL, atol=ATOL, err_msg=what)
    return max_abs
