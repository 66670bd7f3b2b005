"""Parity metric of the hot path: relative L2 <= 2e-3 and max-abs <= 1e-2 * max|ref| per output
tensor against the CPU oracle (the reference's own CPU kernels restated), as BASELINE's north star
states. Integer / index work (shapes, offsets) is compared exactly elsewhere."""
import numpy as np

REL_L2 = 2e-3
MAX_ABS_FRAC = 1e-2


def metrics(got, ref):
    got = np.asarray(got, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.all(np.isfinite(got)), "non-finite values in the CUDA output"
    den = np.linalg.norm(ref)
    rel = np.linalg.norm(got - ref) / (den if den > 0 else 1.0)
    mx = np.abs(ref).max() if ref.size else 0.0
    mabs = np.abs(got - ref).max() if ref.size else 0.0
    return rel, mabs, mx


def assert_close(got, ref, what="", rel_l2=REL_L2, max_abs_frac=MAX_ABS_FRAC):
    rel, mabs, mx = metrics(got, ref)
    assert rel <= rel_l2 and mabs <= max_abs_frac * max(mx, 1e-30), (
        f"{what}: rel-L2 {rel:.3e} (bound {rel_l2:.1e}), max-abs {mabs:.3e} (bound {max_abs_frac * mx:.3e})")
    return rel, mabs
