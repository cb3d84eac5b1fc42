"""Tolerance helpers shared by the parity tests."""
import numpy as np

# north_star tolerance for matmul outputs vs the fp32 oracle
MAX_REL = 1e-2
MIN_COS = 0.9999


def max_rel(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def cosine(got, ref):
    g = np.asarray(got, dtype=np.float64).ravel()
    r = np.asarray(ref, dtype=np.float64).ravel()
    return float(g @ r / max(np.linalg.norm(g) * np.linalg.norm(r), 1e-300))


def assert_close(got, ref, max_rel_tol=MAX_REL, min_cos=MIN_COS, what=""):
    mr, cs = max_rel(got, ref), cosine(got, ref)
    assert np.isfinite(np.asarray(got, dtype=np.float64)).all(), f"{what}: non-finite output"
    assert np.abs(np.asarray(got, dtype=np.float64)).max() > 0, f"{what}: output is all zero"
    assert mr <= max_rel_tol, f"{what}: max rel err {mr:.3e} > {max_rel_tol:.1e}"
    assert cs >= min_cos, f"{what}: cosine {cs:.6f} < {min_cos}"
    return mr, cs
