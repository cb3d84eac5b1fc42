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


def first_divergence(got, ref_tokens, ref_margins, tol, what=""):
    """Greedy tokens must equal the reference's at every step, except that at a
    step whose reference top-2 margin is below ``tol`` (the path's logit
    tolerance) either of the two tokens is a correct greedy choice; the
    trajectories may then part.  Returns the first differing step (printed with
    its margin) or None; fails on a difference anywhere else."""
    got = [int(t) for t in got]
    ref = [int(t) for t in ref_tokens]
    n = min(len(got), len(ref))
    for s in range(n):
        if got[s] != ref[s]:
            m = float(ref_margins[s])
            assert m < tol, (f"{what}: step {s} token {got[s]} != reference {ref[s]} although the reference's "
                             f"top-2 margin {m:.4f} >= tolerance {tol}")
            print(f"{what}: first divergence at step {s} of {n} (reference top-2 margin {m:.4f} < {tol})")
            return s
    print(f"{what}: all {n} tokens equal the reference's")
    return None


def softcap(x, cap):
    return cap * np.tanh(np.asarray(x, dtype=np.float64) / cap)


def check_top8(logits, top8_idx, top8_val, cap, tol, what=""):
    """One step's full logits (pre-softcap) against the reference's 8 largest
    softcapped logits: the values at the reference's ids within ``tol``, no
    other id above the reference's 8th value by more than ``tol``, and the same
    argmax unless the reference's top two are within ``tol``.  Returns the
    largest value error."""
    lg = softcap(logits, cap)
    idx = np.asarray(top8_idx, dtype=np.int64)
    ref = np.asarray(top8_val, dtype=np.float64)
    err = float(np.abs(lg[idx] - ref).max())
    assert err <= tol, f"{what}: top-8 logit error {err:.3e} > {tol}"
    rest = lg.copy()
    rest[idx] = -np.inf
    assert rest.max() <= ref[-1] + tol, (f"{what}: id {int(rest.argmax())} at {rest.max():.4f} outranks the "
                                         f"reference's 8th logit {ref[-1]:.4f}")
    if ref[0] - ref[1] >= tol:
        assert int(np.argmax(lg)) == int(idx[0]), f"{what}: argmax {int(np.argmax(lg))} != reference {int(idx[0])}"
    return err
