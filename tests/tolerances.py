"""Parity bars shared by the tests.

The north-star bar for the MoE path's output (moe_out, before the caller's
post-norm) is max-abs <= 2e-3 and rel-L2 <= 1e-3 against the reference's fp32
CPU path; top-k expert ids must match exactly except where adjacent router
probabilities are closer than 1e-6 (near ties).
"""
import numpy as np

MAX_ABS = 2e-3
REL_L2 = 1e-3
NEAR_TIE = 1e-6


def errors(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    mx = float(np.max(np.abs(got - ref))) if got.size else 0.0
    den = float(np.linalg.norm(ref))
    rel = float(np.linalg.norm(got - ref) / den) if den > 0 else mx
    return mx, rel


def assert_close(got, ref, max_abs=MAX_ABS, rel_l2=REL_L2, what=""):
    mx, rel = errors(got, ref)
    assert mx <= max_abs and rel <= rel_l2, f"{what}: max_abs={mx:.3e} rel_l2={rel:.3e}"
    return mx, rel


def near_tie_tokens(probs, k=8, gap=NEAR_TIE):
    """Tokens whose sorted router probabilities have an adjacent gap < `gap`
    among ranks 0..k (so the top-k set or order may legitimately differ)."""
    s = -np.sort(-np.asarray(probs, np.float64), axis=1)[:, : k + 1]
    return np.where(np.min(np.abs(np.diff(s, axis=1)), axis=1) < gap)[0]
