"""Cases of the diffusion router-subspace FFN bypass shared by the oracle
test (CPU) and the GPU parity test.

``known_answers`` transcribes the reference's own test,
test_diffusion_suite.mojo:562-648 (read as text; Mojo cannot run here): a
32-token batch over a 64-position canvas (token b at position 2b), 16
experts, top-8 ids (b + s) % 16 with id 15 in slot 1 of token 0
(:297-302), then
  1. step 2: tokens 0-7 stationary with matching top-2 (bypassed), 8-15 with
     a flipped second expert, 16-23 with a large logit drift, 24-31 not
     accepted: 24 evaluated, the first of them b = 8 (:562-587);
  2. an uninitialised prev_top2 (-1) is never a match (:589-604);
  3. a drift of 0.035 per step is bypassed once, but the second step's
     cumulative 0.070 is caught, because r_prev only moves on evaluation
     (:606-627);
  4. the scatter restores a bypassed row from the cache and scatters an
     evaluated one into the output and the cache (:629-648).

``random_filter_case`` builds larger seeded cases whose drifts sit around
the tau boundary, so that any deviation from the reference's summation order
would flip decisions.
"""
import numpy as np

B, NUM_EXP, TOP_K, CANVAS, EMBED_DIM = 32, 16, 8, 64, 256


def known_answers(filt, scatter):
    """filt(r_curr, r_prev, top_idx, prev_top2, eb, act, keep, B, E, K, step, tau) -> count
    (updating r_prev / prev_top2 / keep in place); scatter(sub, cache, full, act, keep, B,
    len, dim) in place on cache / full (fp16 rows)."""
    top_idx = np.array([[(b + s) % NUM_EXP for s in range(TOP_K)] for b in range(B)], np.int64)
    top_idx[0, 1] = 15
    r_curr = np.zeros((B, NUM_EXP), np.float32)
    r_prev = np.zeros((CANVAS, NUM_EXP), np.float32)
    prev_top2 = np.full((CANVAS, 2), -1, np.int64)
    eb = np.zeros(CANVAS, np.uint8)
    act = np.arange(B, dtype=np.int64) * 2
    keep = np.zeros(B, np.int64)
    base = ((np.arange(NUM_EXP) % 9) - 4).astype(np.float32) * np.float32(0.2)
    for b in range(B):
        o = 2 * b
        eb[o] = 1 if b < 24 else 0
        prev_top2[o, 0] = top_idx[b, 0]
        prev_top2[o, 1] = top_idx[b, 1] if (b < 8 or b >= 16) else top_idx[b, 1] + 1
        r_prev[o] = base
        r_curr[b] = base if (b < 16 or b >= 24) else base + np.float32(0.5)
    n = filt(r_curr, r_prev, top_idx, prev_top2, eb, act, keep, B, NUM_EXP, TOP_K, 2, 0.05)
    assert n == 24 and keep[0] == 8, (n, keep[:4])

    prev_top2[0] = -1
    saved = top_idx[0, :2].copy()
    top_idx[0, :2] = -1
    assert filt(r_curr, r_prev, top_idx, prev_top2, eb, act, keep, 1, NUM_EXP, TOP_K, 2, 0.05) == 1
    top_idx[0, :2] = saved

    prev_top2[0] = top_idx[0, :2]
    r_prev[0] = 1.0
    r_curr[0] = np.float32(1.035)
    assert filt(r_curr, r_prev, top_idx, prev_top2, eb, act, keep, 1, NUM_EXP, TOP_K, 1, 0.05) == 0
    r_curr[0] = np.float32(1.070)
    assert filt(r_curr, r_prev, top_idx, prev_top2, eb, act, keep, 1, NUM_EXP, TOP_K, 2, 0.05) == 1

    sub = np.full((1, EMBED_DIM), 7.25, np.float16)
    cache = np.zeros((CANVAS, EMBED_DIM), np.float16)
    cache[0] = 2.5
    cache[2] = 1.0
    full = np.zeros((2, EMBED_DIM), np.float16)
    keep[0] = 1
    scatter(sub, cache, full, act, keep, 2, 1, EMBED_DIM)
    assert np.all(full[0] == np.float16(2.5)) and np.all(full[1] == np.float16(7.25))
    assert np.all(cache[2] == np.float16(7.25)) and np.all(cache[0] == np.float16(2.5))


def random_filter_case(seed, B=256, E=128, K=8, canvas=512, tau=0.05):
    """Seeded inputs of one filter step.  Rows draw their drift so that the
    relative change sits within a few percent of tau, a fifth of them match
    the previous top-2 only in the first expert, some are not accepted."""
    rng = np.random.default_rng(seed)
    act = rng.permutation(canvas)[:B].astype(np.int64)
    r_prev = rng.standard_normal((canvas, E)).astype(np.float32)
    top_idx = np.stack([rng.permutation(E)[:K] for _ in range(B)]).astype(np.int64)
    prev_top2 = np.full((canvas, 2), -1, np.int64)
    prev_top2[act] = top_idx[:, :2]
    flip = rng.random(B) < 0.2
    prev_top2[act[flip], 1] = (top_idx[flip, 1] + 1) % E
    prev_top2[act[rng.random(B) < 0.05]] = -1
    eb = (rng.random(canvas) < 0.85).astype(np.uint8)
    direction = rng.standard_normal((B, E)).astype(np.float32)
    direction /= np.linalg.norm(direction, axis=1, keepdims=True)
    rel = tau * (1.0 + rng.uniform(-0.03, 0.03, B)).astype(np.float32)
    norm = np.linalg.norm(r_prev[act], axis=1)
    r_curr = (r_prev[act] + direction * (rel * norm)[:, None]).astype(np.float32)
    still = rng.random(B) < 0.1  # stationary rows: bypassed whenever the rest allows
    r_curr[still] = r_prev[act[still]]
    top_w = rng.random((B, K)).astype(np.float32)
    return dict(r_curr=r_curr, r_prev=r_prev, top_idx=top_idx, prev_top2=prev_top2, eb=eb, act=act,
                top_w=top_w, B=B, E=E, K=K, canvas=canvas, tau=tau)


def random_rows_case(seed, B, canvas, dim, dtype):
    """Rows and a keep list for the sync / scatter row copies: a strictly
    increasing prefix followed, in odd seeds, by an entry that breaks the
    order (the reference's in-order walk never reaches what follows it)."""
    rng = np.random.default_rng(seed)
    act = rng.permutation(canvas)[:B].astype(np.int64)
    kept = np.sort(rng.choice(B, size=max(1, B // 2), replace=False)).astype(np.int64)
    if seed % 2:
        cut = len(kept) // 2
        kept = np.concatenate([kept[:cut], kept[max(0, cut - 3):]])  # goes back: walk stops there
    out = rng.standard_normal((B, dim)).astype(dtype)
    cache = rng.standard_normal((canvas, dim)).astype(dtype)
    sub = rng.standard_normal((len(kept), dim)).astype(dtype)
    return dict(act=act, keep=kept, out=out, cache=cache, sub=sub)
