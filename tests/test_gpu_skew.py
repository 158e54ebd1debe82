"""The skewed prefill layer against the CPU oracle.

Config 5 routes 4 x 2048 tokens through the layer with a Zipf(1.1) bias on
the router logits, scaled so that the busiest expert takes about 5x the mean
load.  Its hot experts then hold hundreds to thousands of tokens, so their
gate/up and down GEMMs run with token tiles wider than 64 on the general
tensor-core kernel (dequantised weights staged in shared memory), a path the
decode-sized tests do not reach.

The oracle applies the same bias before its softmax (oracle/moe_oracle.c,
orc_route).  Routing is compared for every token (top-k ids exact except near
ties).  A token's output depends on that token alone, so the expert outputs
are compared on a sample of tokens, half of them routed to the busiest
expert, while the GPU evaluates the whole batch (the tiling under test
depends on the whole batch's loads).
"""
import numpy as np
import pytest

import moe_b200 as MB
import oracle as O
import synth
from tolerances import assert_close, near_tie_tokens

pytestmark = pytest.mark.gpu
K, E = 8, 128


def _route(ctx, desc, M, x):
    cnt = np.zeros(M, np.int64)
    idx = np.zeros((M, K), np.int64)
    w = np.zeros((M, K), np.float32)
    ctx.route(desc, M, x, cnt, idx, w)
    return cnt, idx, w


def _loads(cnt, idx):
    act = idx[np.arange(K)[None, :] < cnt[:, None]]
    return np.bincount(act, minlength=E)


def _calibrated_bias(ctx, dev, M, x, target=5.0):
    """Zipf(1.1) bias whose scale puts the busiest expert at `target` x the
    mean load (bisection with the library's router)."""
    import torch
    lo, hi = 0.0, 1.0
    for _ in range(12):
        mid = 0.5 * (lo + hi)
        b = torch.from_numpy(synth.zipf_bias(E, 1.1, mid, seed=0)).cuda()
        loads = _loads(*_route(ctx, MB.make_desc(dev, bias=b), M, x)[:2])
        if loads.max() / loads.mean() < target:
            lo = mid
        else:
            hi = mid
    return synth.zipf_bias(E, 1.1, 0.5 * (lo + hi), seed=0)


def _probs(scores, bias):
    s = scores.astype(np.float64) + bias[None, :]
    s = np.exp(s - s.max(1, keepdims=True))
    return s / (s.sum(1, keepdims=True) + 1e-10)


@pytest.mark.parametrize("M,n_sample", [(2048, 320), (8192, 256)])
def test_skewed_prefill_layer_vs_oracle(ctx, full_layer, M, n_sample):
    import torch
    dev, host, _ = full_layer
    x_dev = synth.make_x(M, seed=500 + M)
    x = x_dev.cpu().numpy()
    bias = _calibrated_bias(ctx, dev, M, x_dev)
    desc = MB.make_desc(dev, bias=torch.from_numpy(bias).cuda())
    L = O.make_layer(host, bias=bias)

    out = np.zeros((M, 2816), np.float32)
    cnt = np.zeros(M, np.int64)
    idx = np.zeros((M, K), np.int64)
    w = np.zeros((M, K), np.float32)
    ctx.layer_forward(desc, M, x, out, 0, cnt, idx, w)

    # the skew is real: the hot experts' token tiles are wider than 64
    loads = _loads(cnt, idx)
    assert loads.max() >= 4.0 * loads.mean(), loads.max() / loads.mean()
    assert loads.max() > 256, loads.max()

    # routing of every token against the oracle (near ties exempt)
    ref = O.route(L, x)
    ties = set(near_tie_tokens(_probs(ref["scores"], bias), K).tolist())
    bad = [t for t in range(M) if t not in ties and not (
        cnt[t] == ref["count"][t] and np.array_equal(idx[t, :cnt[t]], ref["idx"][t, :cnt[t]]))]
    assert not bad, f"top-k mismatch outside near ties on {len(bad)} tokens, first {bad[:8]}"
    same = np.array([t for t in range(M) if t not in ties])
    for t in same[:512]:
        np.testing.assert_allclose(w[t, :cnt[t]], ref["w"][t, :cnt[t]], rtol=2e-5, atol=1e-7)

    # expert outputs on a sample: every token of the busiest expert (up to
    # half the sample), the rest drawn at random
    hot = int(np.argmax(loads))
    hot_toks = [t for t in same if hot in idx[t, :cnt[t]]]
    rng = np.random.default_rng(M)
    pick = list(hot_toks[: n_sample // 2])
    rest = np.setdiff1d(same, pick)
    pick += list(rng.choice(rest, n_sample - len(pick), replace=False))
    pick = np.array(sorted(pick))
    moe_ref = O.experts_forward(L, ref["moe_in"][pick], ref["count"][pick], ref["idx"][pick],
                                ref["w"][pick], prec=O.F64)
    assert_close(out[pick], moe_ref, what=f"skewed layer M={M} (busiest expert {loads.max()} tokens)")
