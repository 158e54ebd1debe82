"""The coalesced core in two calls (moe_run_moe_coalesced_stage1 / stage2)
against the one-call core, on the GPU.

Port of test_split_moe_overlap.mojo:12-110: sub_b = 5 tokens routed by the
set-cover rule from the test's top-8 pattern ((b*7 + k*13) % 128, values
0.30 - 0.032k, per-expert scales 0.85 + 0.3*((e*19) % 29)/29), weight bytes
(i*11 + 5) & 255 / (i*19 + 9) & 255 with scales 0.012 / 0.011, inputs
(((i*29) % 23) - 11) * 0.04 in the deinterleaved layout; the split result
must equal the monolithic one bit for bit.  Here another library call runs
between the two halves, and the bucket arrays are checked against a numpy
restatement of moe_kernels.mojo:815-835.
"""
import numpy as np
import pytest

import moe_b200 as MB

pytestmark = pytest.mark.gpu

E, D, F, K = 128, 2816, 704, 8


@pytest.fixture(scope="module")
def pattern_weights():
    import torch
    def pat(n, mul, add):
        return ((torch.arange(n, device="cuda", dtype=torch.int64) * mul + add) & 255).to(torch.uint8)
    gu_p = pat(E * 2 * F * D // 2, 11, 5)
    gu_s = torch.full((E * 2 * F * D // 32,), 0.012, device="cuda")
    dn_p = pat(E * D * F // 2, 19, 9)
    dn_s = torch.full((E * D * F // 32,), 0.011, device="cuda")
    return gu_p, gu_s, dn_p, dn_s


def _routing(ctx, sub_b):
    top_idx = np.array([[(b * 7 + k * 13) % E for k in range(K)] for b in range(sub_b)], np.int64)
    top_val = np.array([[0.30 - 0.032 * k for k in range(K)] for _ in range(sub_b)], np.float32)
    pes = np.array([0.85 + 0.3 * ((e * 19) % 29) / 29.0 for e in range(E)], np.float32)
    cnt = np.zeros(sub_b, np.int64)
    idx = np.zeros((sub_b, K), np.int64)
    w = np.zeros((sub_b, K), np.float32)
    ctx.compute_subbatch_set_cover_moe_weights(sub_b, top_idx, top_val, pes, 1.0, cnt, idx, w,
                                               num_experts=E, top_k=K)
    return cnt, idx, w


def _buckets(cnt, idx, w):
    """moe_kernels.mojo:815-835 in numpy."""
    bc = np.zeros(E, np.int64)
    bt = np.zeros(E * 5, np.int64)
    bw = np.zeros(E * 5, np.float32)
    for b in range(len(cnt)):
        for k in range(cnt[b]):
            e = idx[b, k]
            bt[e * 5 + bc[e]] = b
            bw[e * 5 + bc[e]] = w[b, k]
            bc[e] += 1
    ue = np.nonzero(bc)[0]
    return bc, bt, bw, ue, np.concatenate([[0], np.cumsum(bc[ue])[:-1]]).astype(np.int64)


@pytest.mark.parametrize("sub_b", [5, 1], ids=["five-tokens-tensor-cores", "one-token-cuda-cores"])
def test_split_equals_monolithic_bit_for_bit(ctx, pattern_weights, sub_b):
    gu_p, gu_s, dn_p, dn_s = pattern_weights
    cnt, idx, w = _routing(ctx, sub_b)
    x = ((((np.arange(sub_b * D) * 29) % 23) - 11) * 0.04).astype(np.float32)
    mono = np.zeros((sub_b, D), np.float32)
    ctx.run_moe_coalesced_core(sub_b, gu_p, gu_s, dn_p, dn_s, x, cnt, idx, w, mono,
                               x_layout=MB.X_DEINT_HALVES)
    bc = np.full(E, -1, np.int64)
    bt = np.zeros(E * 5, np.int64)
    bw = np.zeros(E * 5, np.float32)
    ue = np.zeros(E, np.int64)
    ub = np.zeros(E, np.int64)
    act_deint = np.zeros(40 * F, np.float32)
    nu = ctx.run_moe_coalesced_stage1(sub_b, gu_p, gu_s, x, cnt, idx, w, bc, bt, bw, ue, ub, None, None,
                                      act_deint, x_layout=MB.X_DEINT_HALVES)
    rbc, rbt, rbw, rue, rub = _buckets(cnt, idx, w)
    assert nu == len(rue)
    np.testing.assert_array_equal(bc, rbc)
    np.testing.assert_array_equal(bt, rbt)
    np.testing.assert_array_equal(bw, rbw)
    np.testing.assert_array_equal(ue[:nu], rue)
    np.testing.assert_array_equal(ub[:nu], rub)
    # other work on the same context between the halves (what the split is for)
    other = np.zeros((3, 1024), np.float32)
    ctx.q4_matmul_batchN(3, dn_p, dn_s, np.ones((3, 2816), np.float32), other, 2816, 1024)
    split = np.zeros((sub_b, D), np.float32)
    ctx.run_moe_coalesced_stage2(sub_b, nu, dn_p, dn_s, bc, bt, bw, ue, ub, act_deint, split)
    assert np.isfinite(split).all() and np.abs(split).max() > 0
    np.testing.assert_array_equal(split, mono)


def test_stage2_needs_its_stage1(ctx, pattern_weights):
    gu_p, gu_s, dn_p, dn_s = pattern_weights
    cnt, idx, w = _routing(ctx, 5)
    x = np.ones(5 * D, np.float32)
    bufs = [np.zeros(E, np.int64), np.zeros(E * 5, np.int64), np.zeros(E * 5, np.float32),
            np.zeros(E, np.int64), np.zeros(E, np.int64)]
    act_a, act_b = np.zeros(40 * F, np.float32), np.zeros(40 * F, np.float32)
    out = np.zeros((5, D), np.float32)
    nu = ctx.run_moe_coalesced_stage1(5, gu_p, gu_s, x, cnt, idx, w, *bufs, None, None, act_a)
    with pytest.raises(MB.MoeError) as e:  # another scratch: not this result
        ctx.run_moe_coalesced_stage2(5, nu, dn_p, dn_s, *bufs, act_b, out)
    assert e.value.code == 8
    with pytest.raises(MB.MoeError) as e:  # different sub_b
        ctx.run_moe_coalesced_stage2(4, nu, dn_p, dn_s, *bufs, act_a, out)
    assert e.value.code == 1
    ctx.run_moe_coalesced_stage2(5, nu, dn_p, dn_s, *bufs, act_a, out)
    with pytest.raises(MB.MoeError) as e:  # consumed
        ctx.run_moe_coalesced_stage2(5, nu, dn_p, dn_s, *bufs, act_a, out)
    assert e.value.code == 8
    with pytest.raises(MB.MoeError) as e:  # the reference's limit of five tokens
        ctx.run_moe_coalesced_stage1(6, gu_p, gu_s, np.ones(6 * D, np.float32), np.zeros(6, np.int64),
                                     np.zeros((6, K), np.int64), np.zeros((6, K), np.float32), *bufs,
                                     None, None, act_a)
    assert e.value.code == 2
