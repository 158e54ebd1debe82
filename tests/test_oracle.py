"""CPU tests of the oracle (the checker), pinned to the reference's own fixtures.

* Q4_0 quantizer: bit-exact against tests/golden/q4_golden.npz, produced by the
  reference's numpy quantizer (convert_gemma4_moe.py:9-35).
* Routing helpers: the known answers of test_moe_lod_top_p.mojo:28-49,
  test_kernels.mojo:3021-3053 and test_set_cover_moe.mojo:24-118.
* Expert stages: the fp32 restatement agrees with the fp64 scalar oracle the
  way the reference's own tests require (test_moe_lod_top_p.mojo:195 <= 1e-5,
  test_spec_verify_and_coalesce.mojo:201 <= 1e-6 for coalesced vs per-token).
"""
import json
import os

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def q4_golden():
    return np.load(os.path.join(GOLD, "q4_golden.npz"))


@pytest.fixture(scope="module")
def known():
    with open(os.path.join(GOLD, "known_answers.json")) as f:
        return json.load(f)


def test_quantizer_bit_exact_vs_reference(q4_golden):
    names = sorted({k.split("__")[0] for k in q4_golden.files})
    assert len(names) >= 6
    for n in names:
        p, s, ties = O.quantize_q4_0(q4_golden[n + "__x"])
        assert ties == 0, n
        assert np.array_equal(p, q4_golden[n + "__packed"]), n
        assert np.array_equal(s.view(np.uint32), q4_golden[n + "__scales"].view(np.uint32)), n


def test_quantizer_nibble_layout():
    # element 2j -> low nibble of byte j, 2j+1 -> high nibble (moe_kernels.mojo:45-51)
    x = np.zeros(32, np.float32)
    x[0], x[1], x[31] = 7.0, -7.0, 3.0
    p, s, _ = O.quantize_q4_0(x)
    assert s[0] == np.float32(1.0)
    assert p[0] == (7 + 8) | ((-7 + 8) << 4)
    assert p[15] == (0 + 8) | ((3 + 8) << 4)


def test_softmax_vs_numpy():
    g = np.load(os.path.join(GOLD, "softmax_golden.npz"))
    for i in range(3):
        p = O.softmax(g[f"case{i}__x"])
        assert np.max(np.abs(p - g[f"case{i}__p"])) <= 1e-5  # test_kernels.mojo:511


def test_top_k_known_answer(known):
    ka = known["top_k"]
    idx, val = O.get_top_k(np.array(ka["probs"], np.float32), 8)
    assert idx.tolist() == ka["expect_idx"]
    assert val.tolist() == ka["expect_val"]


def test_top_k_ties_keep_lower_index():
    p = np.array([0.5, 0.2, 0.2, 0.1, 0.2], np.float32)
    idx, _ = O.get_top_k(p, 4)
    assert idx.tolist() == [0, 1, 2, 4]


def test_lod_known_answer(known):
    ka = known["lod"]
    pes = np.ones(128, np.float32)
    n, _, _ = O.compute_moe_lod_weights(ka["top_idx"], ka["top_val"], pes, 1.0)
    assert n == ka["expect_count_top_p_1"]
    n, _, w = O.compute_moe_lod_weights(ka["top_idx"], ka["top_val"], pes, 0.80)
    assert n == ka["expect_count_top_p_080"]
    assert abs(w[:n].sum() - ka["expect_weight_sum_top_p_080"]) <= ka["tol_weight_sum"]


def test_lod_nan_top_p_is_lossless(known):
    ka = known["lod"]
    pes = np.ones(128, np.float32)
    n, _, _ = O.compute_moe_lod_weights(ka["top_idx"], ka["top_val"], pes, float("nan"))
    assert n == ka["expect_count_top_p_1"]


def _set_cover_case(known):
    sc = known["set_cover"]
    ti = np.zeros((5, 8), np.int64)
    tv = np.zeros((5, 8), np.float32)
    ti[0], tv[0] = sc["b0_idx"], sc["b0_val"]
    for b in range(1, 5):
        ti[b] = [10, 20, 30 + b, 40, 50, 60, 90 + 2 * b, 91 + 2 * b]
        tv[b] = sc["bk_val"]
    pes = np.array([0.8 + 0.4 * ((e * 17) % 31) / 31.0 for e in range(128)], np.float32)
    return sc, ti, tv, pes


def test_set_cover_known_answer(known):
    sc, ti, tv, pes = _set_cover_case(known)
    cnt, idx, w = O.set_cover(ti, tv, pes, 1.0)
    n0, i0, w0 = O.compute_moe_lod_weights(ti[0], tv[0], pes, 1.0)
    assert cnt[0] == n0 and np.array_equal(idx[0, :n0], i0[:n0]) and np.array_equal(w[0, :n0], w0[:n0])
    for b in range(1, 5):
        assert cnt[b] == sc["expect_count_b_ge_1"]
        assert set(idx[b, : cnt[b]].tolist()) == {10, 20, 30 + b, 40, 50, 60}
        unscaled = sum(w[b, k] / pes[idx[b, k]] for k in range(cnt[b]))
        assert abs(unscaled - sc["expect_renorm_sum"]) <= sc["tol_renorm_sum"]


def test_apply_lod_and_set_cover():
    rng = np.random.default_rng(5)
    B, K = 6, 8
    p = rng.dirichlet(np.ones(16), B).astype(np.float32)
    ti = np.argsort(-p, 1)[:, :K].astype(np.int64)
    tv = np.take_along_axis(p, ti, 1).astype(np.float32)
    pes = np.ones(128, np.float32)
    w = O.apply_moe_lod_and_set_cover(ti, tv, pes, B, K, 8, 1.0)
    for b in range(B):
        norm = tv[b] / (tv[b].sum() + np.float32(1e-10))
        exp = np.where(norm >= np.float32(0.05), norm, 0)
        np.testing.assert_allclose(w[b], exp, rtol=1e-6, atol=0)
    eb = np.array([1, 0, 1, 0, 1, 0], np.uint8)
    w2 = O.apply_moe_lod_and_set_cover(ti, tv, pes, B, K, 8, 1.0, eb_mask=eb, unaccepted_top_k=2)
    for b in (1, 3, 5):
        assert np.count_nonzero(w2[b, 2:]) == 0


def _pattern_experts(n_exp, d, F):
    """Byte/scale patterns of test_moe_lod_top_p.mojo:62-71."""
    rows = 2 * F
    gp = ((np.arange(n_exp * rows * d // 2) * 13 + 7) & 255).astype(np.uint8)
    gs = (((np.arange(n_exp * rows * d // 32) % 19) + 1) * 0.002).astype(np.float32)
    dp = ((np.arange(n_exp * d * F // 2) * 29 + 3) & 255).astype(np.uint8)
    ds = (((np.arange(n_exp * d * F // 32) % 17) + 1) * 0.002).astype(np.float32)
    x = (((np.arange(d) % 31) - 15) * 0.03).astype(np.float32)
    return gp, gs, dp, ds, x


def test_stages_f32_port_vs_f64_pattern():
    d, F = 2816, 704
    gp, gs, dp, ds, x = _pattern_experts(8, d, F)
    idx = np.arange(5, dtype=np.int64)
    w = np.full(5, 0.2, np.float32)
    _, a32 = O.experts_stage1(gp, gs, x, idx, d, F, prec=O.F32)
    _, a64 = O.experts_stage1(gp, gs, x, idx, d, F, prec=O.F64)
    np.testing.assert_allclose(a32, a64, rtol=1e-4, atol=1e-4)
    o32 = O.experts_stage2(dp, ds, a32, idx, w, d, F, prec=O.F32)
    o64 = O.experts_stage2(dp, ds, a32, idx, w, d, F, prec=O.F64)
    assert np.max(np.abs(o32 - o64)) <= 1e-5 * max(1.0, np.max(np.abs(o64)))


def test_stage_active_count_zero_and_small_dims():
    # test_q4_4row_tiling.mojo:200-245 edge cases: active_count 0 zeroes moe_out
    d, F = 64, 32
    gp, gs, dp, ds, x = _pattern_experts(8, d, F)
    out = O.experts_stage2(dp, ds, np.zeros((1, F), np.float32), np.zeros(0, np.int64),
                           np.zeros(0, np.float32), d, F)
    assert np.all(out == 0)
    idx = np.arange(8, dtype=np.int64)
    _, a = O.experts_stage1(gp, gs, x[:d], idx, d, F, prec=O.F32, nthreads=7)
    _, a1 = O.experts_stage1(gp, gs, x[:d], idx, d, F, prec=O.F32, nthreads=1)
    assert np.array_equal(a, a1)


def test_q4_matmul_remainders_f32_vs_f64():
    # test_q4_4row_tiling.mojo:127-193: c_out=67, 707 and the heap path c_in=8224
    rng = np.random.default_rng(0)
    for c_in, c_out in ((2816, 67), (2816, 707), (8224, 19)):
        W = rng.integers(0, 256, c_out * c_in // 2, dtype=np.uint8)
        S = (rng.integers(1, 20, c_out * c_in // 32) * 0.002).astype(np.float32)
        x = rng.standard_normal(c_in).astype(np.float32) * 0.02
        a = O.q4_matmul(W, S, x, c_in, c_out, prec=O.F32)
        b = O.q4_matmul(W, S, x, c_in, c_out, prec=O.F64)
        assert np.max(np.abs(a - b)) <= 1e-4


def _host_layer(d, F, E, K, seed):
    rng = np.random.default_rng(seed)
    w = dict(d=d, F=F, E=E, top_k=K)
    w["router_f32"] = rng.normal(0, 0.02, (E, d)).astype(np.float32)
    w["router_p"], w["router_s"], _ = O.quantize_q4_0(w["router_f32"])
    w["gu_p"], w["gu_s"], _ = O.quantize_q4_0(rng.normal(0, 0.02, E * 2 * F * d).astype(np.float32))
    w["dn_p"], w["dn_s"], _ = O.quantize_q4_0(rng.normal(0, 0.02, E * d * F).astype(np.float32))
    for k in ("router_scale", "pre_norm_w", "post_norm_w"):
        w[k] = np.ones(d, np.float32)
    w["per_expert_scale"] = np.ones(E, np.float32)
    return w


def test_coalesced_vs_per_token_and_f64():
    # test_spec_verify_and_coalesce.mojo:96-202: coalesced == per-token within 1e-6
    w = _host_layer(256, 64, 16, 6, seed=1)
    L = O.make_layer(w)
    x = np.random.default_rng(2).standard_normal((5, 256)).astype(np.float32)
    r = O.route(L, x)
    co = O.experts_forward(L, r["moe_in"], r["count"], r["idx"], r["w"], prec=O.F32)
    for t in range(5):
        n = r["count"][t]
        _, a = O.experts_stage1(w["gu_p"], w["gu_s"], r["moe_in"][t], r["idx"][t, :n], 256, 64, prec=O.F32)
        pt = O.experts_stage2(w["dn_p"], w["dn_s"], a, r["idx"][t, :n], r["w"][t, :n], 256, 64, prec=O.F32)
        assert np.max(np.abs(pt - co[t])) <= 1e-6
    f64 = O.experts_forward(L, r["moe_in"], r["count"], r["idx"], r["w"], prec=O.F64)
    assert np.max(np.abs(f64 - co)) <= 1e-5


def test_diffusion_f32_vs_f64():
    d, F, K, B = 256, 64, 8, 12
    w = _host_layer(d, F, 128, K, seed=4)
    rng = np.random.default_rng(3)
    x16 = rng.standard_normal((B, d)).astype(np.float16)
    ti = np.stack([rng.choice(128, K, replace=False) for _ in range(B)]).astype(np.int64)
    tw = rng.dirichlet(np.ones(K), B).astype(np.float32)
    tw[0, 3] = 0.0  # inactive slot
    a = O.diffusion_experts(w["gu_p"], w["gu_s"], w["dn_p"], w["dn_s"], x16, ti, tw, d, F, K, prec=O.F32)
    b = O.diffusion_experts(w["gu_p"], w["gu_s"], w["dn_p"], w["dn_s"], x16, ti, tw, d, F, K, prec=O.F64)
    # test_diffusion_kfd_q4.mojo:328-450 allows 5e-3 for fp16 I/O
    assert np.max(np.abs(a.astype(np.float32) - b.astype(np.float32))) <= 5e-3


def test_layer_forward_post_norm_and_routing_consistency():
    w = _host_layer(256, 64, 16, 4, seed=6)
    L = O.make_layer(w)
    x = np.random.default_rng(7).standard_normal((3, 256)).astype(np.float32)
    out, cnt, idx, ww = O.layer_forward(L, x, post_norm=True, prec=O.F64)
    r = O.route(L, x)
    assert np.array_equal(cnt, r["count"]) and np.array_equal(idx, r["idx"])
    raw, _, _, _ = O.layer_forward(L, x, post_norm=False, prec=O.F64)
    raw = raw.astype(np.float64)
    exp = raw / np.sqrt((raw ** 2).mean(1, keepdims=True) + 1e-6)
    np.testing.assert_allclose(out, exp, rtol=1e-5, atol=1e-6)


# ------------------------------------------- diffusion router-subspace bypass
def _oracle_filter(r_curr, r_prev, top_idx, prev_top2, eb, act, keep, B, E, K, step, tau, top_w=None):
    k, n = O.router_subspace_ffn_filter(r_curr, r_prev, top_idx, prev_top2, B, E, K, step, tau, eb, act,
                                        top_w)
    keep[:n] = k
    return n


def _oracle_scatter(sub, cache, full, act, keep, B, n, dim):
    O.scatter_and_restore_ffn_subspace(sub, cache, full, keep, B, n, act)


def test_subspace_bypass_known_answers():
    """test_diffusion_suite.mojo:562-648 on the oracle."""
    import subspace_cases
    subspace_cases.known_answers(_oracle_filter, _oracle_scatter)


def test_subspace_filter_zeroes_bypassed_weights_and_keeps_reference_points():
    import subspace_cases
    c = subspace_cases.random_filter_case(3)
    r_prev0, pt0 = c["r_prev"].copy(), c["prev_top2"].copy()
    tw = c["top_w"].copy()
    keep, n = O.router_subspace_ffn_filter(c["r_curr"], c["r_prev"], c["top_idx"], c["prev_top2"], c["B"],
                                           c["E"], c["K"], 1, c["tau"], c["eb"], c["act"], tw)
    assert 0 < n < c["B"]  # the case sits on the boundary: both outcomes occur
    kept = np.zeros(c["B"], bool)
    kept[keep] = True
    assert np.all(np.diff(keep) > 0)
    assert np.all(tw[~kept] == 0) and np.array_equal(tw[kept], c["top_w"][kept])
    o = c["act"]
    assert np.array_equal(c["r_prev"][o[kept]], c["r_curr"][kept])
    assert np.array_equal(c["r_prev"][o[~kept]], r_prev0[o[~kept]])
    assert np.array_equal(c["prev_top2"][o[kept]], c["top_idx"][kept, :2])
    assert np.array_equal(c["prev_top2"][o[~kept]], pt0[o[~kept]])
    # step 0 evaluates everything
    keep0, n0 = O.router_subspace_ffn_filter(c["r_curr"], r_prev0.copy(), c["top_idx"], pt0.copy(), c["B"],
                                             c["E"], c["K"], 0, c["tau"], c["eb"], c["act"])
    assert n0 == c["B"] and np.array_equal(keep0, np.arange(c["B"]))


def test_subspace_sync_walk_stops_at_a_break_in_the_keep_list():
    import subspace_cases
    c = subspace_cases.random_rows_case(1, 40, 64, 16, np.float32)
    out, cache = c["out"].copy(), c["cache"].copy()
    O.sync_moe_subspace_cache(out, cache, c["keep"], 40, len(c["keep"]), c["act"])
    # emulate the walk in Python
    out2, cache2 = c["out"].copy(), c["cache"].copy()
    cur = 0
    for b in range(40):
        o = c["act"][b]
        if cur < len(c["keep"]) and c["keep"][cur] == b:
            cache2[o] = out2[b]
            cur += 1
        else:
            out2[b] = cache2[o]
    assert cur < len(c["keep"])  # the break was hit
    assert np.array_equal(out, out2) and np.array_equal(cache, cache2)
