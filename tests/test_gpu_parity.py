"""GPU parity of libmoe_b200.so against the CPU oracle, through the C ABI.

Bars (tests/tolerances.py): MoE path output max-abs <= 2e-3 and rel-L2 <= 1e-3
vs the oracle; top-k expert ids exact except near ties (adjacent router
probabilities closer than 1e-6); quantizer and integer routing bit-exact.
"""
import json
import os

import numpy as np
import pytest

import moe_b200 as MB
import oracle as O
import synth
from tolerances import assert_close, errors, near_tie_tokens

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def torch():
    import torch as t
    return t


# ---------------------------------------------------------------- quantizer
def test_quantizer_bit_exact_vs_reference_golden(ctx):
    g = np.load(os.path.join(GOLD, "q4_golden.npz"))
    for n in sorted({k.split("__")[0] for k in g.files}):
        x = g[n + "__x"]
        p = np.zeros(x.size // 2, np.uint8)
        s = np.zeros(x.size // 32, np.float32)
        ctx.quantize_fp32_to_q4_0(x, p, s, x.size)
        assert np.array_equal(p, g[n + "__packed"]), n
        assert np.array_equal(s.view(np.uint32), g[n + "__scales"].view(np.uint32)), n


def test_quantizer_large_vs_oracle(ctx):
    x = np.random.default_rng(11).normal(0, 0.02, 1 << 20).astype(np.float32)
    p = np.zeros(x.size // 2, np.uint8)
    s = np.zeros(x.size // 32, np.float32)
    ctx.quantize_fp32_to_q4_0(x, p, s, x.size)
    op, os_, ties = O.quantize_q4_0(x)
    assert ties == 0
    assert np.array_equal(p, op) and np.array_equal(s, os_)


# ------------------------------------------------------------- dense Q4 GEMV
@pytest.fixture()
def gemv(ctx):
    """Pins the CUDA-core (fp32) path, whose bar is far inside the spec."""
    ctx.set_gemm_path(MB.PATH_GEMV)
    yield ctx
    ctx.set_gemm_path(MB.PATH_AUTO)


@pytest.mark.parametrize("c_in,c_out,batch", [(2816, 67, 1), (2816, 707, 1), (8224, 19, 1),
                                              (2816, 4096, 16), (4096, 2816, 16), (704, 2816, 3),
                                              (64, 64, 2), (2816, 1024, 5)])
def test_q4_matmul_vs_oracle(gemv, c_in, c_out, batch):
    ctx = gemv
    rng = np.random.default_rng(c_in + c_out + batch)
    w = rng.normal(0, 0.02, c_out * c_in).astype(np.float32)
    W, S, _ = O.quantize_q4_0(w)
    x = rng.standard_normal((batch, c_in)).astype(np.float32)
    t = torch()
    Wd, Sd = t.from_numpy(W).cuda(), t.from_numpy(S).cuda()
    out = np.zeros((batch, c_out), np.float32)
    if batch == 1:
        ctx.q4_matmul_vec(Wd, Sd, x, out, c_in, c_out)
    else:
        ctx.q4_matmul_batchN(batch, Wd, Sd, x, out, c_in, c_out)
    ref = O.q4_matmul(W, S, x, c_in, c_out, prec=O.F64)
    mx, rel = assert_close(out, ref, what=f"q4_matmul {c_in}x{c_out}x{batch}")
    assert rel <= 1e-5  # fp32 path: far inside the bar


# -------------------------------------------------------------- expert stages
def _pattern(n_exp, d, F):
    rows = 2 * F
    gp = ((np.arange(n_exp * rows * d // 2) * 13 + 7) & 255).astype(np.uint8)
    gs = (((np.arange(n_exp * rows * d // 32) % 19) + 1) * 0.002).astype(np.float32)
    dp = ((np.arange(n_exp * d * F // 2) * 29 + 3) & 255).astype(np.uint8)
    ds = (((np.arange(n_exp * d * F // 32) % 17) + 1) * 0.002).astype(np.float32)
    x = (((np.arange(d) % 31) - 15) * 0.03).astype(np.float32)
    return gp, gs, dp, ds, x


@pytest.mark.parametrize("d,F,count", [(2816, 704, 5), (2816, 704, 8), (2816, 704, 1), (64, 32, 8)])
def test_stage1_stage2_pattern_vs_oracle(ctx, d, F, count):
    """test_moe_lod_top_p.mojo:51-197 data (byte/scale patterns), 8 experts."""
    t = torch()
    gp, gs, dp, ds, x = _pattern(8, d, F)
    dev = [t.from_numpy(a).cuda() for a in (gp, gs, dp, ds)]
    idx = np.arange(count, dtype=np.int64)[::-1].copy()
    w = np.linspace(0.3, 0.05, count).astype(np.float32)
    gu = np.zeros((count, 2 * F), np.float32)
    act = np.zeros((count, F), np.float32)
    ctx.run_moe_experts_stage1_8core(dev[0], dev[1], x, None, idx, count, gu, act, d, F)
    ogu, oact = O.experts_stage1(gp, gs, x, idx, d, F, prec=O.F64)
    assert_close(gu, ogu, what="gate_up_out")
    assert_close(act, oact, what="act")
    out = np.zeros(d, np.float32)
    ctx.run_moe_experts_stage2_8core(dev[2], dev[3], oact, None, idx, w, count, out, d, F)
    ref = O.experts_stage2(dp, ds, oact, idx, w, d, F, prec=O.F64)
    assert_close(out, ref, what="moe_out")


def test_stage_active_count_zero_zeroes_output(ctx):
    t = torch()
    gp, gs, dp, ds, x = _pattern(8, 64, 32)
    out = np.full(64, 7.0, np.float32)
    ctx.run_moe_experts_stage2_8core(t.from_numpy(dp).cuda(), t.from_numpy(ds).cuda(),
                                     np.zeros((1, 32), np.float32), None, np.zeros(1, np.int64),
                                     np.zeros(1, np.float32), 0, out, 64, 32)
    assert np.all(out == 0.0)


def test_gelu_tanh_activation(ctx):
    t = torch()
    gp, gs, dp, ds, x = _pattern(8, 2816, 704)
    idx = np.array([3, 1, 6], np.int64)
    act = np.zeros((3, 704), np.float32)
    ctx.run_moe_experts_stage1_8core(t.from_numpy(gp).cuda(), t.from_numpy(gs).cuda(), x, None, idx,
                                     3, None, act, 2816, 704, activation=MB.ACT_GELU_TANH)
    _, ref = O.experts_stage1(gp, gs, x, idx, 2816, 704, act=O.ACT_GELU_TANH, prec=O.F64)
    assert_close(act, ref, what="gelu_tanh act")


# ---------------------------------------------------------------- routing
def test_lod_batch_vs_oracle(ctx):
    rng = np.random.default_rng(4)
    B, K = 64, 8
    p = rng.dirichlet(np.ones(128) * 0.3, B).astype(np.float32)
    ti = np.argsort(-p, 1)[:, :K].astype(np.int64)
    tv = np.take_along_axis(p, ti, 1).astype(np.float32)
    pes = (0.5 + rng.random(128)).astype(np.float32)
    for top_p in (1.0, 0.8, float("nan")):
        ai = np.zeros((B, K), np.int64)
        aw = np.zeros((B, K), np.float32)
        cnt = ctx.compute_moe_lod_weights(ti, tv, pes, top_p, ai, aw, K, batch=B, active_count=np.zeros(B, np.int64))
        for b in range(B):
            n, oi, ow = O.compute_moe_lod_weights(ti[b], tv[b], pes, top_p)
            assert cnt[b] == n
            assert np.array_equal(ai[b, :n], oi[:n])
            np.testing.assert_allclose(aw[b, :n], ow[:n], rtol=1e-6, atol=0)


def test_lod_known_answer_gpu(ctx):
    with open(os.path.join(GOLD, "known_answers.json")) as f:
        ka = json.load(f)["lod"]
    ti = np.array(ka["top_idx"], np.int64)
    tv = np.array(ka["top_val"], np.float32)
    pes = np.ones(128, np.float32)
    ai, aw = np.zeros(8, np.int64), np.zeros(8, np.float32)
    assert ctx.compute_moe_lod_weights(ti, tv, pes, 1.0, ai, aw) == ka["expect_count_top_p_1"]
    n = ctx.compute_moe_lod_weights(ti, tv, pes, 0.8, ai, aw)
    assert n == ka["expect_count_top_p_080"] and abs(aw[:n].sum() - 1.0) <= ka["tol_weight_sum"]


def test_set_cover_known_answer_gpu(ctx):
    ti = np.zeros((5, 8), np.int64)
    tv = np.zeros((5, 8), np.float32)
    ti[0] = [10, 20, 30, 40, 50, 60, 70, 80]
    tv[0] = [0.28, 0.22, 0.16, 0.10, 0.07, 0.06, 0.06, 0.05]
    for b in range(1, 5):
        ti[b] = [10, 20, 30 + b, 40, 50, 60, 90 + 2 * b, 91 + 2 * b]
        tv[b] = [0.27, 0.23, 0.16, 0.12, 0.060, 0.055, 0.053, 0.052]
    pes = np.array([0.8 + 0.4 * ((e * 17) % 31) / 31.0 for e in range(128)], np.float32)
    cnt = np.zeros(5, np.int64)
    idx = np.zeros((5, 8), np.int64)
    w = np.zeros((5, 8), np.float32)
    ctx.compute_subbatch_set_cover_moe_weights(5, ti, tv, pes, 1.0, cnt, idx, w)
    oc, oi, ow = O.set_cover(ti, tv, pes, 1.0)
    assert np.array_equal(cnt, oc)
    for b in range(5):
        assert np.array_equal(idx[b, :cnt[b]], oi[b, :cnt[b]])
        np.testing.assert_allclose(w[b, :cnt[b]], ow[b, :cnt[b]], rtol=1e-6)
    assert all(c == 6 for c in cnt[1:])


def test_apply_lod_and_set_cover_gpu(ctx):
    rng = np.random.default_rng(9)
    B, K = 40, 8
    p = rng.dirichlet(np.ones(128) * 0.2, B).astype(np.float32)
    ti = np.argsort(-p, 1)[:, :K].astype(np.int64)
    tv = np.take_along_axis(p, ti, 1).astype(np.float32)
    pes = np.ones(128, np.float32)
    eb = (rng.random(B) > 0.5).astype(np.uint8)
    for kw in ({}, {"eb_mask": eb, "unaccepted_top_k": 2}):
        w = np.zeros((B, K), np.float32)
        ctx.apply_moe_lod_and_set_cover(ti, tv, pes, w, B, K, 8, 1.0, **kw)
        ref = O.apply_moe_lod_and_set_cover(ti, tv, pes, B, K, 8, 1.0, **kw)
        np.testing.assert_allclose(w, ref, rtol=1e-6, atol=0)


def _check_routing(cnt, idx, w, ref, probs, K):
    ties = set(near_tie_tokens(probs, K).tolist())
    bad = []
    for t in range(cnt.size):
        same = cnt[t] == ref["count"][t] and np.array_equal(idx[t, :cnt[t]], ref["idx"][t, :cnt[t]])
        if not same and t not in ties:
            bad.append(t)
        if same:
            np.testing.assert_allclose(w[t, :cnt[t]], ref["w"][t, :cnt[t]], rtol=2e-5, atol=1e-7)
    assert not bad, f"top-k mismatch outside near ties on tokens {bad}"
    return ties


def test_route_full_layer_vs_oracle(ctx, full_layer):
    dev, host, L = full_layer
    desc = MB.make_desc(dev)
    M = 64
    x = synth.make_x(M, seed=21).cpu().numpy()
    cnt = np.zeros(M, np.int64)
    idx = np.zeros((M, 8), np.int64)
    w = np.zeros((M, 8), np.float32)
    probs = np.zeros((M, 128), np.float32)
    moe_in = np.zeros((M, 2816), np.float32)
    ctx.route(desc, M, x, cnt, idx, w, scores=probs, moe_in=moe_in)
    ref = O.route(L, x)
    _check_routing(cnt, idx, w, ref, _softmax_rows(ref["scores"]), 8)
    np.testing.assert_allclose(moe_in, ref["moe_in"], rtol=1e-5, atol=1e-6)


def _softmax_rows(s):
    out = np.zeros_like(s)
    for i in range(s.shape[0]):
        out[i] = O.softmax(s[i])
    return out


# --------------------------------------------------------------- whole layer
@pytest.mark.parametrize("M", [1, 5, 16])
def test_layer_forward_full_vs_oracle(ctx, full_layer, M):
    dev, host, L = full_layer
    desc = MB.make_desc(dev)
    x = synth.make_x(M, seed=100 + M).cpu().numpy()
    out = np.zeros((M, 2816), np.float32)
    cnt = np.zeros(M, np.int64)
    idx = np.zeros((M, 8), np.int64)
    w = np.zeros((M, 8), np.float32)
    ctx.layer_forward(desc, M, x, out, flags=0, tok_active_count=cnt, tok_active_idx=idx,
                      tok_active_weights=w)
    ref = O.route(L, x)
    ties = _check_routing(cnt, idx, w, ref, _softmax_rows(ref["scores"]), 8)
    keep = np.array([t for t in range(M) if t not in ties])
    moe_ref = O.experts_forward(L, ref["moe_in"], ref["count"], ref["idx"], ref["w"], prec=O.F64)
    assert_close(out[keep], moe_ref[keep], what=f"layer M={M}")
    # post-norm variant: the bar carries through the norm's 1/rms
    outn = np.zeros((M, 2816), np.float32)
    ctx.layer_forward(desc, M, x, outn, flags=MB.F_POST_NORM)
    r64 = moe_ref.astype(np.float64)
    refn = r64 / np.sqrt((r64 ** 2).mean(1, keepdims=True) + 1e-6)
    scale = float(np.max(1.0 / np.sqrt((r64 ** 2).mean(1) + 1e-6)))
    assert_close(outn[keep], refn[keep], max_abs=2e-3 * scale, what=f"layer+post_norm M={M}")


def test_coalesced_core_deint_input(ctx, full_layer):
    """run_moe_coalesced_core with the reference's deinterleaved-halves input."""
    dev, host, L = full_layer
    x = synth.make_x(5, seed=7).cpu().numpy()
    ref = O.route(L, x)
    mi = ref["moe_in"]
    deint = np.concatenate([mi.reshape(5, -1, 16, 2)[..., 0].reshape(5, -1),
                            mi.reshape(5, -1, 16, 2)[..., 1].reshape(5, -1)], axis=1)
    out = np.zeros((5, 2816), np.float32)
    ctx.run_moe_coalesced_core(5, dev["gu_p"], dev["gu_s"], dev["dn_p"], dev["dn_s"],
                               np.ascontiguousarray(deint), ref["count"], ref["idx"], ref["w"], out)
    moe_ref = O.experts_forward(L, mi, ref["count"], ref["idx"], ref["w"], prec=O.F64)
    assert_close(out, moe_ref, what="coalesced core")


def test_diffusion_block_vs_oracle(ctx, full_layer):
    """run_diffusion_moe_experts_parallel, 256-token canvas, fp16 in/out."""
    dev, host, L = full_layer
    B = 256
    x = synth.make_x(B, seed=31, bf16_representable=True).cpu().numpy()
    ref = O.route(L, x)
    w = O.apply_moe_lod_and_set_cover(ref["top_idx"], ref["top_val"], host["per_expert_scale"], B,
                                      8, 8, 1.0)
    x16 = ref["moe_in"].astype(np.float16)
    out = np.zeros((B, 2816), np.float16)
    ctx.run_diffusion_moe_experts_parallel(dev["gu_p"], dev["gu_s"], dev["dn_p"], dev["dn_s"], x16,
                                           ref["top_idx"], w, out, B, 2816, 704, 8)
    o64 = O.diffusion_experts(host["gu_p"], host["gu_s"], host["dn_p"], host["dn_s"], x16,
                              ref["top_idx"], w, 2816, 704, 8, prec=O.F64)
    assert_close(out.astype(np.float32), o64.astype(np.float32), what="diffusion block")


def test_registered_host_blob_matches_device_weights(ctx):
    rng = np.random.default_rng(12)
    c_in, c_out = 2816, 256
    W, S, _ = O.quantize_q4_0(rng.normal(0, 0.02, c_in * c_out).astype(np.float32))
    blob = np.zeros(W.nbytes + S.nbytes + 4096, np.uint8)
    blob[:W.nbytes] = W
    blob[W.nbytes:W.nbytes + S.nbytes] = S.view(np.uint8)
    ctx.register_weights(blob)
    x = rng.standard_normal(c_in).astype(np.float32)
    out = np.zeros(c_out, np.float32)
    Wv = blob[:W.nbytes]
    Sv = blob[W.nbytes:W.nbytes + S.nbytes].view(np.float32)
    ctx.q4_matmul_vec(Wv, Sv, x, out, c_in, c_out)
    ref = O.q4_matmul(W, S, x, c_in, c_out, prec=O.F64)
    assert_close(out, ref)
    ctx.unregister_weights(blob)


def test_async_enqueue_and_bounded_wait(ctx, full_layer):
    dev, host, L = full_layer
    t = torch()
    desc = MB.make_desc(dev)
    x = synth.make_x(4, seed=5)
    out = t.zeros((4, 2816), device="cuda")
    ctx.set_async(True)
    try:
        ctx.layer_forward(desc, 4, x, out, flags=0)
        ctx.wait(timeout_ns=10_000_000_000)
    finally:
        ctx.set_async(False)
    ref = np.zeros((4, 2816), np.float32)
    ctx.layer_forward(desc, 4, x.cpu().numpy(), ref, flags=0)
    assert np.array_equal(out.cpu().numpy(), ref)


def test_device_wait_deadline_returns_timeout_and_context_recovers(ctx, full_layer):
    """The bounded device-side wait: moe_device_wait_check waits on a barrier
    that nothing completes with the wait code and deadline the pipelined
    expert kernels use (MOE_OPT_DEVICE_TIMEOUT_NS, here 2 ms).  It must give
    up, raise the error word and return MOE_E_TIMEOUT; then the same context
    gives oracle-correct layer output on both expert-kernel families (M=1:
    CUDA-core pair, M=16: tensor-core streaming kernels)."""
    import time
    dev, host, L = full_layer
    desc = MB.make_desc(dev)
    ctx.set_option(MB.OPT_DEVICE_TIMEOUT_NS, 2_000_000)
    try:
        t0 = time.perf_counter()
        with pytest.raises(MB.MoeError) as ei:
            ctx.device_wait_check()
        dt = time.perf_counter() - t0
        assert ei.value.code == 6, ei.value  # MOE_E_TIMEOUT
        assert "deadline" in str(ei.value)
        assert 0.002 <= dt < 2.0, dt
    finally:
        ctx.set_option(MB.OPT_DEVICE_TIMEOUT_NS, 4_000_000_000)
    for M in (1, 16):
        x = synth.make_x(M, seed=41 + M).cpu().numpy()
        out = np.zeros((M, 2816), np.float32)
        cnt = np.zeros(M, np.int64)
        idx = np.zeros((M, 8), np.int64)
        w = np.zeros((M, 8), np.float32)
        ctx.layer_forward(desc, M, x, out, 0, cnt, idx, w)
        r = O.route(L, x)
        ref = O.experts_forward(L, r["moe_in"], cnt, idx, w, prec=O.F64)
        assert_close(out, ref, what=f"after the timeout, M={M}")


# ------------------------------------------------------------- error paths
def test_unregistered_host_weights_are_rejected(ctx):
    W = np.zeros(64 * 32, np.uint8)
    S = np.ones(64 * 2, np.float32)
    with pytest.raises(MB.MoeError) as e:
        ctx.q4_matmul_vec(W, S, np.zeros(64, np.float32), np.zeros(64, np.float32), 64, 64)
    assert e.value.code == 3


def test_bad_shape_is_rejected(ctx):
    t = torch()
    W = t.zeros(64 * 32, dtype=t.uint8, device="cuda")
    S = t.ones(64 * 2, device="cuda")
    with pytest.raises(MB.MoeError) as e:
        ctx.q4_matmul_vec(W, S, np.zeros(33, np.float32), np.zeros(64, np.float32), 33, 64)
    assert e.value.code == 2


def test_out_of_range_expert_index_is_reported(ctx):
    t = torch()
    gp, gs, dp, ds, x = _pattern(8, 64, 32)
    act = np.zeros((2, 32), np.float32)
    with pytest.raises(MB.MoeError) as e:
        ctx.run_moe_experts_stage1_8core(t.from_numpy(gp).cuda(), t.from_numpy(gs).cuda(), x[:64],
                                         None, np.array([1, 5000], np.int64), 2, None, act, 64, 32)
    assert e.value.code == 1
    # the context stays usable
    ctx.run_moe_experts_stage1_8core(t.from_numpy(gp).cuda(), t.from_numpy(gs).cuda(), x[:64], None,
                                     np.array([1, 2], np.int64), 2, None, act, 64, 32)


def test_kernel_launch_counter_advances(ctx):
    n0 = ctx.kernel_launches
    x = np.ones(32 * 4, np.float32)
    ctx.quantize_fp32_to_q4_0(x, np.zeros(64, np.uint8), np.zeros(4, np.float32), x.size)
    assert ctx.kernel_launches == n0 + 1


@pytest.mark.parametrize("M", [1, 7, 16])
def test_fused_routing_matches_separate_kernels(ctx, full_layer, M):
    """The fused cluster launch (MOE_OPT_FUSED_ROUTE=1) and the separate
    routing kernels must give the same routing and, within fp32
    reassociation, the same output, also on an expert range."""
    dev, host, L = full_layer
    desc = MB.make_desc(dev)
    x = synth.make_x(M, seed=300 + M).cpu().numpy()
    res = []
    for fused in (1, 0):
        ctx.set_option(MB.OPT_FUSED_ROUTE, fused)
        try:
            for lo, hi in ((0, 0), (32, 96)):
                ctx.set_expert_range(lo, hi)
                out = np.zeros((M, 2816), np.float32)
                cnt = np.zeros(M, np.int64)
                idx = np.zeros((M, 8), np.int64)
                w = np.zeros((M, 8), np.float32)
                ctx.layer_forward(desc, M, x, out, MB.F_POST_NORM if hi == 0 else 0, cnt, idx, w)
                res.append((out, cnt, idx, w))
        finally:
            ctx.set_expert_range(0, 0)
            ctx.set_option(MB.OPT_FUSED_ROUTE, 0)
    r = O.route(L, x)
    ties = set(near_tie_tokens(np.stack([O.softmax(s) for s in r["scores"]]), 8).tolist())
    for a, b in ((res[0], res[2]), (res[1], res[3])):
        keep = [t for t in range(M) if t not in ties]
        assert np.array_equal(a[1][keep], b[1][keep])
        assert np.array_equal(a[2][keep], b[2][keep])
        np.testing.assert_allclose(a[3][keep], b[3][keep], rtol=1e-5, atol=1e-7)
        assert_close(a[0][keep], b[0][keep], max_abs=1e-4, rel_l2=1e-5, what=f"fused vs separate M={M}")


@pytest.mark.parametrize("M", [1, 5, 16, 33, 64])
def test_one_launch_routing_matches_separate_kernels(ctx, full_layer, M):
    """The routing in one launch (MOE_OPT_FUSED_ROUTE=2; its last CTA routes
    every token) reproduces the separate kernels' arithmetic: up to 16
    tokens (where the separate chain also takes the K-slice router) routing
    outputs equal, bit for bit, on the whole layer and on an expert range,
    outputs within fp32 reassociation (the pairs of an expert may land in
    other tile positions); at every size, routing and outputs against the
    oracle."""
    dev, host, L = full_layer
    desc = MB.make_desc(dev)
    x = synth.make_x(M, seed=320 + M).cpu().numpy()
    res = []
    for mode in (2, 0):
        ctx.set_option(MB.OPT_FUSED_ROUTE, mode)
        try:
            for lo, hi, fl in ((0, 0, MB.F_POST_NORM), (32, 96, 0), (0, 0, 0)):
                ctx.set_expert_range(lo, hi)
                out = np.zeros((M, 2816), np.float32)
                cnt = np.zeros(M, np.int64)
                idx = np.zeros((M, 8), np.int64)
                w = np.zeros((M, 8), np.float32)
                ctx.layer_forward(desc, M, x, out, fl, cnt, idx, w)
                res.append((out, cnt, idx, w))
        finally:
            ctx.set_expert_range(0, 0)
            ctx.set_option(MB.OPT_FUSED_ROUTE, 0)
    if M <= 16:
        for a, b in zip(res[:3], res[3:]):
            assert np.array_equal(a[1], b[1]) and np.array_equal(a[2], b[2])
            assert np.array_equal(a[3].view(np.uint32), b[3].view(np.uint32))
            assert_close(a[0], b[0], max_abs=1e-4, rel_l2=1e-5, what=f"one-launch vs separate M={M}")
    r = O.route(L, x)
    ties = _check_routing(res[2][1], res[2][2], res[2][3], r, _softmax_rows(r["scores"]), 8)
    keep = np.array([t for t in range(M) if t not in ties])
    moe_ref = O.experts_forward(L, r["moe_in"], r["count"], r["idx"], r["w"], prec=O.F64)
    assert_close(res[2][0][keep], moe_ref[keep], what=f"one-launch routing layer M={M}")


def test_one_token_gemv_equals_ring_gemv_and_oracle(ctx, full_layer):
    """One-token batches take the one-warp-per-row GEMV (MOE_OPT_GEMV_ONE_TOKEN,
    default on); it repeats the ring GEMV's arithmetic, so the outputs are the
    same bits, and both meet the oracle.  Also through the expert-stage entry
    points (one token, eight slots) and with gate/up values returned."""
    dev, host, L = full_layer
    desc = MB.make_desc(dev)
    outs = []
    for one in (1, 0):
        ctx.set_option(MB.OPT_GEMV_ONE_TOKEN, one)
        try:
            res = []
            for seed in (61, 62, 63):
                x = synth.make_x(1, seed=seed).cpu().numpy()
                out = np.zeros((1, 2816), np.float32)
                cnt = np.zeros(1, np.int64)
                idx = np.zeros((1, 8), np.int64)
                w = np.zeros((1, 8), np.float32)
                ctx.layer_forward(desc, 1, x, out, 0, cnt, idx, w)
                res.append((x, out, cnt, idx, w))
            outs.append(res)
        finally:
            ctx.set_option(MB.OPT_GEMV_ONE_TOKEN, 1)
    for a, b in zip(*outs):
        assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))
    for x, out, cnt, idx, w in outs[0]:
        r = O.route(L, x)
        ref = O.experts_forward(L, r["moe_in"], cnt, idx, w, prec=O.F64)
        mx, rel = assert_close(out, ref, what="one-token GEMV layer")
        assert rel <= 1e-5  # fp32 path
    # stage entry points: one token, eight experts, raw gate/up values too
    t = torch()
    gp, gs, dp, ds, x = _pattern(8, 2816, 704)
    devp = [t.from_numpy(v).cuda() for v in (gp, gs)]
    idx = np.array([7, 2, 5, 0, 1, 6, 3, 4], np.int64)
    ctx.set_gemm_path(MB.PATH_GEMV)
    try:
        gu = np.zeros((8, 1408), np.float32)
        act = np.zeros((8, 704), np.float32)
        ctx.run_moe_experts_stage1_8core(devp[0], devp[1], x, None, idx, 8, gu, act, 2816, 704)
    finally:
        ctx.set_gemm_path(MB.PATH_AUTO)
    ogu, oact = O.experts_stage1(gp, gs, x, idx, 2816, 704, prec=O.F64)
    assert_close(gu, ogu, what="stage1 gate_up (one token)")
    assert_close(act, oact, what="stage1 act (one token)")


@pytest.mark.parametrize("M", [1, 3, 16])
def test_gemv_path_layer_vs_oracle(ctx, full_layer, M):
    """CUDA-core expert GEMV (MOE_PATH_GEMV): fp32 arithmetic, checked against
    the fp64 oracle on the full layer, with one and several tokens per expert."""
    dev, host, L = full_layer
    desc = MB.make_desc(dev)
    x = synth.make_x(M, seed=700 + M).cpu().numpy()
    out = np.zeros((M, 2816), np.float32)
    cnt = np.zeros(M, np.int64)
    idx = np.zeros((M, 8), np.int64)
    w = np.zeros((M, 8), np.float32)
    ctx.set_gemm_path(MB.PATH_GEMV)
    try:
        ctx.layer_forward(desc, M, x, out, 0, cnt, idx, w)
    finally:
        ctx.set_gemm_path(MB.PATH_AUTO)
    r = O.route(L, x)
    ref = O.experts_forward(L, r["moe_in"], cnt, idx, w, prec=O.F64)
    assert_close(out, ref, max_abs=2e-4, rel_l2=1e-5, what=f"gemv layer M={M}")
