"""The diffusion router-subspace FFN bypass on the GPU, through the C ABI:
router_subspace_ffn_filter, sync_moe_subspace_cache and
scatter_and_restore_ffn_subspace (diffusion_kernels.mojo:2253-2426).

Everything here is decisions and copies, so the bar is bit-exact against
the oracle: the kept-row list and count, the updated reference logits and
top-2 ids, the zeroed routing weights and every copied row.  The reference's
own known answers run first (tests/subspace_cases.py)."""
import numpy as np
import pytest

import oracle as O
import subspace_cases
from tolerances import assert_close

pytestmark = pytest.mark.gpu


def _gpu_filter(ctx):
    def f(r_curr, r_prev, top_idx, prev_top2, eb, act, keep, B, E, K, step, tau, top_w=None):
        return ctx.router_subspace_ffn_filter(r_curr, r_prev, top_idx, prev_top2, eb, act, keep, B, E, K, step,
                                              tau, top_w)
    return f


def _gpu_scatter(ctx):
    def f(sub, cache, full, act, keep, B, n, dim):
        ctx.scatter_and_restore_ffn_subspace(sub, cache, full, act, keep, B, n, dim, elem_bytes=2)
    return f


def test_subspace_known_answers_gpu(ctx):
    subspace_cases.known_answers(_gpu_filter(ctx), _gpu_scatter(ctx))


@pytest.mark.parametrize("seed,step", [(1, 1), (2, 3), (5, 0)])
@pytest.mark.parametrize("device_arrays", [False, True])
def test_subspace_filter_bit_exact_vs_oracle(ctx, seed, step, device_arrays):
    import torch
    c = subspace_cases.random_filter_case(seed)
    B, E, K = c["B"], c["E"], c["K"]
    # oracle
    o_rp, o_pt, o_tw = c["r_prev"].copy(), c["prev_top2"].copy(), c["top_w"].copy()
    o_keep, o_n = O.router_subspace_ffn_filter(c["r_curr"], o_rp, c["top_idx"], o_pt, B, E, K, step, c["tau"],
                                               c["eb"], c["act"], o_tw)
    if step >= 1:
        assert 0 < o_n < B  # both decisions occur on this case
    # library
    arrs = dict(r_curr=c["r_curr"], r_prev=c["r_prev"].copy(), top_idx=c["top_idx"],
                prev_top2=c["prev_top2"].copy(), eb=c["eb"], act=c["act"], top_w=c["top_w"].copy(),
                keep=np.full(B, -7, np.int64))
    if device_arrays:
        arrs = {k: torch.from_numpy(v).cuda() for k, v in arrs.items()}
    n = ctx.router_subspace_ffn_filter(arrs["r_curr"], arrs["r_prev"], arrs["top_idx"], arrs["prev_top2"],
                                       arrs["eb"], arrs["act"], arrs["keep"], B, E, K, step, c["tau"],
                                       arrs["top_w"])
    host = {k: (v.cpu().numpy() if hasattr(v, "cpu") else v) for k, v in arrs.items()}
    assert n == o_n
    assert np.array_equal(host["keep"][:n], o_keep)
    assert np.array_equal(host["r_prev"].view(np.uint32), o_rp.view(np.uint32))
    assert np.array_equal(host["prev_top2"], o_pt)
    assert np.array_equal(host["top_w"].view(np.uint32), o_tw.view(np.uint32))


def test_subspace_filter_without_mask_index_or_weights(ctx):
    """NULL eb_mask, active_canvas_idx and top_weights (all accepted, row b at
    canvas position b), and B larger than one pass of the kernel."""
    c = subspace_cases.random_filter_case(7, B=300, canvas=300)
    c["act"] = np.arange(300, dtype=np.int64)
    c["prev_top2"][:] = c["top_idx"][:, :2]
    o_rp, o_pt = c["r_prev"].copy(), c["prev_top2"].copy()
    o_keep, o_n = O.router_subspace_ffn_filter(c["r_curr"], o_rp, c["top_idx"], o_pt, 300, c["E"], c["K"], 1,
                                               c["tau"])
    rp, pt, keep = c["r_prev"].copy(), c["prev_top2"].copy(), np.zeros(300, np.int64)
    n = ctx.router_subspace_ffn_filter(c["r_curr"], rp, c["top_idx"], pt, None, None, keep, 300, c["E"], c["K"], 1,
                                       c["tau"], None)
    assert n == o_n and np.array_equal(keep[:n], o_keep)
    assert np.array_equal(rp, o_rp) and np.array_equal(pt, o_pt)


@pytest.mark.parametrize("seed,B,canvas,dim,dtype", [(1, 256, 512, 2816, np.float16), (2, 256, 512, 2816, np.float16),
                                                     (3, 37, 64, 2816, np.float32), (4, 19, 40, 37, np.float16),
                                                     (6, 5, 5, 8, np.float32)])
def test_subspace_rows_bit_exact_vs_oracle(ctx, seed, B, canvas, dim, dtype):
    """sync and scatter (16-byte, 4-byte and byte copies; keep lists with and
    without a break in their order) against the oracle."""
    import torch
    c = subspace_cases.random_rows_case(seed, B, canvas, dim, dtype)
    eb = np.dtype(dtype).itemsize
    n = len(c["keep"])
    # sync
    o_out, o_cache = c["out"].copy(), c["cache"].copy()
    O.sync_moe_subspace_cache(o_out, o_cache, c["keep"], B, n, c["act"])
    g_out = torch.from_numpy(c["out"].copy()).cuda()
    g_cache = torch.from_numpy(c["cache"].copy()).cuda()
    ctx.sync_moe_subspace_cache(g_out, g_cache, torch.from_numpy(c["act"]).cuda(), torch.from_numpy(c["keep"]).cuda(),
                                B, n, dim, elem_bytes=eb)
    assert np.array_equal(g_out.cpu().numpy(), o_out) and np.array_equal(g_cache.cpu().numpy(), o_cache)
    # scatter (host arrays: staged by the library)
    o_full, o_cache = np.zeros_like(c["out"]), c["cache"].copy()
    O.scatter_and_restore_ffn_subspace(c["sub"], o_cache, o_full, c["keep"], B, n, c["act"])
    full, cache = np.zeros_like(c["out"]), c["cache"].copy()
    ctx.scatter_and_restore_ffn_subspace(c["sub"], cache, full, c["act"], c["keep"], B, n, dim, elem_bytes=eb)
    assert np.array_equal(full, o_full) and np.array_equal(cache, o_cache)


def test_subspace_bypass_through_the_diffusion_layer(ctx, full_layer):
    """The reference's caller sequence (test_diffusion_suite.mojo:1316-1348):
    filter -> experts on the canvas with the bypassed rows' weights zeroed ->
    sync of the output cache.  Step 0 evaluates every row and fills the
    cache; step 1 with unchanged logits bypasses every accepted row, whose
    output then comes back from the cache: equal, bit for bit, to step 0's.
    The rows evaluated again (not accepted) agree with step 0 within the
    parity bar: the expert GEMMs split each row's K range over accumulators
    by the work list, which changes with the set of active rows."""
    import synth
    dev, host, L = full_layer
    B = 64
    x = synth.make_x(B, seed=77, bf16_representable=True).cpu().numpy()
    ref = O.route(L, x)
    scores = ref["scores"]
    top_idx = ref["top_idx"]
    w0 = O.apply_moe_lod_and_set_cover(top_idx, ref["top_val"], host["per_expert_scale"], B, 8, 8, 1.0)
    x16 = ref["moe_in"].astype(np.float16)
    act = np.arange(B, dtype=np.int64)
    eb = np.ones(B, np.uint8)
    eb[::5] = 0  # not accepted: always evaluated
    r_prev = np.zeros((B, 128), np.float32)
    prev_top2 = np.full((B, 2), -1, np.int64)
    cache = np.zeros((B, 2816), np.float16)
    outs = []
    for step in range(2):
        w = w0.copy()
        keep = np.zeros(B, np.int64)
        n = ctx.router_subspace_ffn_filter(scores, r_prev, top_idx, prev_top2, eb, act, keep, B, 128, 8, step,
                                           0.05, w)
        assert n == (B if step == 0 else int((eb == 0).sum()))
        out = np.zeros((B, 2816), np.float16)
        ctx.run_diffusion_moe_experts_parallel(dev["gu_p"], dev["gu_s"], dev["dn_p"], dev["dn_s"], x16, top_idx, w,
                                               out, B, 2816, 704, 8)
        ctx.sync_moe_subspace_cache(out, cache, act, keep, B, n, 2816, elem_bytes=2)
        outs.append(out)
    byp = eb == 1
    assert np.array_equal(outs[0][byp], outs[1][byp])
    assert_close(outs[1][~byp].astype(np.float32), outs[0][~byp].astype(np.float32), what="re-evaluated rows")
    assert np.abs(outs[0].astype(np.float32)).sum() > 0
