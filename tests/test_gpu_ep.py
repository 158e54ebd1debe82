"""Expert parallelism on the GPU: the expert-range option of the library, the
rms_norm entry point, and the two multi-rank forms over NCCL (all-reduce of
partial outputs; all-to-all dispatch of routed rows), on one rank always and
on two GPUs where the box has them."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import moe_b200 as MB
import synth
from tolerances import assert_close

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_rms_norm_matches_formula(ctx):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((7, 2816)).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(2816)).astype(np.float32)
    out = np.zeros_like(x)
    ctx.rms_norm(x, w, out, 7, 2816)
    x64 = x.astype(np.float64)
    ref = x64 / np.sqrt((x64 ** 2).mean(1, keepdims=True) + 1e-6) * w
    np.testing.assert_allclose(out, ref, rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("M", [1, 16, 64])
def test_expert_ranges_sum_to_the_full_layer(ctx, full_layer, M):
    import torch
    dev, host, L = full_layer
    desc = MB.make_desc(dev)
    x = synth.make_x(M, seed=90 + M)
    full = torch.zeros((M, 2816), device="cuda")
    ctx.layer_forward(desc, M, x, full, 0)
    acc = torch.zeros_like(full)
    for lo, hi in ((0, 40), (40, 41), (41, 128)):
        part = torch.zeros_like(full)
        ctx.set_expert_range(lo, hi)
        try:
            ctx.layer_forward(desc, M, x, part, 0)
        finally:
            ctx.set_expert_range(0, 0)
        acc += part
    torch.cuda.synchronize()
    # A launch over fewer experts hands the CTAs different work items, and the
    # tensor-core kernel splits an item's K stages between accumulators by the
    # CTA's running stage count, so the fp32 sums agree to rounding, not bit
    # for bit; a reordered gate/up sum can also move an activation across an
    # fp16 rounding boundary (one ulp, ~5e-4 relative) before the down
    # projection.  One expert's share of an output is ~5e-2: a missing or
    # doubled expert fails this bar by orders of magnitude.
    assert_close(acc.cpu().numpy(), full.cpu().numpy(), max_abs=1e-4, rel_l2=1e-4, what=f"ranges M={M}")
    # post-norm of the reduced sum = the layer's own post-norm
    w = (1.0 + 0.1 * torch.randn(2816, generator=torch.Generator().manual_seed(1))).cuda()
    d2 = dict(dev)
    d2["post_norm_w"] = w
    normed_ref = torch.zeros_like(full)
    ctx.layer_forward(MB.make_desc(d2), M, x, normed_ref, MB.F_POST_NORM)
    normed = torch.zeros_like(full)
    ctx.rms_norm(acc, w, normed, M, 2816)
    torch.cuda.synchronize()
    # normalised outputs are ~7x the layer's (rms 1), the rounding above with them
    assert_close(normed.cpu().numpy(), normed_ref.cpu().numpy(), max_abs=5e-4, rel_l2=1e-4, what="post-norm")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("nproc", [1, 2])
def test_expert_parallel_ranks(nproc):
    import torch
    if torch.cuda.device_count() < nproc:
        pytest.skip(f"needs {nproc} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "ep_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[:3000]


def test_native_ep_one_rank_equals_the_layer(ctx, full_layer):
    """moe_ep_init with a single rank: the layer call takes the expert-
    parallel path (local range = all experts, NCCL all-reduce, post-norm of
    the sum) and agrees with the plain call; after moe_ep_finalize the
    context is a plain one again."""
    import torch
    dev, _, _ = full_layer
    d2 = dict(dev)
    d2["post_norm_w"] = (1.0 + 0.1 * torch.randn(2816, generator=torch.Generator().manual_seed(7))).cuda()
    desc = MB.make_desc(d2)
    c2 = MB.Context(0)
    try:
        c2.ep_init(MB.ep_unique_id(), 0, 1)
        with pytest.raises(MB.MoeError) as e:
            c2.ep_init(MB.ep_unique_id(), 0, 1)
        assert e.value.code == 8  # MOE_E_STATE: one communicator per context
        for M in (1, 16, 64):
            x = synth.make_x(M, seed=120 + M)
            ref = torch.zeros((M, 2816), device="cuda")
            ctx.layer_forward(desc, M, x, ref, MB.F_POST_NORM)
            got = torch.zeros_like(ref)
            c2.layer_forward(desc, M, x, got, MB.F_POST_NORM)
            raw_ref = torch.zeros_like(ref)
            ctx.layer_forward(desc, M, x, raw_ref, 0)
            raw = torch.zeros_like(ref)
            c2.layer_forward(desc, M, x, raw, 0)
            torch.cuda.synchronize()
            # same experts, same order: the partial sum is the whole sum
            assert torch.equal(raw, raw_ref), f"M={M}"
            # post-norm by the norm kernel instead of inside the combine
            assert_close(got.cpu().numpy(), ref.cpu().numpy(), max_abs=1e-5, rel_l2=1e-6, what=f"ep1 M={M}")
        with pytest.raises(MB.MoeError) as e:
            x = synth.make_x(4, seed=1)
            c2.layer_forward(desc, 4, x, torch.zeros((4, 2816), device="cuda"), MB.F_FP16_OUT)
        assert e.value.code == 1
        c2.ep_finalize()
        x = synth.make_x(16, seed=3)
        a, b = torch.zeros((16, 2816), device="cuda"), torch.zeros((16, 2816), device="cuda")
        ctx.layer_forward(desc, 16, x, a, MB.F_POST_NORM)
        c2.layer_forward(desc, 16, x, b, MB.F_POST_NORM)
        torch.cuda.synchronize()
        assert torch.equal(a, b)
    finally:
        c2.close()


@pytest.mark.parametrize("mode", ["gather", "all_to_all"])
def test_native_ep_token_forms_one_rank(ctx, full_layer, mode):
    """The gather and all-to-all forms on a one-rank communicator (the
    exchange goes to the rank itself) against the plain layer call, the
    routing outputs bit-exact, outputs within fp32 reordering; the
    all-to-all form also with no token at all (M = 0), which must still
    take part in the exchange, and with the local-weights option (the
    descriptor's expert arrays are the rank's slice: here all experts)."""
    import torch
    dev, _, _ = full_layer
    d2 = dict(dev)
    d2["post_norm_w"] = (1.0 + 0.1 * torch.randn(2816, generator=torch.Generator().manual_seed(9))).cuda()
    desc = MB.make_desc(d2)
    c2 = MB.Context(0)
    try:
        c2.ep_init(MB.ep_unique_id(), 0, 1)
        c2.set_option(MB.OPT_EP_MODE, MB.EP_GATHER if mode == "gather" else MB.EP_ALL_TO_ALL)
        for local in (0, 1):
            c2.set_option(MB.OPT_EP_LOCAL_WEIGHTS, local)
            for M in (1, 16, 300):
                x = synth.make_x(M, seed=140 + M)
                ref = torch.zeros((M, 2816), device="cuda")
                rc, ri, rw = (torch.zeros(M, dtype=torch.int64, device="cuda"),
                              torch.zeros((M, 8), dtype=torch.int64, device="cuda"),
                              torch.zeros((M, 8), device="cuda"))
                ctx.layer_forward(desc, M, x, ref, MB.F_POST_NORM, rc, ri, rw)
                got = torch.zeros_like(ref)
                gc, gi, gw = torch.zeros_like(rc), torch.zeros_like(ri), torch.zeros_like(rw)
                c2.layer_forward(desc, M, x, got, MB.F_POST_NORM, gc, gi, gw)
                torch.cuda.synchronize()
                assert torch.equal(gc, rc) and torch.equal(gi, ri) and torch.equal(gw, rw), f"{mode} M={M}"
                bar = (5e-4, 1e-4)
                if mode == "all_to_all" and M == 1:
                    # the plain call takes the fp32 CUDA-core kernels for one
                    # token, the eight dispatched rows the fp16 tensor-core
                    # path: the north-star bar carried through the post-norm
                    raw = torch.zeros_like(ref)
                    ctx.layer_forward(desc, M, x, raw, 0)
                    inv_rms = float((1.0 / torch.sqrt(raw.double().pow(2).mean(1) + 1e-6)).max())
                    bar = (2e-3 * inv_rms, 1e-3)
                assert_close(got.cpu().numpy(), ref.cpu().numpy(), max_abs=bar[0], rel_l2=bar[1],
                             what=f"ep1 {mode} M={M} local={local}")
        if mode == "all_to_all":
            c2.layer_forward(desc, 0, None, None, MB.F_POST_NORM)
    finally:
        c2.close()


_MISSING_RANK = r"""
import sys
sys.path[:0] = sys.argv[1:]
import numpy as np
import moe_b200 as MB
c = MB.Context(0)
c.set_option(MB.OPT_EP_TIMEOUT_NS, 2_000_000_000)
try:
    c.ep_init(MB.ep_unique_id(), 0, 2)   # rank 1 never joins
    print("joined?")
    sys.exit(1)
except MB.MoeError as e:
    assert e.code == 6, e                # MOE_E_TIMEOUT, communicator aborted
x = np.ones((2, 64), np.float32)
out = np.zeros_like(x)
c.rms_norm(x, np.ones(64, np.float32), out, 2, 64)   # the context still works
assert np.allclose(out, 1.0, atol=1e-5)
c.close()
print("OK")
"""


def test_native_ep_missing_rank_times_out():
    """A rank that never joins: moe_ep_init gives up after the communicator
    deadline with MOE_E_TIMEOUT and the context stays usable.  Host-side
    failure only (the bootstrap waits on sockets); run in a child process so
    that nothing here can outlive its time limit."""
    root = os.path.dirname(HERE)
    paths = [os.path.join(root, "llm-mojo_b200"), HERE]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "10", "90", sys.executable, "-c", _MISSING_RANK, *paths],
                       env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
