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
