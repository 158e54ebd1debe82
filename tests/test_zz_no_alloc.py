"""moe_q4_matmul_batchN_noalloc against moe_q4_matmul_batchN.

The no-allocation variant keeps its scratch in a fixed static device array
instead of the context workspace.  Both entry points are called through the
C ABI on the same device buffers; the variant must agree with the workspace
entry point within the parity tolerance on two calls in a row, reject sizes
beyond its scratch with MOE_E_SHAPE, refuse host buffers it would have to
stage, and leave the device's free memory unchanged.

This file is collected last (test_zz_*) so that it also runs after every
other GPU test in the same process; it creates its own context, so it passes
alone as well.
"""
import ctypes as C

import numpy as np
import pytest

from tolerances import assert_close

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 8 << 20


@pytest.fixture(scope="module")
def nctx():
    import moe_b200
    c = moe_b200.Context(0)
    yield c
    c.close()


def _q4_matrix(ctx, c_out, c_in, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn(c_out * c_in, device="cuda", generator=g) * 0.02
    packed = torch.empty(c_out * c_in // 2, dtype=torch.uint8, device="cuda")
    scales = torch.empty(c_out * c_in // 32, dtype=torch.float32, device="cuda")
    ctx.quantize_fp32_to_q4_0(w, packed, scales, c_out * c_in)
    return packed, scales


def _call_noalloc(ctx, batch, packed, scales, x, out, c_in, c_out):
    return ctx.lib.moe_q4_matmul_batchN_noalloc(ctx.h, batch, C.c_void_p(packed.data_ptr()),
                                                C.c_void_p(scales.data_ptr()), C.c_void_p(x.data_ptr()),
                                                C.c_void_p(out.data_ptr()), c_in, c_out)


@pytest.mark.parametrize("batch,c_in,c_out", [(1, 2816, 2816), (16, 2816, 2816), (16, 704, 2816),
                                              (200, 2816, 1408)])
def test_noalloc_matches_workspace_entry_point(nctx, batch, c_in, c_out):
    import torch
    packed, scales = _q4_matrix(nctx, c_out, c_in, seed=batch + c_in)
    g = torch.Generator(device="cuda").manual_seed(7 + batch)
    x = torch.randn(batch, c_in, device="cuda", generator=g)
    ref = torch.empty(batch, c_out, device="cuda")
    assert nctx.lib.moe_q4_matmul_batchN(nctx.h, batch, C.c_void_p(packed.data_ptr()),
                                         C.c_void_p(scales.data_ptr()), C.c_void_p(x.data_ptr()),
                                         C.c_void_p(ref.data_ptr()), c_in, c_out) == 0, nctx.last_error()
    torch.cuda.synchronize()
    ref_h = ref.cpu().numpy()
    for call in range(2):
        out = torch.full((batch, c_out), float("nan"), device="cuda")
        rc = _call_noalloc(nctx, batch, packed, scales, x, out, c_in, c_out)
        assert rc == 0, nctx.last_error()
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        assert_close(got, ref_h, what=f"call {call} batch={batch} c_in={c_in} c_out={c_out}")


def test_noalloc_vs_oracle(nctx):
    """The variant against the CPU oracle itself, not only against the
    workspace entry point (a fault both share would pass that comparison)."""
    import torch
    import oracle as O
    batch, c_in, c_out = 16, 2816, 1024
    rng = np.random.default_rng(21)
    w = rng.normal(0, 0.02, c_out * c_in).astype(np.float32)
    W, S, _ = O.quantize_q4_0(w)
    x = rng.standard_normal((batch, c_in)).astype(np.float32)
    Wd, Sd, xd = torch.from_numpy(W).cuda(), torch.from_numpy(S).cuda(), torch.from_numpy(x).cuda()
    ref = O.q4_matmul(W, S, x, c_in, c_out, prec=O.F64)
    for call in range(2):
        out = torch.full((batch, c_out), float("nan"), device="cuda")
        assert _call_noalloc(nctx, batch, Wd, Sd, xd, out, c_in, c_out) == 0, nctx.last_error()
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), ref, what=f"call {call} vs oracle")


def test_noalloc_honours_the_dense_ksplit_option(nctx):
    """With MOE_OPT_DENSE_KSPLIT set, both entry points split K the same way
    and give the same bits."""
    import torch
    import moe_b200 as MB
    batch, c_in, c_out = 8, 2816, 2816
    packed, scales = _q4_matrix(nctx, c_out, c_in, seed=31)
    x = torch.randn(batch, c_in, device="cuda")
    ref = torch.empty(batch, c_out, device="cuda")
    out = torch.empty(batch, c_out, device="cuda")
    nctx.set_option(MB.OPT_DENSE_KSPLIT, 3)
    try:
        assert nctx.lib.moe_q4_matmul_batchN(nctx.h, batch, C.c_void_p(packed.data_ptr()),
                                             C.c_void_p(scales.data_ptr()), C.c_void_p(x.data_ptr()),
                                             C.c_void_p(ref.data_ptr()), c_in, c_out) == 0, nctx.last_error()
        assert _call_noalloc(nctx, batch, packed, scales, x, out, c_in, c_out) == 0, nctx.last_error()
        torch.cuda.synchronize()
    finally:
        nctx.set_option(MB.OPT_DENSE_KSPLIT, 0)
    assert torch.equal(out, ref)


_FRESH = r"""
import ctypes as C, sys, torch
sys.path[:0] = [{pkg!r}]
import moe_b200
torch.cuda.init()
c_in, c_out, batch = 2816, 2816, 16
w = torch.randn(c_out * c_in, device="cuda") * 0.02
packed = torch.empty(c_out * c_in // 2, dtype=torch.uint8, device="cuda")
scales = torch.empty(c_out * c_in // 32, dtype=torch.float32, device="cuda")
x = torch.randn(batch, c_in, device="cuda")
out = torch.empty(batch, c_out, device="cuda")
ctx = moe_b200.Context(0)
ctx.quantize_fp32_to_q4_0(w, packed, scales, c_out * c_in)
args = (ctx.h, batch, C.c_void_p(packed.data_ptr()), C.c_void_p(scales.data_ptr()),
        C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()), c_in, c_out)
# the workspace entry point first: it loads the kernels both entry points
# launch and grows the context's workspace; neither is what is measured
assert ctx.lib.moe_q4_matmul_batchN(*args) == 0, ctx.last_error()
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
for _ in range(2):
    assert ctx.lib.moe_q4_matmul_batchN_noalloc(*args) == 0, ctx.last_error()
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
print("FREE", free0, free1)
ctx.close()
"""


def test_first_noalloc_call_in_a_fresh_process_allocates_nothing():
    """In a new process the first no-alloc call must not load the static
    scratch (8 MiB) either: creating the context commits it."""
    import os
    import subprocess
    import sys
    pkg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "llm-mojo_b200")
    r = subprocess.run([sys.executable, "-c", _FRESH.format(pkg=pkg)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("FREE")][0]
    free0, free1 = (int(v) for v in line.split()[1:])
    assert free1 == free0, f"free device memory fell by {free0 - free1} bytes during the first no-alloc calls"


def test_noalloc_allocates_nothing(nctx):
    import torch
    batch, c_in, c_out = 32, 2816, 2816
    packed, scales = _q4_matrix(nctx, c_out, c_in, seed=11)
    x = torch.randn(batch, c_in, device="cuda")
    out = torch.empty(batch, c_out, device="cuda")
    assert _call_noalloc(nctx, batch, packed, scales, x, out, c_in, c_out) == 0, nctx.last_error()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(2):
        assert _call_noalloc(nctx, batch, packed, scales, x, out, c_in, c_out) == 0, nctx.last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_noalloc_rejects_sizes_beyond_its_scratch(nctx):
    import torch
    c_in, c_out = 2816, 256
    batch = SCRATCH_BYTES // (2 * c_in) + 1  # one token more than the fp16 copy can hold
    packed, scales = _q4_matrix(nctx, c_out, c_in, seed=5)
    x = torch.zeros(batch, c_in, device="cuda")
    out = torch.empty(batch, c_out, device="cuda")
    rc = _call_noalloc(nctx, batch, packed, scales, x, out, c_in, c_out)
    assert rc == 2  # MOE_E_SHAPE
    assert "8 MiB" in nctx.last_error()
    # the largest batch that fits still runs
    ok = batch - 1
    assert _call_noalloc(nctx, ok, packed, scales, x[:ok], out[:ok], c_in, c_out) == 0, nctx.last_error()


def test_noalloc_refuses_host_buffers(nctx):
    c_in, c_out, batch = 256, 128, 2
    packed, scales = _q4_matrix(nctx, c_out, c_in, seed=9)
    x = np.zeros((batch, c_in), np.float32)
    out = np.zeros((batch, c_out), np.float32)
    rc = nctx.lib.moe_q4_matmul_batchN_noalloc(nctx.h, batch, C.c_void_p(packed.data_ptr()),
                                               C.c_void_p(scales.data_ptr()), C.c_void_p(x.ctypes.data),
                                               C.c_void_p(out.ctypes.data), c_in, c_out)
    assert rc == 1  # MOE_E_ARG
    assert "does not stage host buffers" in nctx.last_error()
