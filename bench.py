#!/usr/bin/env python
"""Benchmark of the Q4_0 MoE-FFN path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload decode16]
    python bench.py --impl reference ...      # the reference's CPU algorithm

Workloads (seeded synthetic data; expert/router weights N(0, 0.02) -> Q4_0,
activations N(0, 1); norm weights, router_scale and per_expert_scale = 1):
  decode16  (default) continuous-batch decode, M=16 independent tokens through
            one 128-expert top-8 MoE layer (d=2816, F=704) with router, LOD,
            post-norm, plus the dense Q4_0 projections q [2816->4096],
            k, v [2816->1024], o [4096->2816] on the same 16 tokens.
  decode1   M=1 decode through the MoE layer.
  block256  one 256-token diffusion block through the MoE layer.
A step is one pass of the path over one batch.  Weights of `--layers`
distinct layers are cycled step by step so every step streams its experts
from HBM (4 layers x 476 MB >> 126 MB L2).

Multi-GPU: one process per GPU (torchrun); every rank runs its own batch
against its own replica of the layers (data-parallel replicas, no
collective on the data path); `value` is the whole-job token rate and
timing is the max over ranks of CUDA-event time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "llm-mojo_b200"))
sys.path.insert(1, os.path.join(ROOT, "oracle"))  # CPU baseline leg only

D, F, E, K = 2816, 704, 128, 8
GU_BYTES = 2 * F * D // 2 + 2 * F * D // 32 * 4   # 2,478,080 per expert
DN_BYTES = D * F // 2 + D * F // 32 * 4           # 1,239,040 per expert
ROUTER_BYTES = E * D // 2 + E * D // 32 * 4       # 225,280
DENSE = [("q", D, 4096), ("k", D, 1024), ("v", D, 1024), ("o", 4096, D)]
# tokens per step, distinct layers cycled (default), skewed routing, step count (default)
WORKLOADS = {
    "decode16": dict(M=16, layers=4),
    "decode1": dict(M=1, layers=4),
    "block256": dict(M=256, layers=4),
    "decode64": dict(M=64, layers=30),
    "prefill8k": dict(M=8192, layers=2, skew=True, steps=50),
}
WORKLOAD_NAMES = {
    "decode16": "cfg2: M=16 decode MoE layer + dense q/k/v/o",
    "decode1": "cfg1: M=1 decode MoE layer",
    "block256": "cfg3: M=256 block through the MoE layer",
    "decode64": "cfg4: M=64 decode, one layer step of a 30-layer stack (independent seeded layers)",
    "prefill8k": "cfg5: M=8192 (4 x 2048) through the MoE layer, Zipf(1.1)-skewed router",
}
METRIC = "moe_layer_tokens_per_s"


def q4_bytes(c_in, c_out):
    return c_out * c_in // 2 + c_out * c_in // 32 * 4


def peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, bf16 TFLOP/s sustained, source)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return (float(j["hbm_gbs"]), float(j["bf16_tflops"]),
                float(j.get("bf16_tflops_sustained", j["bf16_tflops"])), "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


def calibrate_skew(ctx, MB, synth, layer, x, M, target=5.0):
    """Zipf(1.1) router-logit bias scaled so that the busiest expert takes
    `target` x the mean load (active slots after the LOD prune); bisection
    on the scale alpha with the library's own router."""
    import numpy as np
    import torch
    cnt = np.zeros(M, np.int64)
    idx = np.zeros((M, K), np.int64)
    w = np.zeros((M, K), np.float32)

    def ratio(alpha):
        b = torch.from_numpy(synth.zipf_bias(E, 1.1, alpha, seed=0)).cuda()
        ctx.route(MB.make_desc(layer, bias=b), M, x, cnt, idx, w)
        act = idx[np.arange(K)[None, :] < cnt[:, None]]
        loads = np.bincount(act, minlength=E)
        return float(loads.max() / loads.mean()), b

    lo, hi = 0.0, 1.0
    for _ in range(14):
        mid = 0.5 * (lo + hi)
        if ratio(mid)[0] < target:
            lo = mid
        else:
            hi = mid
    alpha = 0.5 * (lo + hi)
    r, b = ratio(alpha)
    return alpha, r, b


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.06)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ----------------------------------------------------------------- CPU leg
def host_layer(seed: int):
    """Layer weights built on the CPU with the oracle's quantizer (no GPU code)."""
    import numpy as np
    import oracle as O
    rng = np.random.default_rng(seed)
    w = dict(d=D, F=F, E=E, top_k=K)
    rf = rng.standard_normal((E, D), dtype=np.float32) * np.float32(0.02)
    w["router_p"], w["router_s"], _ = O.quantize_q4_0(rf)
    gp, gs, dp, ds = [], [], [], []
    for _ in range(E):
        p, s, _ = O.quantize_q4_0(rng.standard_normal(2 * F * D, dtype=np.float32) * np.float32(0.02))
        gp.append(p)
        gs.append(s)
        p, s, _ = O.quantize_q4_0(rng.standard_normal(D * F, dtype=np.float32) * np.float32(0.02))
        dp.append(p)
        ds.append(s)
    w["gu_p"], w["gu_s"] = np.concatenate(gp), np.concatenate(gs)
    w["dn_p"], w["dn_s"] = np.concatenate(dp), np.concatenate(ds)
    for k in ("router_scale", "pre_norm_w", "post_norm_w"):
        w[k] = np.ones(D, np.float32)
    w["per_expert_scale"] = np.ones(E, np.float32)
    dense = {}
    for name, ci, co in DENSE:
        p, s, _ = O.quantize_q4_0(rng.standard_normal(ci * co, dtype=np.float32) * np.float32(0.02))
        dense[name] = (p, s, ci, co)
    return w, dense


def cpu_step(L, dense, x, x_o, nthreads):
    import oracle as O
    O.layer_forward(L, x, post_norm=True, prec=O.F32, nthreads=nthreads)
    for name, (p, s, ci, co) in dense.items():
        O.q4_matmul(p, s, x_o if name == "o" else x, ci, co, prec=O.F32, nthreads=nthreads)


def cpu_time(w, dense, M, budget_s, max_steps, nthreads, warmup=1):
    """Times the oracle's fp32 restatement of the reference kernels."""
    import numpy as np
    import oracle as O
    L = O.make_layer(w)
    rng = np.random.default_rng(5)
    x = rng.standard_normal((M, D)).astype(np.float32)
    x_o = rng.standard_normal((M, 4096)).astype(np.float32)
    use_dense = dense if M == 16 else {}
    for _ in range(warmup):
        cpu_step(L, use_dense, x, x_o, nthreads)
    t0 = time.perf_counter()
    n = 0
    while n < max_steps and (n == 0 or time.perf_counter() - t0 < budget_s):
        cpu_step(L, use_dense, x, x_o, nthreads)
        n += 1
    dt = time.perf_counter() - t0
    return M * n / dt, n, dt


def run_reference(args, ws, rank):
    """--impl reference: the reference's CPU algorithm (oracle fp32 port of
    moe_kernels.mojo; the Mojo toolchain is absent) on the host cores."""
    if rank != 0:
        return 0
    M = WORKLOADS[args.workload]["M"]
    nthreads = os.cpu_count() or 1
    w, dense = host_layer(seed=0)
    # bounded sample: at most ~120 s for the K timed steps
    t_one = cpu_time(w, dense, M, 0.0, 1, nthreads, warmup=0)
    per_step = M / t_one[0]
    budget = 120.0 / max(1, args.steps)
    m = M
    if per_step > budget and M > 1:
        m = 5 if M > 5 and per_step * 5 / M <= budget else 1
    import numpy as np
    import oracle as O
    L = O.make_layer(w)
    rng = np.random.default_rng(5)
    x = rng.standard_normal((m, D)).astype(np.float32)
    x_o = rng.standard_normal((m, 4096)).astype(np.float32)
    use_dense = dense if M == 16 else {}
    for _ in range(max(0, min(args.warmup, 3))):
        cpu_step(L, use_dense, x, x_o, nthreads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_step(L, use_dense, x, x_o, nthreads)
    dt = time.perf_counter() - t0
    value = m * args.steps / dt
    sample = f"{m} of {M} tokens per step, {args.steps} steps, 1 layer (+dense q/k/v/o)" if M == 16 \
        else f"{m} of {M} tokens per step, {args.steps} steps, 1 layer"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(args, M),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": nthreads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def dtype_desc(args, M):
    """The arithmetic the GPU arm's expert GEMMs run (routing, norms and the
    combine are fp32 on CUDA cores in every case)."""
    path = getattr(args, "path", "auto")
    if path == "gemv" or (path == "auto" and M < 2):
        return "f32 (CUDA-core fp32 FMA throughout)"
    return "f32 io and routing; fp16 x fp16 -> fp32 tcgen05 expert GEMMs"


def workload_config(args, M):
    return {"workload": WORKLOAD_NAMES[args.workload],
            "tokens_per_step": M, "embed_dim": D, "expert_mlp_dim": F, "num_experts": E, "top_k": K,
            "layers_cycled": args.layers,
            "l2": f"weights of {args.layers} distinct layers cycled per step ({args.layers * 476} MB > 126 MB L2)",
            "post_norm": True,
            "parallelism": (f"ep{dist_setup()[0]}: 128/{dist_setup()[0]} experts per GPU, tokens replicated, "
                            f"NCCL all-reduce of partial outputs"
                            f"{' inside the layer call (moe_ep_init)' if getattr(args, 'parallel', 'ep') == 'ep-native' else ''}"
                            f"; dense rows sharded"
                            if dist_setup()[0] > 1 and getattr(args, "parallel", "ep") in ("ep", "ep-native")
                            else f"replicas x{dist_setup()[0]}"),
            "gemm_path": getattr(args, "path", "auto"),
            "tc_kernel": getattr(args, "tc_kernel", "stream"),
            "dense_projections": "own contexts and streams, concurrent with the MoE layer",
            "cuda_graph": not getattr(args, "no_graph", False)}


# ----------------------------------------------------------------- GPU leg
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (workload default)")
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode16", choices=sorted(WORKLOADS))
    ap.add_argument("--layers", type=int, default=None, help="distinct layers cycled (workload default)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget-s", type=float, default=12.0)
    ap.add_argument("--no-graph", action="store_true", help="launch every step from the host")
    ap.add_argument("--graph", action="store_true",
                    help="with N > 1, capture steps (NCCL all-reduce included) in CUDA graphs; "
                         "by default N > 1 launches eagerly")
    ap.add_argument("--path", default="auto", choices=["auto", "gemv", "tc"],
                    help="expert/dense GEMM path: CUDA-core GEMV, tcgen05, or automatic")
    ap.add_argument("--parallel", default="ep", choices=["ep", "ep-native", "replicas"],
                    help="N > 1: expert parallel (128/N experts per GPU, tokens replicated, one NCCL "
                         "all-reduce per layer; dense projections row-sharded) with the all-reduce "
                         "issued by torch.distributed (ep) or inside the library's layer call "
                         "(ep-native, moe_ep_init), or independent replicas")
    ap.add_argument("--tc-kernel", default="stream", choices=["stream", "stream-all", "general"],
                    help="tensor-core kernel for token tiles <= 64: streaming for the expert GEMMs "
                         "(default), streaming also for dense projections, or general")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    wl = WORKLOADS[args.workload]
    if int(os.environ.get("WORLD_SIZE", "1")) > 1 and not args.graph:
        # replaying graphs that hold the NCCL all-reduce was slower than eager
        # launches at 8 ranks (825 us per step replayed, 462 us per step for
        # eager calls even with host copies), so N > 1 runs eagerly
        args.no_graph = True
    if args.layers is None:
        args.layers = wl["layers"]
    if args.steps is None:
        args.steps = wl.get("steps", 2000)
    ws, rank, local = dist_setup()
    if args.impl == "reference":
        return run_reference(args, ws, rank)

    import numpy as np
    import torch
    import ep as EP
    import moe_b200 as MB
    import synth

    torch.cuda.set_device(local)
    pg = None
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        pg = dist
    ctx = MB.Context(local)
    stream = torch.cuda.current_stream()
    ctx.set_stream(stream.cuda_stream)
    ctx.set_gemm_path({"auto": MB.PATH_AUTO, "gemv": MB.PATH_GEMV, "tc": MB.PATH_TC}[args.path])
    ctx.set_option(MB.OPT_TC_STREAM, {"general": 0, "stream": 1, "stream-all": 2}[args.tc_kernel])
    M = wl["M"]
    use_ep = ws > 1 and args.parallel in ("ep", "ep-native")
    native_ep = use_ep and args.parallel == "ep-native"
    if native_ep:  # the library's own communicator: rank 0's id to every rank
        uid = [MB.ep_unique_id() if rank == 0 else None]
        pg.broadcast_object_list(uid, src=0)
        ctx.ep_init(uid[0], rank, ws)
    # expert parallel: every rank holds the same layers and tokens and
    # evaluates its own expert range; replicas: independent data per rank
    seed_rank = 0 if use_ep else rank

    layers, descs = [], []
    for li in range(args.layers):
        lw = synth.make_layer(ctx, seed=1000 * seed_rank + li)
        layers.append(lw)
        descs.append(MB.make_desc(lw))
    skew = None
    if wl.get("skew"):
        x_cal = synth.make_x(M, seed=499)
        alpha, ratio, bias = calibrate_skew(ctx, MB, synth, layers[0], x_cal, M)
        descs = [MB.make_desc(lw, bias=bias) for lw in layers]
        skew = {"zipf_s": 1.1, "alpha": alpha, "max_over_mean_load": ratio}
    gen = torch.Generator(device="cuda")
    gen.manual_seed(77 + seed_rank)
    dense = {}
    if M == 16:
        for name, ci, co in DENSE:
            wt = torch.randn(ci * co, generator=gen, device="cuda") * 0.02
            p, s = synth.quantize(ctx, wt)
            if use_ep:  # row-sharded: this rank's slice of the output features
                r0, r1 = EP.row_range(rank, ws, co)
                p, s, co = p[r0 * ci // 2:r1 * ci // 2], s[r0 * ci // 32:r1 * ci // 32], r1 - r0
            dense[name] = (p, s, ci, co)
    xs = [synth.make_x(M, seed=500 + 10 * seed_rank + li) for li in range(args.layers)]
    x_o = torch.randn((M, 4096), generator=gen, device="cuda")
    out = torch.empty((M, D), device="cuda")
    dense_out = {n: torch.empty((M, co), device="cuda") for n, (_, _, _, co) in dense.items()}
    # The dense projections do not depend on the MoE layer or on each other in
    # this workload, so each gets its own context and stream: they run beside
    # the MoE layer (fork / join with events, captured into the same graph).
    dctx, dstream = {}, {}
    for name in dense:
        dctx[name] = MB.Context(local)
        dstream[name] = torch.cuda.Stream()
        dctx[name].set_stream(dstream[name].cuda_stream)
        dctx[name].set_gemm_path({"auto": MB.PATH_AUTO, "gemv": MB.PATH_GEMV, "tc": MB.PATH_TC}[args.path])
        dctx[name].set_option(MB.OPT_TC_STREAM, {"general": 0, "stream": 1, "stream-all": 2}[args.tc_kernel])

    # routing per layer (unique experts of this rank -> algorithmic bytes)
    e_lo, e_hi = EP.expert_range(rank, ws, E) if use_ep else (0, E)
    epl = EP.ExpertParallelLayer(ctx, E) if use_ep and not native_ep else None
    uniq, pairs_l = [], []
    for li in range(args.layers):
        cnt = np.zeros(M, np.int64)
        idx = np.zeros((M, K), np.int64)
        w = np.zeros((M, K), np.float32)
        ctx.layer_forward(descs[li], M, xs[li], out, MB.F_POST_NORM, cnt, idx, w)
        uniq.append(len({int(idx[t, k]) for t in range(M) for k in range(cnt[t])
                         if e_lo <= int(idx[t, k]) < e_hi}))
        pairs = int(cnt.sum())
        pairs_l.append(pairs)

    def moe_step(li, x, o):
        if epl is not None:
            epl.forward(descs[li], M, x, o, MB.F_POST_NORM, layers[li]["post_norm_w"])
        else:
            ctx.layer_forward(descs[li], M, x, o, MB.F_POST_NORM)

    def step(i):
        li = i % args.layers
        main = torch.cuda.current_stream()
        fork = torch.cuda.Event()
        fork.record(main)
        moe_step(li, xs[li], out)
        joins = []
        for name, (p, s, ci, co) in dense.items():
            dstream[name].wait_event(fork)
            dctx[name].q4_matmul_batchN(M, p, s, x_o if name == "o" else xs[li], dense_out[name], ci, co)
            ev = torch.cuda.Event()
            ev.record(dstream[name])
            joins.append(ev)
        for ev in joins:
            main.wait_event(ev)

    def all_launches():
        return ctx.kernel_launches + sum(c.kernel_launches for c in dctx.values())

    ctx.set_async(True)
    for c in dctx.values():
        c.set_async(True)
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    # One CUDA graph per layer holding a whole step (the library's calls are
    # asynchronous and allocation-free once warm), replayed step by step.
    graphs, launches_per_step = [], None
    if not args.no_graph:
        cap = torch.cuda.Stream()
        ctx.set_stream(cap.cuda_stream)
        n_cap = all_launches()
        for li in range(args.layers):
            graphs.append(torch.cuda.CUDAGraph())
            with torch.cuda.graph(graphs[-1], stream=cap):
                step(li)
        launches_per_step = (all_launches() - n_cap) / args.layers
        if pg:
            launches_per_step += 1  # the NCCL all-reduce kernel is not counted by the library
        ctx.set_stream(stream.cuda_stream)
        for i in range(args.warmup):
            graphs[i % args.layers].replay()
        torch.cuda.synchronize()

    def run_step(i):
        if graphs:
            graphs[i % args.layers].replay()
        else:
            step(i)

    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    n0 = all_launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for i in range(args.steps):
            run_step(i)
        ev1.record(stream)
        torch.cuda.synchronize()
    launches = all_launches() - n0 if not graphs else int(round(launches_per_step * args.steps))
    ms = ev0.elapsed_time(ev1)
    if pg:
        t = torch.tensor([ms], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
        pg.barrier()
    torch.cuda.synchronize()
    ms_per_step = ms / args.steps
    # expert parallel: all ranks serve the same M tokens; replicas: M each
    tokens_per_step = M if use_ep else ws * M
    value = tokens_per_step * args.steps / (ms / 1e3)

    # profiled pass over the same steps: per-kernel device time
    for c in [ctx, *dctx.values()]:
        c.profile_enable(True)
    for i in range(args.steps):
        step(i)
    torch.cuda.synchronize()
    prof = ctx.profile_read()
    for c in dctx.values():
        for k, (t_ms, n_l) in c.profile_read().items():
            t0, n0_ = prof.get(k, (0.0, 0))
            prof[k] = (t0 + t_ms, n0_ + n_l)
    for c in [ctx, *dctx.values()]:
        c.profile_enable(False)

    # End to end through the public API with pinned host buffers: every call
    # stages its host inputs (H2D) and copies its outputs back (D2H) on its
    # context's stream; the calls are asynchronous (moe_set_async), the dense
    # projections run on their own contexts' streams as in the device-timed
    # step, and the step ends when the main stream has joined them.
    x_h = [x.cpu().pin_memory() for x in xs]
    xo_h = x_o.cpu().pin_memory()
    out_h = torch.empty((M, D)).pin_memory()
    dout_h = {n: torch.empty((M, co)).pin_memory() for n, (_, _, _, co) in dense.items()}
    h2d = M * D * 4 + sum((M * (4096 if n == "o" else D) * 4) for n in dense)
    d2h = M * D * 4 + sum(M * co * 4 for (_, _, _, co) in dense.values())

    x_d = torch.empty((M, D), device="cuda")

    def step_e2e(i):
        li = i % args.layers
        if epl is not None:  # the collective needs device buffers: copy in, reduce, copy out
            x_d.copy_(x_h[li], non_blocking=True)
            epl.forward(descs[li], M, x_d, out, MB.F_POST_NORM, layers[li]["post_norm_w"])
            out_h.copy_(out, non_blocking=True)
            for name, (p, s, ci, co) in dense.items():
                ctx.q4_matmul_batchN(M, p, s, xo_h if name == "o" else x_h[li], dout_h[name], ci, co)
            return
        main = torch.cuda.current_stream()
        fork = torch.cuda.Event()
        fork.record(main)
        ctx.layer_forward(descs[li], M, x_h[li], out_h, MB.F_POST_NORM)
        joins = []
        for name, (p, s, ci, co) in dense.items():
            dstream[name].wait_event(fork)
            dctx[name].q4_matmul_batchN(M, p, s, xo_h if name == "o" else x_h[li], dout_h[name], ci, co)
            ev = torch.cuda.Event()
            ev.record(dstream[name])
            joins.append(ev)
        for ev in joins:
            main.wait_event(ev)

    e2e_steps = max(1, min(args.steps, 500))
    for i in range(3):
        step_e2e(i)
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(e2e_steps):
        step_e2e(i)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if pg:
        t = torch.tensor([e2e_ms], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = tokens_per_step * e2e_steps / (e2e_ms / 1e3)

    # roofline of the dominant kernel (largest share of profiled time)
    hbm, tf_burst, tf_sust, src = peaks()
    pairs_mean = sum(pairs_l) / len(pairs_l)
    u_mean = sum(uniq) / len(uniq)
    # the dominant kernel of the MoE path (the dense projections run on their
    # own streams beside it, and their summed time is not one kernel's)
    dom = max((kv for kv in prof.items() if kv[0] in ("gemv_gate_up", "gemv_down", "tc_gate_up", "tc_down")),
              key=lambda kv: kv[1][0])[0] if prof else None
    alg = {
        "gemv_gate_up": u_mean * GU_BYTES + M * D * 4 + M * K * F * 4,
        "gemv_down": u_mean * DN_BYTES + M * K * F * 4 + M * K * D * 4,
        "tc_gate_up": u_mean * GU_BYTES + M * K * D * 2 + M * K * F * 2,
        "tc_down": u_mean * DN_BYTES + M * K * F * 2 + M * K * D * 4,
        "q4_matmul": sum(q4_bytes(ci, co) + M * (ci + co) * 4 for (_, _, ci, co) in dense.values()) / max(1, len(dense)),
        "router": ROUTER_BYTES + M * D * 4 + M * E * 4,
        "prep": 4 * M * D * 4,
    }
    roof = None
    if wl.get("skew") and dom in ("tc_gate_up", "tc_down") and prof[dom][1] > 0:
        # prefill scale: tensor-bound; FLOPs of the dominant grouped GEMM per launch
        flops = pairs_mean * 2 * (2 * F * D if dom == "tc_gate_up" else D * F)
        avg_ms = prof[dom][0] / prof[dom][1]
        achieved = flops / (avg_ms / 1e3) / 1e12
        roof = {"bound": "tensor", "kernel": dom, "achieved": achieved, "peak": tf_sust, "unit": "TFLOP/s",
                "frac": achieved / tf_sust, "traffic": None, "flops_per_launch": flops, "avg_launch_ms": avg_ms,
                "peak_source": f"MEASURED_PEAKS.json bf16_tflops_sustained ({'of measured' if src == 'measured' else 'of fallback'})"}
    elif dom in alg and prof[dom][1] > 0:
        avg_ms = prof[dom][0] / prof[dom][1]
        achieved = alg[dom] / (avg_ms / 1e3) / 1e9
        traffic = None
        tp = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tp):
            with open(tp) as f:
                traffic = json.load(f).get(args.workload, {}).get(dom)
        roof = {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "traffic": traffic,
                "alg_bytes_per_launch": alg[dom], "avg_launch_ms": avg_ms,
                "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({'of measured' if src == 'measured' else 'of fallback'})"}
    step_bytes = u_mean * (GU_BYTES + DN_BYTES) + ROUTER_BYTES + 2 * M * D * 4 + \
        sum(q4_bytes(ci, co) for (_, _, ci, co) in dense.values())
    step_roof = {"alg_bytes_per_step": step_bytes, "achieved_gbs": step_bytes / (ms_per_step / 1e3) / 1e9,
                 "frac_of_hbm": step_bytes / (ms_per_step / 1e3) / 1e9 / hbm,
                 "unique_experts_per_step": u_mean, "pairs_per_step": pairs,
                 "kernel_ms_per_step": {k: v[0] / args.steps for k, v in prof.items()}}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        host = synth.to_host(layers[0])
        hd = {n: (p.cpu().numpy(), s.cpu().numpy(), ci, co) for n, (p, s, ci, co) in dense.items()}
        nth = os.cpu_count() or 1
        v, n, dt = cpu_time(host, hd, M, args.cpu_budget_s, 200, nth)
        cpu = {"value": v, "unit": "tokens/s", "cores": nth, "kind": "port",
               "sample": f"{n} full steps of {M} tokens (layer 0{', + dense q/k/v/o' if hd else ''}) in {dt:.1f} s"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong" if use_ep else "weak", "vs_baseline": None, "dtype": dtype_desc(args, M),
            "data": "synthetic",
            "config": dict(workload_config(args, M), **({"skew": skew} if skew else {})),
            "roofline": roof, "step_roofline": step_roof,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps},
            "gpu_launches": launches, "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    # graphs that hold NCCL calls must be gone before the process group is
    graphs.clear()
    import gc
    gc.collect()
    torch.cuda.synchronize()
    for c in dctx.values():
        c.close()
    ctx.close()
    if pg:
        pg.barrier()
        torch.cuda.synchronize()
        pg.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
