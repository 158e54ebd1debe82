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
# tokens per step, distinct layers, whether a step runs the whole stack of
# layers, skewed routing, default step count, the N > 1 form
WORKLOADS = {
    "decode16": dict(M=16, layers=4),
    "decode1": dict(M=1, layers=4),
    "block256": dict(M=256, layers=4),
    "decode64": dict(M=64, layers=30, stack=True, steps=100),
    "prefill8k": dict(M=8192, layers=30, stack=True, skew=True, steps=5, a2a=True),
}
WORKLOAD_NAMES = {
    "decode16": "cfg2: M=16 decode MoE layer + dense q/k/v/o",
    "decode1": "cfg1: M=1 decode MoE layer",
    "block256": "cfg3: M=256 block through the MoE layer",
    "decode64": "cfg4: M=64 decode through the 30-layer stack (independent seeded layers); a step is all 30 layers",
    "prefill8k": "cfg5: M=8192 (4 x 2048) through the 30-layer stack, Zipf(1.1)-skewed router; a step is all 30 layers",
}
SUB_WORKLOADS = ("decode1", "block256", "decode64", "prefill8k")
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
    """nvidia-smi clocks/throttle sampling during the timed region.

    nvidia-smi needs a few hundred ms to start, so it is started ahead of the
    timed region and its rows carry their arrival time; begin()/end() mark the
    region on the host (from the start event to the final synchronize).  A
    region shorter than the sampling interval keeps the row nearest to it,
    taken while the warm-up steps ran."""

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None
        self.t0 = self.t1 = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            deadline = time.monotonic() + 3.0
            while not self.rows and time.monotonic() < deadline and self.proc.poll() is None:
                time.sleep(0.01)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.monotonic(), [c.strip() for c in line.split(",")]))

    def begin(self):
        self.t0 = time.monotonic()

    def end(self):
        self.t1 = time.monotonic()
        time.sleep(0.03)  # the row sampled at the end of the region

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        rows = self.rows
        if self.t0 is not None and self.t1 is not None:
            inside = [r for t, r in rows if self.t0 <= t <= self.t1]
            if not inside and rows:
                # shorter than the interval: the row nearest to the region
                t_mid = 0.5 * (self.t0 + self.t1)
                inside = [min(rows, key=lambda tr: abs(tr[0] - t_mid))[1]]
            rows_used = inside
        else:
            rows_used = [r for _, r in rows]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows_used:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
               "reasons": sorted(reasons), "samples": len(sm)}
        if self.t0 is not None and self.t1 is not None:
            out["window_ms"] = round((self.t1 - self.t0) * 1e3, 1)
        return out


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
    n_lay = args.layers if WORKLOADS[args.workload].get("stack") else 1
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
    value = m * args.steps / dt / n_lay
    sample = f"{m} of {M} tokens per step, {args.steps} steps, 1 layer (+dense q/k/v/o)" if M == 16 \
        else f"{m} of {M} tokens per step, {args.steps} steps, 1 layer"
    if n_lay > 1:
        sample += f"; rate divided by {n_lay} for the {n_lay}-layer step"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps * n_lay,
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


def workload_config(args, M, par="replicas", ws=1):
    wl = WORKLOADS[args.workload]
    stack = bool(wl.get("stack"))
    n_mb = args.layers * 476
    par_desc = {
        "replicas": f"replicas x{ws}",
        "ep": f"ep{ws}: 128/{ws} experts per GPU, tokens replicated, torch.distributed NCCL all-reduce of "
              f"partial outputs; dense rows sharded",
        "ep-native": f"ep{ws}: 128/{ws} experts per GPU, tokens replicated, NCCL all-reduce inside the layer "
                     f"call (moe_ep_init); dense rows sharded",
        "ep-gather": f"ep{ws}: 128/{ws} experts per GPU (weight slices), {M} own tokens per GPU; the layer "
                     f"call all-gathers the tokens and reduce-scatters the partial outputs (NCCL)",
        "ep-a2a": f"ep{ws}: 128/{ws} experts per GPU (weight slices), the {M} tokens sharded over the GPUs; "
                  f"the layer call sends routed rows to the expert owners and back (NCCL send/recv)",
    }[par]
    return {"workload": WORKLOAD_NAMES[args.workload],
            "tokens_per_step": M, "embed_dim": D, "expert_mlp_dim": F, "num_experts": E, "top_k": K,
            "layers": args.layers, "layers_per_step": args.layers if stack else 1,
            "l2": f"weights of {args.layers} distinct layers ({n_mb} MB > 126 MB L2) "
                  f"{'run back to back in every step' if stack else 'cycled step by step'}",
            "post_norm": True, "parallelism": par_desc,
            "gemm_path": getattr(args, "path", "auto"),
            "tc_kernel": getattr(args, "tc_kernel", "stream"),
            "dense_projections": "own contexts and streams, concurrent with the MoE layer" if M == 16 else "none",
            "cuda_graph": not getattr(args, "no_graph", False)}


# ----------------------------------------------------------------- GPU leg
PAR_HELP = ("N > 1: ep-gather (default: each rank its own tokens, routed on that rank, 128/N experts per "
            "rank, the library all-gathers the routed rows and reduce-scatters the partial outputs inside the "
            "layer call), ep-a2a (each rank a shard of the workload's tokens, routed rows to the expert owners "
            "and back over NCCL inside the layer call), ep / ep-native (tokens replicated, NCCL all-reduce of "
            "partial outputs by torch.distributed / inside the library), or replicas")


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (workload default)")
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode16", choices=sorted(WORKLOADS))
    ap.add_argument("--layers", type=int, default=None, help="distinct layers (workload default)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget-s", type=float, default=12.0)
    ap.add_argument("--no-workloads", action="store_true",
                    help="N = 1, default workload: skip the other configurations' sub-lines")
    ap.add_argument("--no-graph", action="store_true", help="launch every step from the host")
    ap.add_argument("--graph", action="store_true",
                    help="with N > 1, capture steps (collectives included) in CUDA graphs; "
                         "by default N > 1 launches eagerly")
    ap.add_argument("--path", default="auto", choices=["auto", "gemv", "tc"],
                    help="expert/dense GEMM path: CUDA-core GEMV, tcgen05, or automatic")
    ap.add_argument("--parallel", default=None,
                    choices=["ep-gather", "ep-a2a", "ep", "ep-native", "replicas"], help=PAR_HELP)
    ap.add_argument("--fused-route", type=int, default=None, choices=[0, 1, 2],
                    help="routing of small batches: separate kernels (0), one cluster (1), one cooperative "
                         "grid launch (2); default: the library's")
    ap.add_argument("--tc-kernel", default="stream", choices=["stream", "stream-all", "general"],
                    help="tensor-core kernel for token tiles <= 64: streaming for the expert GEMMs "
                         "(default), streaming also for dense projections, or general")
    return ap.parse_args(argv)


def main():
    args = parse_args()
    args.warmup = max(args.warmup, 3)
    ws, rank, local = dist_setup()
    explicit_steps, explicit_layers = args.steps, args.layers
    fill_defaults(args, ws)
    if args.impl == "reference":
        return run_reference(args, ws, rank)

    import torch
    torch.cuda.set_device(local)
    pg = None
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        pg = dist
    line = measure(args, pg, ws, rank, local)
    if ws == 1 and args.workload == "decode16" and not args.no_workloads:
        # the other configurations, each measured the same way in this run
        subs = {}
        for name in SUB_WORKLOADS:
            sa = parse_args([])
            sa.workload, sa.warmup, sa.path, sa.tc_kernel = name, 3, args.path, args.tc_kernel
            sa.fused_route = args.fused_route
            sa.no_cpu_baseline = args.no_cpu_baseline
            sa.cpu_budget_s = min(args.cpu_budget_s, 4.0)
            fill_defaults(sa, ws)
            sub = measure(sa, None, 1, 0, local)
            subs[name] = {k: sub[k] for k in ("value", "unit", "ms_per_step", "steps", "warmup", "dtype",
                                              "config", "roofline", "step_roofline", "cpu_baseline", "e2e",
                                              "gpu_launches", "clocks") if k in sub}
        line["workloads"] = subs
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        torch.cuda.synchronize()
        pg.destroy_process_group()
    return 0


def fill_defaults(args, ws):
    wl = WORKLOADS[args.workload]
    if args.parallel is None:
        # the gather form for every workload: at 2 ranks it gave prefill8k
        # 159.9k tokens/s and decode64 22.6k against the all-to-all form's
        # 73.1k and 7.1k (one GPU: 98.1k and 10.1k); the all-to-all form moves
        # up to K rows per token, the gather form one
        args.parallel = "ep-gather" if ws > 1 else "replicas"
    if ws > 1 and not args.graph and args.parallel not in ("ep-gather",):
        # replaying graphs that hold NCCL calls was slower than eager launches
        # at 8 ranks for the replicated all-reduce form (825 us per step
        # replayed against 462 us eager); the gather form is faster replayed
        # (229 against 497 us at 8 ranks, 199 against 231 at 2)
        args.no_graph = True
    if args.parallel == "ep-a2a":
        args.no_graph = True  # the all-to-all form reads its row counts on the host
    if args.layers is None:
        args.layers = wl["layers"]
    if args.steps is None:
        args.steps = wl.get("steps", 2000)


def measure(args, pg, ws, rank, local):
    import numpy as np
    import torch
    import ep as EP
    import moe_b200 as MB
    import synth

    wl = WORKLOADS[args.workload]
    stack = bool(wl.get("stack"))
    ctx = MB.Context(local)
    stream = torch.cuda.current_stream()
    ctx.set_stream(stream.cuda_stream)
    ctx.set_gemm_path({"auto": MB.PATH_AUTO, "gemv": MB.PATH_GEMV, "tc": MB.PATH_TC}[args.path])
    ctx.set_option(MB.OPT_TC_STREAM, {"general": 0, "stream": 1, "stream-all": 2}[args.tc_kernel])
    if args.fused_route is not None:
        ctx.set_option(MB.OPT_FUSED_ROUTE, args.fused_route)
    M_total = wl["M"]
    par = args.parallel if ws > 1 else "replicas"
    lib_ep = par in ("ep-native", "ep-gather", "ep-a2a")
    shared_layers = par != "replicas"       # every rank holds (a slice of) the same layers
    if par == "ep-a2a":  # a shard of the workload's tokens per rank (strong scaling)
        t0_, t1_ = EP.row_range(rank, ws, M_total)
        M = t1_ - t0_
    else:
        M = M_total
    if lib_ep:  # the library's own communicator: rank 0's id to every rank
        uid = [MB.ep_unique_id() if rank == 0 else None]
        pg.broadcast_object_list(uid, src=0)
        ctx.ep_init(uid[0], rank, ws)
        ctx.set_option(MB.OPT_EP_MODE, {"ep-native": MB.EP_REPLICATED, "ep-gather": MB.EP_GATHER,
                                        "ep-a2a": MB.EP_ALL_TO_ALL}[par])
    seed_rank = 0 if shared_layers else rank
    # own batches per rank (gather form, replicas); the all-to-all form shards
    # one global batch; the replicated forms share one batch
    tok_seed = rank if par in ("ep-gather", "replicas") else 0
    e_lo, e_hi = EP.expert_range(rank, ws, E) if par != "replicas" else (0, E)

    layers, descs = [], []
    for li in range(args.layers):
        lw = synth.make_layer(ctx, seed=1000 * seed_rank + li)
        layers.append(lw)
    skew = None
    bias = None
    if wl.get("skew"):
        x_cal = synth.make_x(M_total, seed=499)
        alpha, ratio, bias = calibrate_skew(ctx, MB, synth, layers[0], x_cal, M_total)
        skew = {"zipf_s": 1.1, "alpha": alpha, "max_over_mean_load": ratio}
    full_descs = [MB.make_desc(lw, bias=bias) for lw in layers]
    if par in ("ep-gather", "ep-a2a"):
        # each rank hands the library only its experts' weights
        ctx.set_option(MB.OPT_EP_LOCAL_WEIGHTS, 1)
        El = e_hi - e_lo
        for lw in layers:
            loc = dict(lw)
            loc["gu_p"] = lw["gu_p"][e_lo * 2 * F * D // 2:e_hi * 2 * F * D // 2]
            loc["gu_s"] = lw["gu_s"][e_lo * 2 * F * D // 32:e_hi * 2 * F * D // 32]
            loc["dn_p"] = lw["dn_p"][e_lo * D * F // 2:e_hi * D * F // 2]
            loc["dn_s"] = lw["dn_s"][e_lo * D * F // 32:e_hi * D * F // 32]
            descs.append(MB.make_desc(loc, bias=bias))
        assert El * ws == E
    else:
        descs = full_descs
    gen = torch.Generator(device="cuda")
    gen.manual_seed(77 + tok_seed)
    dense = {}
    if M_total == 16:
        for name, ci, co in DENSE:
            wt = torch.randn(ci * co, generator=gen, device="cuda") * 0.02
            p, s = synth.quantize(ctx, wt)
            if par in ("ep", "ep-native"):  # row-sharded: this rank's slice of the output features
                r0, r1 = EP.row_range(rank, ws, co)
                p, s, co = p[r0 * ci // 2:r1 * ci // 2], s[r0 * ci // 32:r1 * ci // 32], r1 - r0
            dense[name] = (p, s, ci, co)
    n_x = 1 if stack else args.layers

    def make_tokens(r):
        xs_r = []
        for li in range(n_x):
            xf = synth.make_x(M_total, seed=500 + 10 * r + li)
            if par == "ep-a2a":
                xf = xf[t0_:t1_].contiguous()
            xs_r.append(xf)
        return xs_r
    xs = make_tokens(tok_seed)
    x_o = torch.randn((max(M, 1), 4096), generator=gen, device="cuda")
    out = torch.empty((max(M, 1), D), device="cuda")
    out2 = torch.empty((max(M, 1), D), device="cuda")
    dense_out = {n: torch.empty((M, co), device="cuda") for n, (_, _, _, co) in dense.items()}
    dctx, dstream = {}, {}
    for name in dense:
        dctx[name] = MB.Context(local)
        dstream[name] = torch.cuda.Stream()
        dctx[name].set_stream(dstream[name].cuda_stream)
        dctx[name].set_gemm_path({"auto": MB.PATH_AUTO, "gemv": MB.PATH_GEMV, "tc": MB.PATH_TC}[args.path])
        dctx[name].set_option(MB.OPT_TC_STREAM, {"general": 0, "stream": 1, "stream-all": 2}[args.tc_kernel])

    # routing of the tokens this rank's experts see, per layer (unique experts
    # -> algorithmic bytes), on a plain context over the full layer
    rctx = MB.Context(local)
    rctx.set_stream(stream.cuda_stream)
    uniq, pairs_l = [], []
    for li in range(args.layers):
        if par == "ep-gather":
            xr = torch.cat([make_tokens(r)[li % n_x] for r in range(ws)])
        elif par == "ep-a2a":
            xr = synth.make_x(M_total, seed=500 + (li % n_x))
        else:
            xr = xs[li % n_x]
        Mr = xr.shape[0]
        cnt = np.zeros(Mr, np.int64)
        idx = np.zeros((Mr, K), np.int64)
        w = np.zeros((Mr, K), np.float32)
        tmp = torch.empty((Mr, D), device="cuda")
        rctx.route(full_descs[li], Mr, xr, cnt, idx, w)
        act = idx[np.arange(K)[None, :] < cnt[:, None]]
        uniq.append(int(np.unique(act[(act >= e_lo) & (act < e_hi)]).size))
        pairs_l.append(int(((act >= e_lo) & (act < e_hi)).sum()))
        del tmp
    rctx.close()
    epl = EP.ExpertParallelLayer(ctx, E) if par == "ep" else None

    def moe_layer(li, x, o):
        if epl is not None:
            epl.forward(descs[li], M, x, o, MB.F_POST_NORM, layers[li]["post_norm_w"])
        elif M > 0:
            ctx.layer_forward(descs[li], M, x, o, MB.F_POST_NORM)
        else:  # an empty token shard still takes part in the exchange
            ctx.layer_forward(descs[li], 0, None, None, MB.F_POST_NORM)

    def step(i):
        main = torch.cuda.current_stream()
        fork = torch.cuda.Event()
        fork.record(main)
        if stack:  # the whole stack: every layer's output is the next layer's input
            h = xs[0]
            for li in range(args.layers):
                o = (out, out2)[li % 2]
                moe_layer(li, h, o)
                h = o
        else:
            li = i % args.layers
            moe_layer(li, xs[li], out)
        joins = []
        for name, (p, s, ci, co) in dense.items():
            dstream[name].wait_event(fork)
            dctx[name].q4_matmul_batchN(M, p, s, x_o if name == "o" else xs[i % n_x], dense_out[name], ci, co)
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
    # the clock sampler starts now, so that it runs by the timed region
    clk = ClockSampler(local).__enter__()
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    # One CUDA graph per distinct step (the library's calls are asynchronous
    # and allocation-free once warm), replayed step by step.  With several
    # ranks the expert-parallel forms replay graphs too: at 8 ranks the gather
    # form took 229 us per step replayed against 497 us launched eagerly (its
    # NCCL calls are captured in the graph).
    n_graphs = 1 if stack else args.layers
    graphs, launches_per_step = [], None
    if not args.no_graph:
        cap = torch.cuda.Stream()
        ctx.set_stream(cap.cuda_stream)
        n_cap = all_launches()
        for gi in range(n_graphs):
            graphs.append(torch.cuda.CUDAGraph())
            with torch.cuda.graph(graphs[-1], stream=cap):
                step(gi)
        launches_per_step = (all_launches() - n_cap) / n_graphs
        if pg:
            launches_per_step += 2 * (args.layers if stack else 1)  # NCCL kernels are not counted by the library
        ctx.set_stream(stream.cuda_stream)
        for i in range(args.warmup):
            graphs[i % n_graphs].replay()
        torch.cuda.synchronize()

    def run_step(i):
        if graphs:
            graphs[i % n_graphs].replay()
        else:
            step(i)

    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    n0 = all_launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    try:
        clk.begin()
        ev0.record(stream)
        for i in range(args.steps):
            run_step(i)
        ev1.record(stream)
        torch.cuda.synchronize()
        clk.end()
    finally:
        clk.__exit__(None, None, None)
    launches = all_launches() - n0 if not graphs else int(round(launches_per_step * args.steps))
    ms = ev0.elapsed_time(ev1)
    if pg:
        t = torch.tensor([ms], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
        pg.barrier()
    torch.cuda.synchronize()
    ms_per_step = ms / args.steps
    # tokens of the whole job per step: expert-parallel forms with replicated
    # tokens serve M; own-token forms serve M per rank (the all-to-all form's
    # shards add up to the workload's M)
    tokens_per_step = {"ep": M_total, "ep-native": M_total, "ep-a2a": M_total}.get(par, ws * M_total)
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
    if pg:
        pg.barrier()

    # End to end through the public API with pinned host buffers: the layer
    # input x goes to the device once per step (the MoE layer and q/k/v read
    # that copy), the o projection stages its own host input, and every call
    # copies its outputs back to the host (D2H) on its context's stream; the
    # calls are asynchronous (moe_set_async), the dense projections run on
    # their own contexts' streams as in the device-timed step, and the step
    # ends when the main stream has joined them.  A stack keeps its
    # activations on the device between layers.
    x_h = [x.cpu().pin_memory() for x in xs]
    xo_h = x_o.cpu().pin_memory()
    out_h = torch.empty((max(M, 1), D)).pin_memory()
    dout_h = {n: torch.empty((M, co)).pin_memory() for n, (_, _, _, co) in dense.items()}
    # the layer input x crosses once per step (the MoE layer and q/k/v read its
    # device copy); the o projection's input and every output cross as well
    h2d = M * D * 4 + sum(M * 4096 * 4 for n in dense if n == "o")
    d2h = M * D * 4 + sum(M * co * 4 for (_, _, _, co) in dense.values())
    x_d = torch.empty((max(M, 1), D), device="cuda")
    h_d = torch.empty((max(M, 1), D), device="cuda")

    def step_e2e(i):
        main = torch.cuda.current_stream()
        fork = torch.cuda.Event()
        fork.record(main)
        xh = x_h[i % n_x]
        if epl is not None:  # the torch collective needs device buffers
            x_d[:M].copy_(xh, non_blocking=True)
            moe_layer(i % args.layers, x_d[:M], out)
            out_h[:M].copy_(out[:M], non_blocking=True)
        elif stack and M > 0:  # host in, 30 layers on the device, host out
            bufs = (h_d[:M], x_d[:M])
            ctx.layer_forward(descs[0], M, xh, bufs[0], MB.F_POST_NORM)
            for li in range(1, args.layers - 1):
                moe_layer(li, bufs[(li - 1) % 2], bufs[li % 2])
            ctx.layer_forward(descs[args.layers - 1], M, bufs[(args.layers - 2) % 2], out_h[:M], MB.F_POST_NORM)
        elif stack:
            for li in range(args.layers):
                moe_layer(li, None, None)
        elif M > 0 and dense:
            # x once to the device; the layer and q/k/v read that copy
            x_d[:M].copy_(xh, non_blocking=True)
            fork.record(main)
            ctx.layer_forward(descs[i % args.layers], M, x_d[:M], out_h[:M], MB.F_POST_NORM)
        elif M > 0:
            ctx.layer_forward(descs[i % args.layers], M, xh, out_h[:M], MB.F_POST_NORM)
        else:
            moe_layer(i % args.layers, None, None)
        joins = []
        for name, (p, s, ci, co) in dense.items():
            dstream[name].wait_event(fork)
            dctx[name].q4_matmul_batchN(M, p, s, xo_h if name == "o" else x_d[:M], dout_h[name], ci, co)
            ev = torch.cuda.Event()
            ev.record(dstream[name])
            joins.append(ev)
        for ev in joins:
            main.wait_event(ev)

    e2e_steps = max(1, min(args.steps, 500))
    for i in range(3):
        step_e2e(i)
    torch.cuda.synchronize()
    # As the device-timed step, the end-to-end step replays CUDA graphs when
    # the run uses them, on one GPU: the public calls with host buffers,
    # captured with their copies from and to the pinned host buffers (each
    # replay copies that step's inputs in and its results out), as a
    # throughput-oriented caller would issue a decode loop.  With several
    # ranks (the layer call holding NCCL collectives) the capture of the
    # host-buffer calls hung a 2-rank run, so there the calls run eagerly.
    e2e_graphs = []
    if graphs and ws == 1:
        cap2 = torch.cuda.Stream()
        cap2.wait_stream(stream)
        try:
            ctx.set_stream(cap2.cuda_stream)
            for gi in range(n_graphs):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=cap2):
                    step_e2e(gi)
                e2e_graphs.append(g)
        except Exception as exc:  # capture refused: time the eager calls
            print(f"e2e graph capture failed ({exc}); timing eager calls", file=sys.stderr)
            e2e_graphs = []
        finally:
            ctx.set_stream(stream.cuda_stream)
        for i in range(3):
            if e2e_graphs:
                e2e_graphs[i % n_graphs].replay()
        torch.cuda.synchronize()
    if pg:
        pg.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(e2e_steps):
        if e2e_graphs:
            e2e_graphs[i % n_graphs].replay()
        else:
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
    Mx = M_total * ws if par == "ep-gather" else M_total  # tokens a rank's experts see
    # the dominant kernel of the MoE path (the dense projections run on their
    # own streams beside it, and their summed time is not one kernel's)
    cand = [kv for kv in prof.items() if kv[0] in ("gemv_gate_up", "gemv_down", "tc_gate_up", "tc_down")]
    dom = max(cand, key=lambda kv: kv[1][0])[0] if cand else None
    alg = {
        "gemv_gate_up": u_mean * GU_BYTES + Mx * D * 4 + pairs_mean * F * 4,
        "gemv_down": u_mean * DN_BYTES + pairs_mean * F * 4 + pairs_mean * D * 4,
        "tc_gate_up": u_mean * GU_BYTES + pairs_mean * D * 2 + pairs_mean * F * 2,
        "tc_down": u_mean * DN_BYTES + pairs_mean * F * 2 + pairs_mean * D * 4,
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
        if os.path.exists(tp) and ws == 1:
            with open(tp) as f:
                traffic = json.load(f).get(args.workload, {}).get(dom)
        roof = {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "traffic": traffic,
                "alg_bytes_per_launch": alg[dom], "avg_launch_ms": avg_ms,
                "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({'of measured' if src == 'measured' else 'of fallback'})"}
    n_lay = args.layers if stack else 1
    step_bytes = n_lay * (u_mean * (GU_BYTES + DN_BYTES) + ROUTER_BYTES + 2 * M * D * 4) + \
        sum(q4_bytes(ci, co) for (_, _, ci, co) in dense.values())
    step_roof = {"alg_bytes_per_step": step_bytes, "achieved_gbs": step_bytes / (ms_per_step / 1e3) / 1e9,
                 "frac_of_hbm": step_bytes / (ms_per_step / 1e3) / 1e9 / hbm,
                 "unique_experts_per_layer": u_mean, "pairs_per_layer": pairs_mean, "layers_per_step": n_lay,
                 "kernel_ms_per_step": {k: v[0] / args.steps for k, v in prof.items()}}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        host = synth.to_host(layers[0])
        hd = {n: (p.cpu().numpy(), s.cpu().numpy(), ci, co) for n, (p, s, ci, co) in dense.items()}
        nth = os.cpu_count() or 1
        m_cpu = min(M_total, 512)
        v, n, dt = cpu_time(host, hd, m_cpu, args.cpu_budget_s, 200, nth)
        v = v / n_lay
        tag = f"{n} steps of {m_cpu}{' of ' + str(M_total) if m_cpu < M_total else ''} tokens through layer 0"
        tag += ", + dense q/k/v/o" if hd else ""
        tag += f" in {dt:.1f} s" + (f"; rate divided by {n_lay} for the {n_lay}-layer step" if n_lay > 1 else "")
        cpu = {"value": v, "unit": "tokens/s", "cores": nth, "kind": "port", "sample": tag}

    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong" if par in ("ep", "ep-native", "ep-a2a") else "weak", "vs_baseline": None,
        "dtype": dtype_desc(args, M_total), "data": "synthetic",
        "config": dict(workload_config(args, M_total, par, ws), **({"skew": skew} if skew else {})),
        "roofline": roof, "step_roofline": step_roof,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps, "cuda_graph": bool(e2e_graphs)},
        "gpu_launches": launches, "clocks": clk.summary(),
    }
    # graphs that hold NCCL calls must be gone before the process group is
    graphs.clear()
    e2e_graphs.clear()
    import gc
    gc.collect()
    torch.cuda.synchronize()
    for c in dctx.values():
        c.close()
    if lib_ep:
        ctx.ep_finalize()
    ctx.close()
    del layers, descs, full_descs, xs
    gc.collect()
    torch.cuda.empty_cache()
    return line


if __name__ == "__main__":
    sys.exit(main())
