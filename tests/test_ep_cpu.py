"""Expert parallelism, host side, on CPU: two gloo ranks each evaluate their
contiguous expert range with the oracle and all-reduce the partial outputs;
the sum must equal the one-process result.  No GPU is involved."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

import ep


def test_expert_ranges_partition_all_experts():
    for world in (1, 2, 3, 4, 8):
        seen = []
        for r in range(world):
            lo, hi = ep.expert_range(r, world, 128)
            assert lo <= hi
            seen.extend(range(lo, hi))
        assert seen == list(range(128))
    assert ep.expert_range(7, 8, 128) == (112, 128)
    with pytest.raises(ValueError):
        ep.expert_range(2, 2, 128)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _layer(d, F, E, K, seed):
    import oracle as O
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


def _worker(rank, world, port, q):
    try:
        import torch
        import torch.distributed as dist
        import oracle as O
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        d, F, E, K, M = 256, 64, 16, 4, 6
        w = _layer(d, F, E, K, seed=11)
        L = O.make_layer(w)
        x = np.random.default_rng(12).standard_normal((M, d)).astype(np.float32)
        r = O.route(L, x)
        lo, hi = ep.expert_range(rank, world, E)
        local = (r["idx"] >= lo) & (r["idx"] < hi)
        w_local = np.where(local, r["w"], 0.0).astype(np.float32)
        part = O.experts_forward(L, r["moe_in"], r["count"], r["idx"], w_local, prec=O.F64)
        t = torch.from_numpy(part.astype(np.float64))
        dist.all_reduce(t)
        full = O.experts_forward(L, r["moe_in"], r["count"], r["idx"], r["w"], prec=O.F64)
        err = float(np.max(np.abs(t.numpy() - full)))
        # post-norm after the reduction, as ep.ExpertParallelLayer applies it
        s = t.numpy()
        normed = s / np.sqrt((s ** 2).mean(1, keepdims=True) + 1e-6)
        ref, _, _, _ = O.layer_forward(L, x, post_norm=True, prec=O.F64)
        err_norm = float(np.max(np.abs(normed - ref)))
        n_local = int(local.sum())
        dist.destroy_process_group()
        q.put((rank, err, err_norm, n_local))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e), None, None))


def test_two_gloo_ranks_reproduce_the_full_layer():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    for rank, err, err_norm, n_local in res:
        assert not isinstance(err, str), err
        assert err < 1e-6 and err_norm < 1e-5, (rank, err, err_norm)
    assert res[0][3] + res[1][3] > 0


def _a2a_worker(rank, world, port, q, M, dedup=False):
    """All-to-all expert parallelism on gloo ranks: tokens sharded over the
    ranks, routed rows dispatched to the owners of their experts and the
    results returned; route and expert evaluation by the oracle."""
    try:
        import torch
        import torch.distributed as dist
        import oracle as O
        import datetime
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        d, F, E, K = 256, 64, 16, 4
        L = O.make_layer(_layer(d, F, E, K, seed=21))
        x_all = np.random.default_rng(22).standard_normal((M, d)).astype(np.float32)
        t0, t1 = ep.row_range(rank, world, M)
        x = x_all[t0:t1]
        lo, hi = ep.expert_range(rank, world, E)

        def route_fn(xt):
            m = xt.shape[0]
            if m == 0:
                return (torch.zeros(0, dtype=torch.int64), torch.zeros((0, K), dtype=torch.int64),
                        torch.zeros((0, K)), torch.zeros((0, d)))
            r = O.route(L, xt.numpy())
            return (torch.from_numpy(r["count"]), torch.from_numpy(r["idx"]), torch.from_numpy(r["w"]),
                    torch.from_numpy(r["moe_in"]))

        def experts_fn(rows, local_ids, weights=None, count=None):
            n = rows.shape[0]
            if n == 0:
                return torch.zeros((0, d))
            if dedup:  # each row's leading `count` slots, weighted
                gidx = local_ids.numpy() + lo
                c = count.numpy()
                for r in range(n):
                    assert ((gidx[r, :c[r]] >= lo) & (gidx[r, :c[r]] < hi)).all()
                y = O.experts_forward(L, rows.numpy(), c.astype(np.int64), gidx.astype(np.int64),
                                      weights.numpy().astype(np.float32), prec=O.F64)
                return torch.from_numpy(y)
            idx = np.zeros((n, K), np.int64)
            idx[:, 0] = local_ids.numpy() + lo
            assert ((idx[:, 0] >= lo) & (idx[:, 0] < hi)).all()
            wt = np.zeros((n, K), np.float32)
            wt[:, 0] = 1.0
            y = O.experts_forward(L, rows.numpy(), np.ones(n, np.int64), idx, wt, prec=O.F64)
            return torch.from_numpy(y)

        layer = ep.AllToAllExpertParallelLayer(E, route_fn, experts_fn, dedup=dedup)
        sent = []  # rows of every exchange this rank sends
        exchange = layer._exchange
        layer._exchange = lambda send, sc, rc: (sent.append(int(sum(sc))), exchange(send, sc, rc))[1]
        ones = torch.ones(d)
        out = layer.forward(torch.from_numpy(x), post_norm_w=ones).numpy()
        m = t1 - t0
        pairs = int(O.route(L, x)["count"].sum()) if m else 0
        rows = sent[0]  # the dispatch of the activation rows
        assert rows <= pairs
        if dedup:
            assert rows <= m * world
        else:
            assert rows == pairs
        ref, _, _, _ = O.layer_forward(L, x_all, post_norm=True, prec=O.F64)
        err = float(np.max(np.abs(out - ref[t0:t1]))) if t1 > t0 else 0.0
        dist.destroy_process_group()
        q.put((rank, err, t1 - t0))
    except Exception as e:  # reported to the parent
        import traceback
        q.put((rank, traceback.format_exc(), None))


@pytest.mark.parametrize("dedup", [False, True], ids=["per-pair", "per-token"])
@pytest.mark.parametrize("world,M", [(2, 7), (3, 2)])
def test_all_to_all_ranks_reproduce_the_full_layer(world, M, dedup):
    """Uneven token shards (7 over 2 ranks; 2 over 3, one rank without
    tokens): the dispatched, evaluated and combined output equals the
    one-process layer, with one row per routed pair or (dedup) one row per
    token and destination rank."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_a2a_worker, args=(r, world, port, q, M, dedup)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, m in res:
        assert not isinstance(err, str), err
        assert err < 1e-5, (rank, err)
    assert sum(m for _, _, m in res) == M


def test_expert_owner_matches_expert_range():
    import torch
    for world in (1, 2, 3, 8):
        e = torch.arange(128)
        own = ep.expert_owner(e, world, 128)
        for r in range(world):
            lo, hi = ep.expert_range(r, world, 128)
            assert (own[lo:hi] == r).all()


class _OracleCtx:
    """Stands in for moe_b200.Context on CPU: the three calls make_library_fns
    makes (route, run_moe_coalesced_core, rms_norm) evaluated by the oracle on
    CPU tensors, with the library's argument meaning."""

    def __init__(self, L):
        self.L = L

    def route(self, desc, M, x, count, idx, w, moe_in=None):
        import oracle as O
        import torch
        r = O.route(self.L, x.numpy())
        count.copy_(torch.from_numpy(r["count"]))
        idx.copy_(torch.from_numpy(r["idx"]))
        w.copy_(torch.from_numpy(r["w"]))
        moe_in.copy_(torch.from_numpy(r["moe_in"]))

    def run_moe_coalesced_core(self, n, gu_p, gu_s, dn_p, dn_s, rows, cnt, idx, wt, out, embed_dim,
                               expert_mlp_dim, num_experts, x_layout, top_k):
        import oracle as O
        import torch
        import moe_b200 as MB
        assert x_layout == MB.X_NATURAL and idx.shape == (n, top_k)
        for r in range(n):
            assert (idx[r, :cnt[r]] >= 0).all() and (idx[r, :cnt[r]] < num_experts).all()
        sub = dict(d=embed_dim, F=expert_mlp_dim, E=num_experts, top_k=top_k,
                   gu_p=np.ascontiguousarray(gu_p), gu_s=np.ascontiguousarray(gu_s),
                   dn_p=np.ascontiguousarray(dn_p), dn_s=np.ascontiguousarray(dn_s))
        for k in ("router_scale", "pre_norm_w", "post_norm_w"):
            sub[k] = np.ones(embed_dim, np.float32)
        sub["per_expert_scale"] = np.ones(num_experts, np.float32)
        y = O.experts_forward(O.make_layer(sub), rows.numpy(), cnt.numpy(), idx.numpy(), wt.numpy(),
                              prec=O.F64)
        out.copy_(torch.from_numpy(y))

    def rms_norm(self, x, w, out, M, d):
        x64 = x.double()
        out.copy_((x64 / (x64.pow(2).mean(1, keepdim=True) + 1e-6).sqrt() * w.double()).float())


def _lib_worker(rank, world, port, q, dedup=False):
    """make_library_fns' weight slices and calls, through the oracle stand-in."""
    try:
        import torch
        import torch.distributed as dist
        import oracle as O
        import datetime
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        d, F, E, K, M = 256, 64, 16, 4, 9
        w = _layer(d, F, E, K, seed=31)
        L = O.make_layer(w)
        x_all = np.random.default_rng(32).standard_normal((M, d)).astype(np.float32)
        t0, t1 = ep.row_range(rank, world, M)
        route_fn, experts_fn, rms_norm_fn = ep.make_library_fns(_OracleCtx(L), None, w, rank, world)
        layer = ep.AllToAllExpertParallelLayer(E, route_fn, experts_fn, rms_norm_fn=rms_norm_fn, dedup=dedup)
        out = layer.forward(torch.from_numpy(x_all[t0:t1].copy()), post_norm_w=torch.ones(d)).numpy()
        ref, _, _, _ = O.layer_forward(L, x_all, post_norm=True, prec=O.F64)
        err = float(np.max(np.abs(out - ref[t0:t1]))) if t1 > t0 else 0.0
        dist.destroy_process_group()
        q.put((rank, err, t1 - t0))
    except Exception:  # reported to the parent
        import traceback
        q.put((rank, traceback.format_exc(), None))


@pytest.mark.parametrize("dedup", [False, True], ids=["per-pair", "per-token"])
def test_all_to_all_library_functions_slice_the_weights(dedup):
    """make_library_fns hands each rank's expert slice and local ids (and,
    per token, the local slot lists and weights) to the coalesced core; with
    the oracle behind the calls, three ranks reproduce the one-process
    layer."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_lib_worker, args=(r, 3, port, q, dedup)) for r in range(3)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, m in res:
        assert not isinstance(err, str), err
        assert err < 1e-5, (rank, err)
