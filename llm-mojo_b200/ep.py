"""Expert parallelism for the MoE layer over torch.distributed.

One process per GPU.  Every rank holds the whole (replicated) router and the
experts of one contiguous range, 128/N of them; the tokens of a decode step
are replicated.  A layer step is:

    route all experts locally -> evaluate the local experts' (token, slot)
    pairs -> per-token weighted sum over the local slots (a partial output)
    -> all-reduce of the partial outputs (NCCL over NVLink) -> post-norm

The sum over ranks replaces the reference's single in-order sum over a
token's slots (moe_kernels.mojo:775-779), so results equal the one-GPU
output up to fp32 reassociation.  torch.distributed carries the collective;
the library (libmoe_b200) evaluates only the experts of the range set with
Context.set_expert_range.
"""
from __future__ import annotations

import moe_b200 as MB


def expert_range(rank: int, world: int, num_experts: int) -> tuple[int, int]:
    """Contiguous expert range of `rank`: [rank*E/N, (rank+1)*E/N)."""
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    return rank * num_experts // world, (rank + 1) * num_experts // world


def row_range(rank: int, world: int, rows: int) -> tuple[int, int]:
    """Contiguous row slice of a dense projection for `rank`."""
    return rank * rows // world, (rank + 1) * rows // world


class ExpertParallelLayer:
    """Runs moe_layer_forward with this rank's experts and reduces the partial
    outputs over the process group."""

    def __init__(self, ctx: "MB.Context", num_experts: int, group=None):
        import torch.distributed as dist
        self.ctx = ctx
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.begin, self.end = expert_range(self.rank, self.world, num_experts)

    def forward(self, desc, M: int, x, out, flags: int = MB.F_POST_NORM, post_norm_w=None):
        """x: [M, d] (device tensor, the same on every rank); out: [M, d] fp32
        device tensor.  With MB.F_POST_NORM the post-norm weights come from
        `post_norm_w` (device tensor [d])."""
        self.ctx.set_expert_range(self.begin, self.end)
        try:
            self.ctx.layer_forward(desc, M, x, out, flags & ~MB.F_POST_NORM)
        finally:
            self.ctx.set_expert_range(0, 0)
        if self.world > 1:
            self.dist.all_reduce(out, group=self.group)
        if flags & MB.F_POST_NORM:
            if post_norm_w is None:
                raise ValueError("post-norm needs post_norm_w")
            d = out.shape[-1]
            self.ctx.rms_norm(out, post_norm_w, out, M, d)
        return out


def expert_owner(e, world: int, num_experts: int):
    """Rank owning expert id(s) `e` under expert_range (torch tensor of ids)."""
    import torch
    starts = torch.tensor([expert_range(r, world, num_experts)[0] for r in range(world)], device=e.device)
    return torch.searchsorted(starts, e, right=True) - 1


class AllToAllExpertParallelLayer:
    """Expert parallelism with the tokens sharded over the ranks (the large-M
    form: configs with thousands of routed tokens).  Each rank holds the
    experts of expert_range(rank) and its own tokens; a layer step is:

        route the local tokens -> send every routed (token, slot) row to the
        rank that owns the slot's expert (all-to-all) -> evaluate the received
        rows, one expert each -> send the results back (all-to-all) ->
        per-token weighted sum over the token's slots, in slot order -> post-norm

    The weighted sum runs at the token's home rank in slot order, as the
    reference's per-token accumulation does (moe_kernels.mojo:775-779).

    With dedup=True a token travels once to each rank that owns any of its
    experts, with that rank's slots (local expert ids and weights, in slot
    order); the rank returns one weighted partial sum per token, and the home
    rank adds the partial sums in rank order.  That moves min(K, ranks
    touched) rows per token each way instead of K, and equals the slot-order
    sum within fp32 reassociation (as the all-reduce form does).

    route_fn(x) -> (count [m], idx [m, K] global expert ids, w [m, K],
    moe_in [m, d]) and experts_fn are supplied by the caller: with the
    library they are Context.route and Context.run_moe_coalesced_core over
    this rank's weight slice (make_library_fns); the CPU tests pass the
    oracle.  experts_fn(rows [n, d], local_ids [n]) -> [n, d] returns the
    unweighted expert outputs (one expert per row); with dedup,
    experts_fn(rows [n, d], local_idx [n, K], weights [n, K], count [n]) ->
    [n, d] returns each row's weighted sum over its `count` leading slots.
    """

    def __init__(self, num_experts: int, route_fn, experts_fn, *, group=None, rms_norm_fn=None,
                 dedup: bool = False):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.E = num_experts
        self.begin, self.end = expert_range(self.rank, self.world, num_experts)
        self.route_fn = route_fn
        self.experts_fn = experts_fn
        self.rms_norm_fn = rms_norm_fn
        self.dedup = dedup

    def _exchange(self, send, send_counts, recv_counts):
        import torch
        recv = torch.empty((int(sum(recv_counts)),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        self.dist.all_to_all_single(recv, send.contiguous(), output_split_sizes=recv_counts,
                                    input_split_sizes=send_counts, group=self.group)
        return recv

    def _starts(self, dev):
        import torch
        return torch.tensor([expert_range(r, self.world, self.E)[0] for r in range(self.world)], device=dev)

    def _exchange_counts(self, dest_sorted):
        import torch
        send_counts = torch.bincount(dest_sorted, minlength=self.world)
        recv_counts = torch.empty_like(send_counts)
        self.dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        return send_counts.tolist(), recv_counts.tolist()

    def _forward_tokens(self, count, idx, w, moe_in):
        """dedup: one row per (token, rank owning one of its experts)."""
        import torch
        m, K = idx.shape
        d = moe_in.shape[1]
        dev = moe_in.device
        slot = torch.arange(K, device=dev).unsqueeze(0)
        active = slot < count.unsqueeze(1)
        owner = torch.where(active, expert_owner(idx.long().clamp(0, self.E - 1), self.world, self.E),
                            torch.full_like(idx, -1, dtype=torch.long))
        has = torch.zeros((m, self.world), dtype=torch.bool, device=dev)
        t_a, k_a = torch.nonzero(active, as_tuple=True)
        has[t_a, owner[t_a, k_a]] = True
        t_idx, r_idx = torch.nonzero(has, as_tuple=True)  # token order, then rank
        dest_sorted, order = torch.sort(r_idx, stable=True)
        t_sorted = t_idx[order]
        # this rank's slots of each (token, rank) row, compacted in slot order
        mask = owner[t_sorted] == dest_sorted.unsqueeze(1)  # [n, K]
        pos = torch.cumsum(mask.long(), 1) - 1
        lcnt = mask.sum(1)
        lidx = torch.zeros((len(t_sorted), K), dtype=torch.long, device=dev)
        lw = torch.zeros((len(t_sorted), K), dtype=torch.float32, device=dev)
        ri, ci = torch.nonzero(mask, as_tuple=True)
        lidx[ri, pos[ri, ci]] = idx[t_sorted][ri, ci].long() - self._starts(dev)[dest_sorted][ri]
        lw[ri, pos[ri, ci]] = w[t_sorted][ri, ci].to(torch.float32)
        sc, rc = self._exchange_counts(dest_sorted)
        rows = self._exchange(moe_in[t_sorted], sc, rc)
        r_cnt = self._exchange(lcnt, sc, rc)
        r_idx2 = self._exchange(lidx, sc, rc)
        r_w = self._exchange(lw, sc, rc)
        y = self.experts_fn(rows, r_idx2, r_w, r_cnt)
        back = self._exchange(y, rc, sc)
        out = torch.zeros((m, d), dtype=torch.float32, device=dev)
        for r in range(self.world):  # rank order; each token at most once per rank
            sel = dest_sorted == r
            if bool(sel.any()):
                out.index_add_(0, t_sorted[sel], back[sel])
        return out

    def forward(self, x, post_norm_w=None):
        """x: this rank's tokens [m, d] fp32 (m may be 0).  Returns [m, d]."""
        import torch
        count, idx, w, moe_in = self.route_fn(x)
        if self.dedup:
            out = self._forward_tokens(count, idx, w, moe_in)
            return self._post_norm(out, post_norm_w)
        m, K = idx.shape
        d = moe_in.shape[1]
        dev = moe_in.device
        slot = torch.arange(K, device=dev).unsqueeze(0)
        t_idx, k_idx = torch.nonzero(slot < count.unsqueeze(1), as_tuple=True)  # token order, slot order
        e = idx[t_idx, k_idx].long()
        dest = expert_owner(e, self.world, self.E)
        dest_sorted, order = torch.sort(dest, stable=True)
        send_counts = torch.bincount(dest_sorted, minlength=self.world)
        recv_counts_t = torch.empty_like(send_counts)
        self.dist.all_to_all_single(recv_counts_t, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts_t.tolist()
        starts = torch.tensor([expert_range(r, self.world, self.E)[0] for r in range(self.world)], device=dev)
        rows = self._exchange(moe_in[t_idx[order]], sc, rc)
        local_ids = self._exchange(e[order] - starts[dest_sorted], sc, rc)
        y = self.experts_fn(rows, local_ids)
        back = self._exchange(y, rc, sc)
        y_pairs = torch.empty_like(back)
        y_pairs[order] = back
        out = torch.zeros((m, d), dtype=torch.float32, device=dev)
        wp = w[t_idx, k_idx].to(torch.float32)
        for k in range(K):  # slot order
            sel = k_idx == k
            if bool(sel.any()):
                out.index_add_(0, t_idx[sel], y_pairs[sel] * wp[sel].unsqueeze(1))
        return self._post_norm(out, post_norm_w)

    def _post_norm(self, out, post_norm_w):
        import torch
        if post_norm_w is not None:
            if self.rms_norm_fn is not None:
                self.rms_norm_fn(out, post_norm_w, out)
            else:
                out = out * torch.rsqrt((out * out).mean(1, keepdim=True) + 1e-6) * post_norm_w
        return out


def make_library_fns(ctx: "MB.Context", desc, layer: dict, rank: int, world: int):
    """route_fn / experts_fn / rms_norm_fn for AllToAllExpertParallelLayer
    over the library: routing with Context.route, the received rows through
    Context.run_moe_coalesced_core (one active slot of weight 1 per row) with
    the weights of this rank's experts, which the caller keeps resident."""
    import torch
    d, F, E, K = layer["d"], layer["F"], layer["E"], layer["top_k"]
    lo, hi = expert_range(rank, world, E)
    gu = d * F            # packed bytes of one expert's 2F x d gate/up rows
    gs = 2 * F * d // 32  # its scales
    dn = d * F // 2
    ds = d * F // 32
    gu_p = layer["gu_p"][lo * gu:hi * gu]
    gu_s = layer["gu_s"][lo * gs:hi * gs]
    dn_p = layer["dn_p"][lo * dn:hi * dn]
    dn_s = layer["dn_s"][lo * ds:hi * ds]

    def route_fn(x):
        m = x.shape[0]
        count = torch.empty(m, dtype=torch.int64, device=x.device)
        idx = torch.empty((m, K), dtype=torch.int64, device=x.device)
        w = torch.empty((m, K), dtype=torch.float32, device=x.device)
        moe_in = torch.empty((m, d), dtype=torch.float32, device=x.device)
        if m:
            ctx.route(desc, m, x, count, idx, w, moe_in=moe_in)
        return count, idx, w, moe_in

    def experts_fn(rows, local_ids, weights=None, count=None):
        n = rows.shape[0]
        out = torch.empty((n, d), dtype=torch.float32, device=rows.device)
        if not n:
            return out
        if local_ids.dim() == 1:  # one expert per row, weight 1
            cnt = torch.ones(n, dtype=torch.int64, device=rows.device)
            wt = torch.ones((n, 1), dtype=torch.float32, device=rows.device)
            ids, k = local_ids.reshape(n, 1), 1
        else:  # dedup: each row's leading `count` slots, weighted
            cnt, wt, ids, k = count.to(torch.int64), weights, local_ids, local_ids.shape[1]
        ctx.run_moe_coalesced_core(n, gu_p, gu_s, dn_p, dn_s, rows.contiguous(), cnt.contiguous(),
                                   ids.to(torch.int64).contiguous(), wt.to(torch.float32).contiguous(), out,
                                   embed_dim=d, expert_mlp_dim=F, num_experts=hi - lo,
                                   x_layout=MB.X_NATURAL, top_k=k)
        return out

    def rms_norm_fn(x, w, out):
        if x.shape[0]:
            ctx.rms_norm(x, w, out, x.shape[0], d)

    return route_fn, experts_fn, rms_norm_fn
