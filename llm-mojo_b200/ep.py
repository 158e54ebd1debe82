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
