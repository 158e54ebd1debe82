"""Seeded synthetic MoE layers and activations at the reference's shapes.

There are no real Gemma-4 weights on these hosts, so every workload is drawn
from the distributions the benchmark configurations name: expert and router
weights ~ N(0, 0.02) quantised to Q4_0, activations ~ N(0, 1), norm weights,
router_scale and per_expert_scale = 1.

Weights are generated on the GPU (torch's Philox generator, seeded) and
quantised by this library's own Q4_0 kernel (bit-exact with the reference
quantizer); ``to_host`` copies a layer back for CPU-side use.
"""
from __future__ import annotations

import numpy as np

D, F, E, TOP_K = 2816, 704, 128, 8


def _torch():
    import torch
    return torch


def _randn(shape, std, gen, device):
    torch = _torch()
    return torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std


def quantize(ctx, w):
    """Q4_0-quantise a CUDA fp32 tensor with the library kernel -> (packed, scales)."""
    torch = _torch()
    w = w.contiguous().view(-1)
    packed = torch.empty(w.numel() // 2, dtype=torch.uint8, device=w.device)
    scales = torch.empty(w.numel() // 32, dtype=torch.float32, device=w.device)
    ctx.quantize_fp32_to_q4_0(w, packed, scales, w.numel())
    return packed, scales


def make_layer(ctx, d=D, F_=F, E_=E, top_k=TOP_K, seed=0, device="cuda", std=0.02,
               chunk_experts=16):
    """One MoE layer as CUDA tensors (keys used by moe_b200.make_desc)."""
    torch = _torch()
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    router_f32 = _randn((E_, d), std, gen, device)
    rp, rs = quantize(ctx, router_f32)
    gu_p = torch.empty(E_ * 2 * F_ * d // 2, dtype=torch.uint8, device=device)
    gu_s = torch.empty(E_ * 2 * F_ * d // 32, dtype=torch.float32, device=device)
    dn_p = torch.empty(E_ * d * F_ // 2, dtype=torch.uint8, device=device)
    dn_s = torch.empty(E_ * d * F_ // 32, dtype=torch.float32, device=device)
    for e0 in range(0, E_, chunk_experts):
        n = min(chunk_experts, E_ - e0)
        w = _randn((n, 2 * F_, d), std, gen, device)
        p, s = quantize(ctx, w)
        gu_p[e0 * F_ * d:(e0 + n) * F_ * d] = p
        gu_s[e0 * 2 * F_ * d // 32:(e0 + n) * 2 * F_ * d // 32] = s
        w = _randn((n, d, F_), std, gen, device)
        p, s = quantize(ctx, w)
        dn_p[e0 * d * F_ // 2:(e0 + n) * d * F_ // 2] = p
        dn_s[e0 * d * F_ // 32:(e0 + n) * d * F_ // 32] = s
        del w
    ones_d = torch.ones(d, dtype=torch.float32, device=device)
    return dict(d=d, F=F_, E=E_, top_k=top_k, router_f32=router_f32, router_p=rp, router_s=rs,
                router_scale=ones_d, per_expert_scale=torch.ones(E_, dtype=torch.float32, device=device),
                pre_norm_w=ones_d.clone(), post_norm_w=ones_d.clone(),
                gu_p=gu_p, gu_s=gu_s, dn_p=dn_p, dn_s=dn_s)


def to_host(layer: dict) -> dict:
    out = {}
    for k, v in layer.items():
        out[k] = v.detach().cpu().numpy() if hasattr(v, "detach") else v
    return out


def make_x(M, d=D, seed=1, device="cuda", bf16_representable=False):
    torch = _torch()
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    x = torch.randn((M, d), generator=gen, device=device, dtype=torch.float32)
    if bf16_representable:
        x = x.to(torch.bfloat16).to(torch.float32)
    return x


def zipf_bias(E_=E, s=1.1, alpha=1.0, seed=0):
    """Router-logit bias b_e = -alpha * s * ln(rank_e) with a seeded rank permutation
    (skewed-load workload; no counterpart in the reference, which routes unbiased)."""
    rng = np.random.default_rng(seed)
    rank = rng.permutation(E_) + 1
    return (-alpha * s * np.log(rank)).astype(np.float32)
