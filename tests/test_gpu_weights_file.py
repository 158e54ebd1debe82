"""Weights file straight to HBM on the GPU: moe_load_weights_file moves the
file's bytes exactly (whole file and a sub-range at a layer offset), and a
layer descriptor built from the loaded image (moe_layer_desc_from_weights)
evaluates the MoE layer bit for bit like the same tensors uploaded one by
one.  The file has the reference's MoE dimensions (d 2816, F 704, top-8)
with 32 experts and small attention / shared-MLP shapes, two layers."""
import os
import time

import numpy as np
import pytest

import moe_b200 as MB
import synth
import weights_file as W

pytestmark = pytest.mark.gpu

CFG = dict(W.DEFAULT_CONFIG, standard_mlp_dim=64, num_experts=32, num_layers=2, num_heads=1,
           head_dim_sliding=64, kv_heads_sliding=1, head_dim_global=128, kv_heads_global=1)


@pytest.fixture(scope="module")
def weights(tmp_path_factory):
    rng = np.random.default_rng(11)
    layers = [W.random_quantized_layer(CFG, l, rng) for l in range(CFG["num_layers"])]
    path = str(tmp_path_factory.mktemp("wf") / "gemma4_moe_weights_q4.bin")
    n = W.write_weights_file(path, layers)
    assert n == W.file_size(CFG)
    return path, layers


def test_whole_file_and_a_layer_range_arrive_intact(ctx, weights):
    import torch
    path, _ = weights
    cfg = MB.default_model_config(**CFG)
    host = torch.from_numpy(np.fromfile(path, np.uint8))
    buf, descs = MB.load_weights_file(ctx, path, cfg)
    # the second load reuses the context's pinned staging buffers
    t0 = time.perf_counter()
    n = ctx.load_weights_file(path, buf)
    dt = time.perf_counter() - t0
    assert n == host.numel()
    print(f"loaded {n / 1e6:.1f} MB in {dt * 1e3:.1f} ms ({n / dt / 1e9:.2f} GB/s, page-cached file)")
    assert len(descs) == CFG["num_layers"]
    assert torch.equal(buf.cpu(), host)
    L1 = MB.weights_layout(cfg, 1)
    part = torch.zeros(L1.layer_bytes + 4096, dtype=torch.uint8, device="cuda")
    n = ctx.load_weights_file(path, part[4096:], L1.layer_offset, L1.layer_bytes)
    assert n == L1.layer_bytes
    assert torch.equal(part[4096:].cpu(), host[L1.layer_offset:L1.layer_offset + L1.layer_bytes])
    assert not part[:4096].any()


def test_load_errors_are_reported(ctx, weights):
    import torch
    path, _ = weights
    size = os.path.getsize(path)
    small = torch.empty(4096, dtype=torch.uint8, device="cuda")
    with pytest.raises(MB.MoeError) as e:
        ctx.load_weights_file(path, small, size - 100, 200)  # past the end of the file
    assert e.value.code == 2
    with pytest.raises(MB.MoeError) as e:
        ctx.load_weights_file(path + ".missing", small, 0, 16)
    assert e.value.code == 1
    with pytest.raises(MB.MoeError) as e:
        ctx.load_weights_file(path, np.zeros(4096, np.uint8), 0, 16)  # host destination
    assert e.value.code == 1
    # a range larger than the destination's allocation is refused before
    # anything is copied (the check sees the allocator's whole block, so the
    # range here exceeds any block a 4 KiB tensor can sit in)
    assert size > 64 << 20
    with pytest.raises(MB.MoeError) as e:
        ctx.load_weights_file(path, small, 0, size)
    assert e.value.code == 2


@pytest.mark.parametrize("M", [1, 16, 200])
def test_layer_from_the_loaded_image_matches_uploaded_tensors(ctx, weights, M):
    import torch
    path, layers = weights
    cfg = MB.default_model_config(**CFG)
    buf, descs = MB.load_weights_file(ctx, path, cfg)
    for layer in range(CFG["num_layers"]):
        q = layers[layer]
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
        w = dict(d=CFG["embed_dim"], F=CFG["expert_mlp_dim"], E=CFG["num_experts"], top_k=CFG["top_k"],
                 router_p=dev(q["router"][0]), router_s=dev(q["router"][1]),
                 router_scale=dev(q["router_scale"]), per_expert_scale=dev(q["router_per_expert_scale"]),
                 pre_norm_w=dev(q["pre_feedforward_layernorm_2"]),
                 post_norm_w=dev(q["post_feedforward_layernorm_2"]),
                 gu_p=dev(q["experts_gate_up"][0]), gu_s=dev(q["experts_gate_up"][1]),
                 dn_p=dev(q["experts_down"][0]), dn_s=dev(q["experts_down"][1]))
        x = synth.make_x(M, seed=300 + M + layer)
        a = torch.zeros((M, CFG["embed_dim"]), device="cuda")
        b = torch.zeros_like(a)
        ctx.layer_forward(descs[layer], M, x, a, MB.F_POST_NORM)
        ctx.layer_forward(MB.make_desc(w), M, x, b, MB.F_POST_NORM)
        torch.cuda.synchronize()
        assert torch.isfinite(a).all()
        assert float(a.abs().max()) > 0
        assert torch.equal(a, b), f"layer {layer} M={M}"
