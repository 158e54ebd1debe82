"""CPU restatement of the weights-file format (gemma4_moe_weights_q4.bin).

TEST INFRASTRUCTURE ONLY.  Imported by tests/ as the checker of the
library's weights-file layout and loader; the product package never imports
this module.

Writer: convert_gemma4_moe.py:164-262 -- per layer, the Q4_0 packed bytes of
the ten matrices in file order, then their fp32 scales in the same order,
then twelve fp32 vectors, zero-padded to a multiple of 4096 bytes; layers
back to back, no header.  Its quantizer is convert_gemma4_moe.py:9-35.
Reader: MoEConfig.get_layer_aligned_size / get_layer_offset /
get_layer_weights, model_speculative_moe_batched.mojo:57-231.

Configurations are plain dicts with the field names of moe_model_config
(include/moe_b200.h).
"""
from __future__ import annotations

import numpy as np

BLOB_ALIGN = 4096

# file order of the matrices (convert_gemma4_moe.py:192-203) with the
# safetensors names the converter loads them from (:172-189)
MATRICES = (
    ("q_proj", "self_attn.q_proj.weight"),
    ("k_proj", "self_attn.k_proj.weight"),
    ("v_proj", "self_attn.v_proj.weight"),
    ("o_proj", "self_attn.o_proj.weight"),
    ("gate_proj", "mlp.gate_proj.weight"),
    ("up_proj", "mlp.up_proj.weight"),
    ("down_proj", "mlp.down_proj.weight"),
    ("router", "router.proj.weight"),
    ("experts_gate_up", "experts.gate_up_proj"),
    ("experts_down", "experts.down_proj"),
)
# file order of the fp32 vectors (convert_gemma4_moe.py:218-246)
VECTORS = (
    ("input_layernorm", "input_layernorm.weight"),
    ("post_attention_layernorm", "post_attention_layernorm.weight"),
    ("pre_feedforward_layernorm", "pre_feedforward_layernorm.weight"),
    ("pre_feedforward_layernorm_2", "pre_feedforward_layernorm_2.weight"),
    ("post_feedforward_layernorm", "post_feedforward_layernorm.weight"),
    ("post_feedforward_layernorm_1", "post_feedforward_layernorm_1.weight"),
    ("post_feedforward_layernorm_2", "post_feedforward_layernorm_2.weight"),
    ("q_norm", "self_attn.q_norm.weight"),
    ("k_norm", "self_attn.k_norm.weight"),
    ("router_scale", "router.scale"),
    ("router_per_expert_scale", "router.per_expert_scale"),
    ("layer_scalar", "layer_scalar"),
)

DEFAULT_CONFIG = dict(embed_dim=2816, standard_mlp_dim=2112, expert_mlp_dim=704, num_experts=128,
                      top_k=8, num_layers=30, num_heads=16, head_dim_sliding=256,
                      kv_heads_sliding=8, head_dim_global=512, kv_heads_global=2, global_every=6)

# The small model the golden weights file was made from (30 layers: the
# converter's fixed layer count).
TINY_CONFIG = dict(embed_dim=64, standard_mlp_dim=64, expert_mlp_dim=32, num_experts=8, top_k=2,
                   num_layers=30, num_heads=2, head_dim_sliding=32, kv_heads_sliding=2,
                   head_dim_global=64, kv_heads_global=1, global_every=6)


def is_global(cfg: dict, layer: int) -> bool:
    """model_speculative_moe_batched.mojo:52-54 (layer % 6 == 5)."""
    return layer % cfg["global_every"] == cfg["global_every"] - 1


def tensor_shapes(cfg: dict, layer: int) -> dict:
    """Shapes of every tensor of a layer as the converter reads them; the
    matrices' last axis is the inner (Q4_0 block) dimension.  v_proj is
    absent ((0,)) on global layers (convert_gemma4_moe.py:175-178)."""
    d, S, F, E, H = (cfg[k] for k in ("embed_dim", "standard_mlp_dim", "expert_mlp_dim",
                                       "num_experts", "num_heads"))
    g = is_global(cfg, layer)
    hd = cfg["head_dim_global"] if g else cfg["head_dim_sliding"]
    kv = cfg["kv_heads_global"] if g else cfg["kv_heads_sliding"]
    return {
        "q_proj": (H * hd, d), "k_proj": (kv * hd, d), "v_proj": (0,) if g else (kv * hd, d),
        "o_proj": (d, H * hd), "gate_proj": (S, d), "up_proj": (S, d), "down_proj": (d, S),
        "router": (E, d), "experts_gate_up": (E, 2 * F, d), "experts_down": (E, d, F),
        "input_layernorm": (d,), "post_attention_layernorm": (d,),
        "pre_feedforward_layernorm": (d,), "pre_feedforward_layernorm_2": (d,),
        "post_feedforward_layernorm": (d,), "post_feedforward_layernorm_1": (d,),
        "post_feedforward_layernorm_2": (d,), "q_norm": (hd,), "k_norm": (hd,),
        "router_scale": (d,), "router_per_expert_scale": (E,), "layer_scalar": (1,),
    }


def layer_layout(cfg: dict, layer: int) -> dict:
    """Byte offsets of one layer's tensors within its blob, the blob's size
    and its offset in the file (model_speculative_moe_batched.mojo:57-231)."""
    def blob(l):
        shp = tensor_shapes(cfg, l)
        elems = [int(np.prod(shp[n])) for n, _ in MATRICES]
        packed, scales, off = {}, {}, 0
        for (n, _), e in zip(MATRICES, elems):
            packed[n] = off
            off += e // 2
        for (n, _), e in zip(MATRICES, elems):
            scales[n] = off
            off += e // 32 * 4
        vec = {}
        for n, _ in VECTORS:
            vec[n] = off
            off += int(np.prod(shp[n])) * 4
        return dict(packed=packed, scales=scales, vec=vec, payload=off,
                    bytes=(off + BLOB_ALIGN - 1) // BLOB_ALIGN * BLOB_ALIGN, shapes=shp)
    out = blob(layer)
    out["offset"] = sum(blob(l)["bytes"] for l in range(layer))
    return out


def file_size(cfg: dict) -> int:
    last = layer_layout(cfg, cfg["num_layers"] - 1)
    return last["offset"] + last["bytes"]


def quantize(x: np.ndarray):
    """convert_gemma4_moe.py:9-35 with its numpy arithmetic: per block of 32,
    scale = max(max|x| / 7, 1e-5) in fp32, q = clip(round(x * (1 / scale)),
    -8, 7) rounding half to even, stored as q + 8, even element in the low
    nibble.  Returns (packed uint8, scales fp32), both flat."""
    b = np.asarray(x, np.float32).reshape(-1, 32)
    scale = np.maximum(np.abs(b).max(axis=1) / 7.0, 1e-5)
    inv = 1.0 / scale
    q = np.clip(np.round(b * inv[:, None]), -8, 7).astype(np.int8)
    u = (q + 8).astype(np.uint8)
    return (u[:, 0::2] | (u[:, 1::2] << 4)).reshape(-1), scale.astype(np.float32).reshape(-1)


def tiny_model(cfg: dict, seed: int) -> list:
    """Seeded fp32 tensors of every layer, keyed by short name: matrices
    N(0, 0.02), norms 1 + N(0, 0.1), router_scale / per_expert_scale
    around 1, layer_scalar 0.5 + layer / 100."""
    rng = np.random.default_rng(seed)
    layers = []
    for l in range(cfg["num_layers"]):
        shp = tensor_shapes(cfg, l)
        t = {}
        for n, _ in MATRICES:
            t[n] = (rng.standard_normal(shp[n]) * 0.02).astype(np.float32)
        for n, _ in VECTORS:
            t[n] = (1.0 + 0.1 * rng.standard_normal(shp[n])).astype(np.float32)
        t["layer_scalar"] = np.array([0.5 + l / 100], np.float32)
        layers.append(t)
    return layers


def quantized_layer(t: dict) -> dict:
    """Float tensors of a layer -> {matrix: (packed, scales), vector: fp32}."""
    out = {}
    for n, _ in MATRICES:
        out[n] = quantize(t[n]) if t[n].size else (np.zeros(0, np.uint8), np.zeros(0, np.float32))
    for n, _ in VECTORS:
        out[n] = np.ascontiguousarray(t[n], np.float32).reshape(-1)
    return out


def layer_blob(q: dict) -> bytes:
    """One layer's bytes (convert_gemma4_moe.py:205-254)."""
    payload = b"".join(q[n][0].tobytes() for n, _ in MATRICES)
    payload += b"".join(q[n][1].tobytes() for n, _ in MATRICES)
    payload += b"".join(q[n].tobytes() for n, _ in VECTORS)
    pad = (-len(payload)) % BLOB_ALIGN
    return payload + b"\0" * pad


def write_weights_file(path, quantized_layers: list) -> int:
    """Writes the layers' blobs back to back; returns the file size."""
    n = 0
    with open(path, "wb") as f:
        for q in quantized_layers:
            b = layer_blob(q)
            f.write(b)
            n += len(b)
    return n


def random_quantized_layer(cfg: dict, layer: int, rng) -> dict:
    """A layer with arbitrary Q4_0 content, already quantized (uniform
    nibbles, scales 0.002-0.006, norms 1 + N(0, 0.1), router scales 1):
    large-model files without a float round trip."""
    shp = tensor_shapes(cfg, layer)
    out = {}
    for n, _ in MATRICES:
        e = int(np.prod(shp[n]))
        out[n] = (rng.integers(0, 256, e // 2, dtype=np.uint8),
                  rng.uniform(0.002, 0.006, e // 32).astype(np.float32))
    for n, _ in VECTORS:
        out[n] = (1.0 + 0.1 * rng.standard_normal(int(np.prod(shp[n])))).astype(np.float32)
    out["router_scale"][:] = 1.0
    out["router_per_expert_scale"][:] = 1.0
    return out
