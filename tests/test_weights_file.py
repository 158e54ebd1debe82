"""Weights-file layout, on CPU: the library's layout functions against the
reference's own numbers and files.  No GPU call is made here.

Pins:
  * the whole-file size for the reference's configuration equals the size
    model_speculative_moe_batched.mojo:1347 hard-codes (15311790080 bytes);
  * the restated writer (oracle/weights_file.py) reproduces, byte for byte,
    the file the reference's convert_gemma4_moe.py wrote for a small seeded
    model (SHA-256 in tests/golden/weights_file_tiny.json, made by
    tests/golden/gen_weights_file_golden.py);
  * the library's layout finds every tensor of that file where the
    converter put it.
"""
import ctypes as C
import hashlib
import json
import os

import numpy as np
import pytest

import moe_b200 as MB
import weights_file as W

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = json.load(open(os.path.join(HERE, "golden", "weights_file_tiny.json")))
REFERENCE_FILE_BYTES = 15311790080  # model_speculative_moe_batched.mojo:1347


def _cfg(d: dict) -> "MB.ModelConfig":
    return MB.default_model_config(**d)


@pytest.fixture(scope="module")
def tiny_file(tmp_path_factory):
    cfg = GOLDEN["config"]
    path = tmp_path_factory.mktemp("wf") / "gemma4_moe_weights_q4.bin"
    layers = W.tiny_model(cfg, GOLDEN["seed"])
    W.write_weights_file(path, [W.quantized_layer(t) for t in layers])
    return cfg, layers, path


def test_default_config_is_the_references():
    c = MB.default_model_config()
    assert {n: getattr(c, n) for n, _ in MB.ModelConfig._fields_} == W.DEFAULT_CONFIG


def test_file_size_is_the_size_the_reference_hard_codes():
    assert MB.weights_file_size(MB.default_model_config()) == REFERENCE_FILE_BYTES
    assert W.file_size(W.DEFAULT_CONFIG) == REFERENCE_FILE_BYTES


@pytest.mark.parametrize("cfg", [W.DEFAULT_CONFIG, W.TINY_CONFIG], ids=["default", "tiny"])
def test_library_layout_equals_the_restatement(cfg):
    c = _cfg(cfg)
    names = [n for n, _ in W.MATRICES]
    vnames = [n for n, _ in W.VECTORS]
    for layer in range(cfg["num_layers"]):
        lib = MB.weights_layout(c, layer)
        ref = W.layer_layout(cfg, layer)
        assert lib.layer_offset == ref["offset"] and lib.layer_bytes == ref["bytes"]
        assert lib.payload_bytes == ref["payload"]
        assert bool(lib.is_global) == W.is_global(cfg, layer)
        for m, n in enumerate(names):
            assert lib.packed_offset[m] == ref["packed"][n], (layer, n)
            assert lib.scales_offset[m] == ref["scales"][n], (layer, n)
            shp = ref["shapes"][n]
            assert lib.rows[m] * lib.cols[m] == int(np.prod(shp)), (layer, n)
            if lib.rows[m]:
                assert lib.cols[m] == shp[-1]
        for v, n in enumerate(vnames):
            assert lib.vec_offset[v] == ref["vec"][n], (layer, n)
            assert lib.vec_len[v] == int(np.prod(ref["shapes"][n]))


def test_global_layers_have_no_v_proj():
    c = MB.default_model_config()
    for layer in range(30):
        L = MB.weights_layout(c, layer)
        assert (L.rows[MB.W_V] == 0) == (layer % 6 == 5)
        assert L.head_dim == (512 if layer % 6 == 5 else 256)


def test_restated_writer_reproduces_the_converter(tiny_file):
    cfg, _, path = tiny_file
    data = open(path, "rb").read()
    assert len(data) == GOLDEN["file_bytes"] == MB.weights_file_size(_cfg(cfg))
    assert [W.layer_layout(cfg, l)["bytes"] for l in range(30)] == GOLDEN["layer_bytes"]
    off = 0
    for l, (n, h) in enumerate(zip(GOLDEN["layer_bytes"], GOLDEN["layer_sha256"])):
        assert hashlib.sha256(data[off:off + n]).hexdigest() == h, f"layer {l}"
        off += n
    assert hashlib.sha256(data).hexdigest() == GOLDEN["sha256"]


def test_library_layout_finds_every_tensor_of_the_converter_file(tiny_file):
    cfg, layers, path = tiny_file
    data = np.fromfile(path, np.uint8)
    c = _cfg(cfg)
    for l, t in enumerate(layers):
        L = MB.weights_layout(c, l)
        blob = data[L.layer_offset:L.layer_offset + L.layer_bytes]
        for m, (n, _) in enumerate(W.MATRICES):
            elems = L.rows[m] * L.cols[m]
            assert elems == t[n].size
            if not elems:
                continue
            packed = blob[L.packed_offset[m]:L.packed_offset[m] + elems // 2]
            scales = blob[L.scales_offset[m]:L.scales_offset[m] + elems // 8].view(np.float32)
            # dequantised values sit within half a step of the original weights
            lo = (packed & 15).astype(np.float32) - 8
            hi = (packed >> 4).astype(np.float32) - 8
            deq = np.stack([lo, hi], 1).reshape(-1, 32) * scales[:, None]
            err = np.abs(deq - t[n].reshape(-1, 32))
            assert (err <= 0.5 * scales[:, None] * (1 + 1e-6) + 1e-12).all(), (l, n)
        for v, (n, _) in enumerate(W.VECTORS):
            got = blob[L.vec_offset[v]:L.vec_offset[v] + 4 * L.vec_len[v]].view(np.float32)
            np.testing.assert_array_equal(got, t[n].reshape(-1), err_msg=f"layer {l} {n}")
        assert not blob[L.payload_bytes:].any()


def test_layer_desc_points_into_the_image():
    c = MB.default_model_config()
    base = 1 << 40  # address arithmetic only: nothing is dereferenced
    for layer in (0, 5, 29):
        L = MB.weights_layout(c, layer)
        d = MB.layer_desc_from_weights(c, base, layer)
        b = base + L.layer_offset
        assert (d.embed_dim, d.expert_mlp_dim, d.num_experts, d.top_k) == (2816, 704, 128, 8)
        assert d.activation == MB.ACT_SIGMOID1702 and d.moe_top_p == 1.0
        assert np.float32(d.r_scale_factor) == np.float32(1.0) / np.sqrt(np.float32(2816))
        assert d.router_packed == b + L.packed_offset[MB.W_ROUTER]
        assert d.router_scales == b + L.scales_offset[MB.W_ROUTER]
        assert d.gate_up_packed == b + L.packed_offset[MB.W_EXPERTS_GATE_UP]
        assert d.gate_up_scales == b + L.scales_offset[MB.W_EXPERTS_GATE_UP]
        assert d.down_packed == b + L.packed_offset[MB.W_EXPERTS_DOWN]
        assert d.down_scales == b + L.scales_offset[MB.W_EXPERTS_DOWN]
        assert d.router_scale == b + L.vec_offset[MB.V_ROUTER_SCALE]
        assert d.per_expert_scale == b + L.vec_offset[MB.V_ROUTER_PER_EXPERT_SCALE]
        assert d.pre_norm_w == b + L.vec_offset[MB.V_PRE_FEEDFORWARD_LAYERNORM_2]
        assert d.post_norm_w == b + L.vec_offset[MB.V_POST_FEEDFORWARD_LAYERNORM_2]
        assert d.router_f32 is None and d.router_logit_bias is None
        # the kernels' TMA loads need 16-byte aligned weight and scale arrays
        for p in (d.router_packed, d.gate_up_packed, d.down_packed, d.gate_up_scales, d.down_scales):
            assert p % 16 == 0


def test_bad_arguments_are_rejected():
    lib = MB.load_library()
    c = MB.default_model_config()
    out = MB.LayerLayout()
    assert lib.moe_weights_layout(C.byref(c), 30, C.byref(out)) == 1
    assert lib.moe_weights_layout(C.byref(c), -1, C.byref(out)) == 1
    assert lib.moe_weights_layout(None, 0, C.byref(out)) == 1
    bad = MB.default_model_config(expert_mlp_dim=40)  # experts_down inner dim not a multiple of 32
    assert lib.moe_weights_layout(C.byref(bad), 0, C.byref(out)) == 2
    zero = MB.default_model_config(num_heads=0)
    assert lib.moe_weights_layout(C.byref(zero), 0, C.byref(out)) == 1
    d = MB.LayerDesc()
    assert lib.moe_layer_desc_from_weights(C.byref(c), None, 0, C.byref(d)) == 1
    many = MB.default_model_config(top_k=200)
    assert lib.moe_layer_desc_from_weights(C.byref(many), 4096, 0, C.byref(d)) == 2
    n = C.c_int64(0)
    assert lib.moe_load_weights_file(None, b"x", 0, -1, 4096, C.byref(n)) == 1
    with pytest.raises(TypeError):
        MB.default_model_config(no_such_field=1)
