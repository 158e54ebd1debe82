"""Python host mirror of the reference's Mojo entry points over libmoe_b200.so.

Function names, argument order and meaning follow phildrip/llm-mojo's
``moe_kernels.mojo`` / ``diffusion_kernels.mojo`` / the layer glue in
``model_speculative_moe_batched.mojo`` (file:line in each docstring); the
``num_tasks`` thread-count arguments of the CPU originals are accepted and
ignored.  Arrays may be numpy (host; staged by the library) or torch CUDA
tensors (used in place).  Every call goes through the C ABI of
include/moe_b200.h; there is no CPU fallback: without a CUDA device
``Context()`` raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmoe_b200.so")

ACT_SIGMOID1702, ACT_GELU_TANH = 0, 1
X_NATURAL, X_DEINT_HALVES, X_DEINT_BLOCK32 = 0, 1, 2
F_POST_NORM, F_SET_COVER, F_FP16_OUT = 1, 4, 8
OPT_GEMM_PATH, OPT_TC_MIN_TOKENS, OPT_DEVICE_TIMEOUT_NS = 1, 2, 3
OPT_DENSE_TC_MIN_TOKENS, OPT_TC_A_IN_SMEM, OPT_ROUTER_TC_MIN_TOKENS = 4, 5, 6
OPT_TC_STREAM = 7
OPT_EXPERT_BEGIN, OPT_EXPERT_END = 8, 9
OPT_FUSED_ROUTE = 10
OPT_DENSE_KSPLIT = 11
OPT_EP_TIMEOUT_NS = 12
OPT_EP_MODE, OPT_EP_LOCAL_WEIGHTS, OPT_GEMV_ONE_TOKEN, OPT_DENSE_ONE_LAUNCH = 13, 14, 15, 16
EP_REPLICATED, EP_GATHER, EP_ALL_TO_ALL = 0, 1, 2
EP_UNIQUE_ID_BYTES = 128
PATH_AUTO, PATH_GEMV, PATH_TC = 0, 1, 2

STATUS = {0: "MOE_OK", 1: "MOE_E_ARG", 2: "MOE_E_SHAPE", 3: "MOE_E_UNREGISTERED",
          4: "MOE_E_CUDA", 5: "MOE_E_NCCL", 6: "MOE_E_TIMEOUT", 7: "MOE_E_NOMEM",
          8: "MOE_E_STATE"}

# every symbol declared in include/moe_b200.h
EXPORTS = [
    "moe_ctx_create", "moe_ctx_destroy", "moe_last_error", "moe_kernel_launches",
    "moe_set_stream", "moe_set_async", "moe_wait", "moe_set_option", "moe_profile_enable",
    "moe_profile_read",
    "moe_register_weights",
    "moe_unregister_weights", "moe_quantize_fp32_to_q4_0", "moe_q4_matmul_vec",
    "moe_q4_matmul_batchN", "moe_compute_moe_lod_weights", "moe_apply_moe_lod_and_set_cover",
    "moe_compute_subbatch_set_cover_moe_weights", "moe_run_moe_experts_stage1",
    "moe_run_moe_experts_stage2", "moe_run_moe_coalesced_core",
    "moe_run_diffusion_moe_experts_parallel", "moe_route", "moe_layer_forward",
    "moe_q4_matmul_batchN_noalloc", "moe_rms_norm",
    "moe_default_model_config", "moe_weights_layout", "moe_weights_file_size",
    "moe_layer_desc_from_weights", "moe_load_weights_file",
    "moe_ep_get_unique_id", "moe_ep_init", "moe_ep_finalize",
    "moe_run_moe_coalesced_stage1", "moe_run_moe_coalesced_stage2",
    "moe_router_subspace_ffn_filter", "moe_sync_moe_subspace_cache",
    "moe_scatter_and_restore_ffn_subspace", "moe_device_wait_check",
]


class MoeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


_lib = None


def load_library(path: str = LIB_PATH):
    """Loads the shared library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise OSError(f"{path} not built: run python llm-mojo_b200/build.py")
        _lib = C.CDLL(path)
        _declare(_lib)
    return _lib


_p, _i64, _int, _f, _u64 = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_uint64


class LayerDesc(C.Structure):
    """moe_layer_desc of include/moe_b200.h."""
    _fields_ = [
        ("embed_dim", _i64), ("expert_mlp_dim", _i64), ("num_experts", _i64), ("top_k", _i64),
        ("activation", C.c_int32), ("r_scale_factor", _f), ("moe_top_p", _f),
        ("router_packed", _p), ("router_scales", _p), ("router_f32", _p),
        ("router_logit_bias", _p), ("router_scale", _p), ("per_expert_scale", _p),
        ("pre_norm_w", _p), ("post_norm_w", _p), ("gate_up_packed", _p),
        ("gate_up_scales", _p), ("down_packed", _p), ("down_scales", _p),
    ]


W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN, W_ROUTER, W_EXPERTS_GATE_UP, W_EXPERTS_DOWN = range(10)
W_COUNT = 10
WEIGHT_MATRICES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj",
                   "router", "experts_gate_up", "experts_down")
(V_INPUT_LAYERNORM, V_POST_ATTENTION_LAYERNORM, V_PRE_FEEDFORWARD_LAYERNORM,
 V_PRE_FEEDFORWARD_LAYERNORM_2, V_POST_FEEDFORWARD_LAYERNORM, V_POST_FEEDFORWARD_LAYERNORM_1,
 V_POST_FEEDFORWARD_LAYERNORM_2, V_Q_NORM, V_K_NORM, V_ROUTER_SCALE, V_ROUTER_PER_EXPERT_SCALE,
 V_LAYER_SCALAR) = range(12)
V_COUNT = 12


class ModelConfig(C.Structure):
    """moe_model_config of include/moe_b200.h (MoEConfig,
    model_speculative_moe_batched.mojo:41-63)."""
    _fields_ = [(n, _i64) for n in (
        "embed_dim", "standard_mlp_dim", "expert_mlp_dim", "num_experts", "top_k", "num_layers",
        "num_heads", "head_dim_sliding", "kv_heads_sliding", "head_dim_global", "kv_heads_global",
        "global_every")]


class LayerLayout(C.Structure):
    """moe_layer_layout of include/moe_b200.h: where each tensor of one layer
    sits in the weights file (offsets within the layer's blob)."""
    _fields_ = [("layer_offset", _i64), ("layer_bytes", _i64), ("payload_bytes", _i64),
                ("is_global", _i64), ("head_dim", _i64), ("kv_heads", _i64),
                ("rows", _i64 * W_COUNT), ("cols", _i64 * W_COUNT),
                ("packed_offset", _i64 * W_COUNT), ("scales_offset", _i64 * W_COUNT),
                ("vec_offset", _i64 * V_COUNT), ("vec_len", _i64 * V_COUNT)]


def _declare(L):
    L.moe_ctx_create.argtypes = [_int, C.POINTER(_p)]
    L.moe_ctx_destroy.argtypes = [_p]
    L.moe_last_error.argtypes = [_p]
    L.moe_last_error.restype = C.c_char_p
    L.moe_kernel_launches.argtypes = [_p]
    L.moe_kernel_launches.restype = _u64
    L.moe_set_stream.argtypes = [_p, _p]
    L.moe_set_async.argtypes = [_p, _int]
    L.moe_wait.argtypes = [_p, _u64]
    L.moe_set_option.argtypes = [_p, _int, _i64]
    L.moe_profile_enable.argtypes = [_p, _int]
    L.moe_profile_read.argtypes = [_p, _int, _p, _p, _p, C.POINTER(_int)]
    L.moe_register_weights.argtypes = [_p, _p, C.c_size_t]
    L.moe_unregister_weights.argtypes = [_p, _p]
    L.moe_quantize_fp32_to_q4_0.argtypes = [_p, _p, _p, _p, _i64]
    L.moe_q4_matmul_vec.argtypes = [_p, _p, _p, _p, _p, _i64, _i64]
    L.moe_q4_matmul_batchN.argtypes = [_p, _i64, _p, _p, _p, _p, _i64, _i64]
    L.moe_q4_matmul_batchN_noalloc.argtypes = [_p, _i64, _p, _p, _p, _p, _i64, _i64]
    L.moe_rms_norm.argtypes = [_p, _p, _p, _p, _i64, _i64]
    L.moe_compute_moe_lod_weights.argtypes = [_p, _i64, _p, _p, _p, _f, _p, _p, _p, _i64]
    L.moe_apply_moe_lod_and_set_cover.argtypes = [_p, _p, _p, _p, _p, _i64, _i64, _i64, _f, _p,
                                                  _p, _i64]
    L.moe_compute_subbatch_set_cover_moe_weights.argtypes = [_p, _i64, _p, _p, _p, _f, _p, _p,
                                                             _p, _i64, _i64, _f, _f]
    L.moe_run_moe_experts_stage1.argtypes = [_p, _p, _p, _p, _p, _i64, _p, _p, _i64, _i64, _int]
    L.moe_run_moe_experts_stage2.argtypes = [_p, _p, _p, _p, _p, _p, _i64, _p, _i64, _i64]
    L.moe_run_moe_coalesced_core.argtypes = [_p, _i64, _p, _p, _p, _p, _p, _int, _p, _p, _p, _p,
                                             _i64, _i64, _i64, _i64, _int]
    L.moe_run_diffusion_moe_experts_parallel.argtypes = [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64,
                                                         _i64, _i64, _i64, _int]
    L.moe_route.argtypes = [_p, C.POINTER(LayerDesc), _i64, _p, _int, _p, _p, _p, _p, _p, _p, _p]
    L.moe_layer_forward.argtypes = [_p, C.POINTER(LayerDesc), _i64, _p, _p, _int, _p, _p, _p]
    L.moe_default_model_config.argtypes = [C.POINTER(ModelConfig)]
    L.moe_weights_layout.argtypes = [C.POINTER(ModelConfig), _i64, C.POINTER(LayerLayout)]
    L.moe_weights_file_size.argtypes = [C.POINTER(ModelConfig), C.POINTER(_i64)]
    L.moe_layer_desc_from_weights.argtypes = [C.POINTER(ModelConfig), _p, _i64, C.POINTER(LayerDesc)]
    L.moe_load_weights_file.argtypes = [_p, C.c_char_p, _i64, _i64, _p, C.POINTER(_i64)]
    L.moe_run_moe_coalesced_stage1.argtypes = [_p, _i64, _p, _p, _p, _int, _p, _p, _p, _p, _p, _p, _p, _p,
                                               _p, _i64, _i64, _i64, _i64, _int, C.POINTER(_i64)]
    L.moe_run_moe_coalesced_stage2.argtypes = [_p, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64]
    L.moe_router_subspace_ffn_filter.argtypes = [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _f,
                                                 _p, C.POINTER(_i64)]
    L.moe_sync_moe_subspace_cache.argtypes = [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64]
    L.moe_scatter_and_restore_ffn_subspace.argtypes = [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64]
    L.moe_device_wait_check.argtypes = [_p]
    L.moe_ep_get_unique_id.argtypes = [_p]
    L.moe_ep_init.argtypes = [_p, _p, _int, _int]
    L.moe_ep_finalize.argtypes = [_p]
    for name in EXPORTS:
        if name not in ("moe_last_error", "moe_kernel_launches"):
            getattr(L, name).restype = _int


def _addr(a):
    """Address of a numpy array or torch tensor (None -> NULL)."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        assert a.flags["C_CONTIGUOUS"], "arrays must be C-contiguous"
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        assert a.is_contiguous(), "tensors must be contiguous"
        return a.data_ptr()
    if isinstance(a, int):
        return a
    raise TypeError(f"unsupported buffer type {type(a)}")


class Context:
    """One device context (moe_ctx_create); use one per host thread."""

    def __init__(self, device: int = 0):
        self.lib = load_library()
        h = _p()
        rc = self.lib.moe_ctx_create(device, C.byref(h))
        if rc != 0:
            raise MoeError(rc, f"moe_ctx_create(device={device}) failed (no CUDA device?)")
        self.h = h
        self.device = device
        self._keep = []

    def close(self):
        if self.h:
            self.lib.moe_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, rc: int):
        if rc != 0:
            raise MoeError(rc, self.lib.moe_last_error(self.h).decode())

    def last_error(self) -> str:
        return self.lib.moe_last_error(self.h).decode()

    @property
    def kernel_launches(self) -> int:
        return int(self.lib.moe_kernel_launches(self.h))

    def set_stream(self, stream_ptr: int | None):
        self.check(self.lib.moe_set_stream(self.h, stream_ptr))

    def set_async(self, on: bool):
        self.check(self.lib.moe_set_async(self.h, int(on)))

    def wait(self, timeout_ns: int = 0):
        self.check(self.lib.moe_wait(self.h, timeout_ns))

    def set_option(self, option: int, value: int):
        self.check(self.lib.moe_set_option(self.h, option, value))

    def set_expert_range(self, begin: int = 0, end: int = 0):
        """Evaluate only experts [begin, end) in the multi-token expert paths
        (expert parallelism); end 0 selects all experts."""
        self.set_option(OPT_EXPERT_BEGIN, begin)
        self.set_option(OPT_EXPERT_END, end)

    def rms_norm(self, x, w, out, M, d):
        """model_speculative_moe_batched.mojo:857-879."""
        self.check(self.lib.moe_rms_norm(self.h, _addr(x), _addr(w), _addr(out), M, d))

    def set_gemm_path(self, path: int):
        """PATH_AUTO, PATH_GEMV (CUDA cores, fp32) or PATH_TC (tcgen05, fp16 operands)."""
        self.set_option(OPT_GEMM_PATH, path)

    def profile_enable(self, on: bool = True):
        self.check(self.lib.moe_profile_enable(self.h, int(on)))

    def profile_read(self) -> dict:
        """{kernel name: (total device ms, launches)} since profile_enable."""
        n_max = 64
        names = C.create_string_buffer(32 * n_max)
        ms = (C.c_double * n_max)()
        cnt = (C.c_uint64 * n_max)()
        n = _int(0)
        self.check(self.lib.moe_profile_read(self.h, n_max, names, ms, cnt, C.byref(n)))
        out = {}
        for i in range(min(n.value, n_max)):
            nm = names.raw[32 * i:32 * i + 32].split(b"\0", 1)[0].decode()
            out[nm] = (ms[i], int(cnt[i]))
        return out

    def register_weights(self, arr: np.ndarray):
        self.check(self.lib.moe_register_weights(self.h, _addr(arr), arr.nbytes))
        self._keep.append(arr)

    def unregister_weights(self, arr: np.ndarray):
        self.check(self.lib.moe_unregister_weights(self.h, _addr(arr)))

    # ------------------------------------------------- moe_kernels.mojo API
    def quantize_fp32_to_q4_0(self, src, dst_packed, dst_scales, num_elements, num_tasks=None):
        """moe_kernels.mojo:7-56."""
        self.check(self.lib.moe_quantize_fp32_to_q4_0(self.h, _addr(src), _addr(dst_packed),
                                                      _addr(dst_scales), num_elements))

    def q4_matmul_vec(self, W_packed, scales, x, out_ptr, c_in, c_out, num_tasks=None):
        """moe_kernels.mojo:59-67."""
        self.check(self.lib.moe_q4_matmul_vec(self.h, _addr(W_packed), _addr(scales), _addr(x),
                                              _addr(out_ptr), c_in, c_out))

    def q4_matmul_batchN(self, batch_size, W_packed, scales, x_batch, out_batch, c_in, c_out,
                         num_tasks=None):
        """moe_kernels.mojo:254-264 (and q4_matmul_batch5 :165)."""
        self.check(self.lib.moe_q4_matmul_batchN(self.h, batch_size, _addr(W_packed),
                                                 _addr(scales), _addr(x_batch), _addr(out_batch),
                                                 c_in, c_out))

    def q4_matmul_batchN_noalloc(self, batch_size, W_packed, scales, x_batch, out_batch, c_in, c_out):
        """q4_matmul_batchN on device buffers with the library's fixed static
        scratch instead of the context workspace: no allocation during the call."""
        self.check(self.lib.moe_q4_matmul_batchN_noalloc(self.h, batch_size, _addr(W_packed),
                                                         _addr(scales), _addr(x_batch),
                                                         _addr(out_batch), c_in, c_out))

    def compute_moe_lod_weights(self, top_idx, top_val, per_expert_scale, moe_top_p,
                                active_idx, active_weights, top_k=8, batch=1, active_count=None):
        """moe_kernels.mojo:445-490; returns the count (batch == 1) or fills active_count."""
        cnt = np.zeros(batch, np.int64) if active_count is None else active_count
        self.check(self.lib.moe_compute_moe_lod_weights(self.h, batch, _addr(top_idx),
                                                        _addr(top_val), _addr(per_expert_scale),
                                                        moe_top_p, _addr(active_idx),
                                                        _addr(active_weights), _addr(cnt), top_k))
        if active_count is None and batch == 1:
            return int(cnt[0])
        return cnt

    def compute_subbatch_set_cover_moe_weights(self, sub_b, all_top_idx, all_top_val,
                                               per_expert_scale, moe_top_p, tok_active_count,
                                               tok_active_idx, tok_active_weights,
                                               num_experts=128, top_k=8, core_top_p=0.85,
                                               singleton_min_prob=0.068):
        """moe_kernels.mojo:493-611."""
        self.check(self.lib.moe_compute_subbatch_set_cover_moe_weights(
            self.h, sub_b, _addr(all_top_idx), _addr(all_top_val), _addr(per_expert_scale),
            moe_top_p, _addr(tok_active_count), _addr(tok_active_idx),
            _addr(tok_active_weights), num_experts, top_k, core_top_p, singleton_min_prob))

    def run_moe_experts_stage1_8core(self, experts_gate_up_packed, experts_gate_up_scales, moe_in,
                                     moe_in_deint, active_idx, active_count, gate_up_out_all,
                                     act_all, embed_dim=2816, expert_mlp_dim=704, num_tasks=8,
                                     activation=ACT_SIGMOID1702):
        """moe_kernels.mojo:614-627 (moe_in_deint scratch unused)."""
        self.check(self.lib.moe_run_moe_experts_stage1(
            self.h, _addr(experts_gate_up_packed), _addr(experts_gate_up_scales), _addr(moe_in),
            _addr(active_idx), active_count, _addr(gate_up_out_all), _addr(act_all), embed_dim,
            expert_mlp_dim, activation))

    def run_moe_experts_stage2_8core(self, experts_down_packed, experts_down_scales, act_all,
                                     act_deint, active_idx, active_weights, active_count, moe_out,
                                     embed_dim=2816, expert_mlp_dim=704, num_tasks=8):
        """moe_kernels.mojo:699-712 (act_deint scratch unused)."""
        self.check(self.lib.moe_run_moe_experts_stage2(
            self.h, _addr(experts_down_packed), _addr(experts_down_scales), _addr(act_all),
            _addr(active_idx), _addr(active_weights), active_count, _addr(moe_out), embed_dim,
            expert_mlp_dim))

    def run_moe_coalesced_core(self, sub_b, experts_gate_up_packed, experts_gate_up_scales,
                               experts_down_packed, experts_down_scales, batch_in_deint,
                               tok_active_count, tok_active_idx, tok_active_weights,
                               batch_moe_out, embed_dim=2816, expert_mlp_dim=704, num_experts=128,
                               num_tasks=8, x_layout=X_DEINT_HALVES, top_k=8,
                               activation=ACT_SIGMOID1702):
        """moe_kernels.mojo:1321-1345 (bucket/scratch arguments are internal here)."""
        self.check(self.lib.moe_run_moe_coalesced_core(
            self.h, sub_b, _addr(experts_gate_up_packed), _addr(experts_gate_up_scales),
            _addr(experts_down_packed), _addr(experts_down_scales), _addr(batch_in_deint),
            x_layout, _addr(tok_active_count), _addr(tok_active_idx), _addr(tok_active_weights),
            _addr(batch_moe_out), embed_dim, expert_mlp_dim, num_experts, top_k, activation))

    def run_moe_coalesced_stage1(self, sub_b, experts_gate_up_packed, experts_gate_up_scales,
                                 batch_in_deint, tok_active_count, tok_active_idx,
                                 tok_active_weights, bucket_counts, bucket_toks, bucket_weights,
                                 unique_experts, unique_base_slot, gu_out_scratch, act_scratch,
                                 act_deint_scratch, embed_dim=2816, expert_mlp_dim=704,
                                 num_experts=128, num_tasks=8, x_layout=X_DEINT_HALVES, top_k=8,
                                 activation=ACT_SIGMOID1702) -> int:
        """moe_kernels.mojo:784-805; returns num_unique.  gu_out_scratch and
        act_scratch are accepted for signature parity (the device keeps its
        own); act_deint_scratch names the result for stage 2."""
        n = _i64(0)
        self.check(self.lib.moe_run_moe_coalesced_stage1(
            self.h, sub_b, _addr(experts_gate_up_packed), _addr(experts_gate_up_scales),
            _addr(batch_in_deint), x_layout, _addr(tok_active_count), _addr(tok_active_idx),
            _addr(tok_active_weights), _addr(bucket_counts), _addr(bucket_toks),
            _addr(bucket_weights), _addr(unique_experts), _addr(unique_base_slot),
            _addr(act_deint_scratch), embed_dim, expert_mlp_dim, num_experts, top_k, activation,
            C.byref(n)))
        return int(n.value)

    def run_moe_coalesced_stage2(self, sub_b, num_unique, experts_down_packed,
                                 experts_down_scales, bucket_counts, bucket_toks, bucket_weights,
                                 unique_experts, unique_base_slot, act_deint_scratch,
                                 batch_moe_out, embed_dim=2816, expert_mlp_dim=704, num_tasks=8):
        """moe_kernels.mojo:1072-1088."""
        self.check(self.lib.moe_run_moe_coalesced_stage2(
            self.h, sub_b, num_unique, _addr(experts_down_packed), _addr(experts_down_scales),
            _addr(bucket_counts), _addr(bucket_toks), _addr(bucket_weights),
            _addr(unique_experts), _addr(unique_base_slot), _addr(act_deint_scratch),
            _addr(batch_moe_out), embed_dim, expert_mlp_dim))

    # ------------------------------------------- diffusion_kernels.mojo API
    def run_diffusion_moe_experts_parallel(self, experts_gate_up_packed, experts_gate_up_scales,
                                           experts_down_packed, experts_down_scales,
                                           canvas_moe_in, canvas_top_idx, canvas_top_weights,
                                           canvas_moe_out, B, embed_dim, expert_mlp_dim,
                                           top_k_experts, num_tasks=8,
                                           activation=ACT_SIGMOID1702):
        """diffusion_kernels.mojo:236-253 (fp16 canvas in/out)."""
        self.check(self.lib.moe_run_diffusion_moe_experts_parallel(
            self.h, _addr(experts_gate_up_packed), _addr(experts_gate_up_scales),
            _addr(experts_down_packed), _addr(experts_down_scales), _addr(canvas_moe_in),
            _addr(canvas_top_idx), _addr(canvas_top_weights), _addr(canvas_moe_out), B,
            embed_dim, expert_mlp_dim, top_k_experts, activation))

    def router_subspace_ffn_filter(self, r_curr, r_prev, top_idx, prev_top2, eb_mask,
                                   active_canvas_idx, ffn_keep_b, B, num_experts, top_k, step,
                                   tau_ffn=0.05, top_weights=None) -> int:
        """diffusion_kernels.mojo:2253-2337; returns the number of kept rows
        (listed in ffn_keep_b); r_prev, prev_top2 and top_weights are updated."""
        n = _i64(0)
        self.check(self.lib.moe_router_subspace_ffn_filter(
            self.h, _addr(r_curr), _addr(r_prev), _addr(top_idx), _addr(prev_top2), _addr(eb_mask),
            _addr(active_canvas_idx), _addr(ffn_keep_b), B, num_experts, top_k, step, tau_ffn,
            _addr(top_weights), C.byref(n)))
        return int(n.value)

    def sync_moe_subspace_cache(self, moe_out, moe_prev_cache, active_canvas_idx, ffn_keep_b, B,
                                ffn_active_len, dim, elem_bytes=2):
        """diffusion_kernels.mojo:2345-2381 (elem_bytes 2: fp16 rows, 4: fp32)."""
        self.check(self.lib.moe_sync_moe_subspace_cache(
            self.h, _addr(moe_out), _addr(moe_prev_cache), _addr(active_canvas_idx),
            _addr(ffn_keep_b), B, ffn_active_len, dim, elem_bytes))

    def scatter_and_restore_ffn_subspace(self, ffn_sub_out, ffn_prev_cache, ffn_full_out,
                                         active_canvas_idx, ffn_keep_b, B, ffn_active_len, dim,
                                         elem_bytes=2):
        """diffusion_kernels.mojo:2386-2426 (elem_bytes 2: fp16 rows, 4: fp32)."""
        self.check(self.lib.moe_scatter_and_restore_ffn_subspace(
            self.h, _addr(ffn_sub_out), _addr(ffn_prev_cache), _addr(ffn_full_out),
            _addr(active_canvas_idx), _addr(ffn_keep_b), B, ffn_active_len, dim, elem_bytes))

    def device_wait_check(self):
        """Runs the bounded-wait check (moe_device_wait_check): raises
        MoeError with code 6 (MOE_E_TIMEOUT) when the wait gave up as designed."""
        self.check(self.lib.moe_device_wait_check(self.h))

    def apply_moe_lod_and_set_cover(self, canvas_top_idx, canvas_top_val, router_per_expert_scale,
                                    canvas_top_weights, B, top_k_experts, active_top_k,
                                    moe_top_p, eb_mask=None, active_canvas_idx=None,
                                    unaccepted_top_k=8):
        """diffusion_kernels.mojo:3607-3664."""
        self.check(self.lib.moe_apply_moe_lod_and_set_cover(
            self.h, _addr(canvas_top_idx), _addr(canvas_top_val), _addr(router_per_expert_scale),
            _addr(canvas_top_weights), B, top_k_experts, active_top_k, moe_top_p,
            _addr(eb_mask), _addr(active_canvas_idx), unaccepted_top_k))

    # ------------------------------------------------------- layer glue
    def route(self, desc: LayerDesc, M, x, tok_active_count, tok_active_idx, tok_active_weights,
              flags=0, scores=None, top_idx=None, top_val=None, moe_in=None):
        """Router half of model_speculative_moe_batched.mojo:957-1083 / :2102-2118."""
        self.check(self.lib.moe_route(self.h, C.byref(desc), M, _addr(x), flags, _addr(scores),
                                      _addr(top_idx), _addr(top_val), _addr(tok_active_count),
                                      _addr(tok_active_idx), _addr(tok_active_weights),
                                      _addr(moe_in)))

    def ep_init(self, unique_id: bytes, rank: int, nranks: int):
        """Joins an NCCL communicator (moe_ep_init): from then on
        layer_forward evaluates this rank's experts, sums the ranks' partial
        outputs and applies the post-norm to the sum."""
        if len(unique_id) != EP_UNIQUE_ID_BYTES:
            raise ValueError("the communicator id has 128 bytes")
        buf = C.create_string_buffer(bytes(unique_id), EP_UNIQUE_ID_BYTES)
        self.check(self.lib.moe_ep_init(self.h, C.addressof(buf), rank, nranks))

    def ep_finalize(self):
        self.check(self.lib.moe_ep_finalize(self.h))

    def load_weights_file(self, path: str, dst, file_offset: int = 0, nbytes: int = -1) -> int:
        """Reads bytes [file_offset, file_offset + nbytes) of the weights file
        into the device buffer `dst` (nbytes -1: to the end of the file);
        replaces the host-RAM load of model_speculative_moe_batched.mojo:1333-1380.
        Returns the byte count."""
        n = _i64(0)
        self.check(self.lib.moe_load_weights_file(self.h, os.fsencode(path), file_offset, nbytes,
                                                  _addr(dst), C.byref(n)))
        return int(n.value)

    def layer_forward(self, desc: LayerDesc, M, x, out, flags=F_POST_NORM, tok_active_count=None,
                      tok_active_idx=None, tok_active_weights=None):
        """run_moe_coalesced_subbatch, model_speculative_moe_batched.mojo:1155-1204, any M."""
        self.check(self.lib.moe_layer_forward(self.h, C.byref(desc), M, _addr(x), _addr(out),
                                              flags, _addr(tok_active_count),
                                              _addr(tok_active_idx), _addr(tok_active_weights)))


def make_desc(w: dict, act=ACT_SIGMOID1702, top_p=1.0, r_scale_factor=None, bias=None,
              router_fp32=False) -> LayerDesc:
    """Builds a LayerDesc from a dict of arrays/tensors (keys as in synth.make_layer)."""
    d = LayerDesc()
    d.embed_dim, d.expert_mlp_dim, d.num_experts, d.top_k = w["d"], w["F"], w["E"], w["top_k"]
    d.activation = act
    d.r_scale_factor = float(1.0 / np.sqrt(np.float32(w["d"]))) if r_scale_factor is None else r_scale_factor
    d.moe_top_p = top_p
    if router_fp32:
        d.router_f32 = _addr(w["router_f32"])
    else:
        d.router_packed = _addr(w["router_p"])
        d.router_scales = _addr(w["router_s"])
    d.router_logit_bias = _addr(bias)
    d.router_scale = _addr(w["router_scale"])
    d.per_expert_scale = _addr(w["per_expert_scale"])
    d.pre_norm_w = _addr(w["pre_norm_w"])
    d.post_norm_w = _addr(w["post_norm_w"])
    d.gate_up_packed = _addr(w["gu_p"])
    d.gate_up_scales = _addr(w["gu_s"])
    d.down_packed = _addr(w["dn_p"])
    d.down_scales = _addr(w["dn_s"])
    d._keep = (w, bias)
    return d


def _status(rc: int, what: str):
    if rc != 0:
        raise MoeError(rc, what)


def default_model_config(**overrides) -> ModelConfig:
    """MoEConfig's defaults (model_speculative_moe_batched.mojo:41-63), with
    any field replaced by keyword."""
    cfg = ModelConfig()
    _status(load_library().moe_default_model_config(C.byref(cfg)), "moe_default_model_config")
    for k, v in overrides.items():
        if k not in dict(ModelConfig._fields_):
            raise TypeError(f"unknown model config field {k}")
        setattr(cfg, k, int(v))
    return cfg


def weights_layout(cfg: ModelConfig, layer: int) -> LayerLayout:
    """Offsets of layer `layer`'s tensors in the weights file
    (get_layer_offset / get_layer_weights, model_speculative_moe_batched.mojo:113-231)."""
    out = LayerLayout()
    _status(load_library().moe_weights_layout(C.byref(cfg), layer, C.byref(out)),
            f"moe_weights_layout(layer={layer})")
    return out


def weights_file_size(cfg: ModelConfig) -> int:
    n = _i64(0)
    _status(load_library().moe_weights_file_size(C.byref(cfg), C.byref(n)), "moe_weights_file_size")
    return int(n.value)


def layer_desc_from_weights(cfg: ModelConfig, weights_base, layer: int) -> LayerDesc:
    """The MoE layer descriptor of layer `layer` of a weights-file image at
    `weights_base` (a device tensor or an address); keeps the image alive."""
    d = LayerDesc()
    _status(load_library().moe_layer_desc_from_weights(C.byref(cfg), _addr(weights_base), layer,
                                                       C.byref(d)),
            f"moe_layer_desc_from_weights(layer={layer})")
    d._keep = weights_base
    return d


def load_weights_file(ctx: Context, path: str, cfg: ModelConfig | None = None, device=None):
    """Loads the whole weights file into one device buffer and returns
    (buffer, [LayerDesc per layer]): the B200 counterpart of the model's
    start-up load (model_speculative_moe_batched.mojo:1333-1387).  The file
    size must match the configuration."""
    import torch
    cfg = cfg if cfg is not None else default_model_config()
    size = weights_file_size(cfg)
    if os.path.getsize(path) != size:
        raise MoeError(2, f"{path} holds {os.path.getsize(path)} bytes; the configuration needs {size}")
    buf = torch.empty(size, dtype=torch.uint8, device=device if device is not None else f"cuda:{ctx.device}")
    n = ctx.load_weights_file(path, buf)
    assert n == size
    return buf, [layer_desc_from_weights(cfg, buf, layer) for layer in range(cfg.num_layers)]


def ep_unique_id() -> bytes:
    """A new NCCL communicator id (moe_ep_get_unique_id), to be passed to
    every rank's Context.ep_init."""
    buf = C.create_string_buffer(EP_UNIQUE_ID_BYTES)
    _status(load_library().moe_ep_get_unique_id(C.addressof(buf)), "moe_ep_get_unique_id")
    return buf.raw
