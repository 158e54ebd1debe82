"""ctypes loader for the CPU oracle (libmoe_oracle.so).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py, as the checker or the timed
CPU baseline.  The product package never imports this module.

Each wrapper names the reference routine it restates (file:line in
phildrip/llm-mojo).  Arrays are numpy, C-contiguous, host memory.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmoe_oracle.so")

F32, F64 = 0, 1
ACT_SIGMOID1702, ACT_GELU_TANH = 0, 1

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


_p = C.c_void_p
_i64 = C.c_int64
_int = C.c_int
_f = C.c_float


class OrcLayer(C.Structure):
    _fields_ = [
        ("d", _i64), ("F", _i64), ("E", _i64), ("top_k", _i64),
        ("act", _int), ("r_scale_factor", _f), ("top_p", _f),
        ("router_p", _p), ("router_s", _p), ("router_f32", _p),
        ("router_scale", _p), ("per_expert_scale", _p),
        ("pre_norm_w", _p), ("post_norm_w", _p),
        ("gu_p", _p), ("gu_s", _p), ("dn_p", _p), ("dn_s", _p),
        ("router_logit_bias", _p),
    ]


def _declare(L):
    L.orc_quantize_q4_0.argtypes = [_p, _i64, _p, _p]
    L.orc_quantize_q4_0.restype = _i64
    L.orc_q4_matmul.argtypes = [_p, _p, _p, _p, _i64, _i64, _i64, _int, _int]
    L.orc_rms_norm.argtypes = [_p, _p, _p, _i64]
    L.orc_softmax.argtypes = [_p, _i64]
    L.orc_get_top_k.argtypes = [_p, _i64, _i64, _p, _p]
    L.orc_compute_moe_lod_weights.argtypes = [_p, _p, _p, _f, _p, _p, _i64]
    L.orc_compute_moe_lod_weights.restype = _i64
    L.orc_compute_subbatch_set_cover_moe_weights.argtypes = [
        _i64, _p, _p, _p, _f, _p, _p, _p, _i64, _i64, _f, _f]
    L.orc_apply_moe_lod_and_set_cover.argtypes = [
        _p, _p, _p, _p, _i64, _i64, _i64, _f, _p, _p, _i64]
    L.orc_experts_stage1.argtypes = [_p, _p, _p, _p, _i64, _p, _p, _i64, _i64, _int, _int, _int]
    L.orc_experts_stage2.argtypes = [_p, _p, _p, _p, _p, _i64, _p, _i64, _i64, _int, _int]
    L.orc_route.argtypes = [C.POINTER(OrcLayer), _i64, _p, _int, _p, _p, _p, _p, _p, _p, _p, _int]
    L.orc_experts_forward.argtypes = [C.POINTER(OrcLayer), _i64, _p, _p, _p, _p, _p, _int, _int]
    L.orc_layer_forward.argtypes = [C.POINTER(OrcLayer), _i64, _p, _p, _int, _int, _int, _p, _p, _p]
    L.orc_diffusion_experts.argtypes = [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
                                        _int, _int, _int]
    L.orc_router_subspace_ffn_filter.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
                                                 _f, _p]
    L.orc_router_subspace_ffn_filter.restype = _i64
    L.orc_sync_moe_subspace_cache.argtypes = [_p, _p, _p, _p, _i64, _i64, _i64]
    L.orc_scatter_and_restore_ffn_subspace.argtypes = [_p, _p, _p, _p, _p, _i64, _i64, _i64]


def _ptr(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


def nthreads_default() -> int:
    return os.cpu_count() or 1


# ---------------------------------------------------------------- wrappers
def quantize_q4_0(w: np.ndarray):
    """moe_kernels.mojo:7-56 / convert_gemma4_moe.py:9-35 -> (packed u8, scales f32, ties)."""
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    assert w.size % 32 == 0
    packed = np.empty(w.size // 2, np.uint8)
    scales = np.empty(w.size // 32, np.float32)
    ties = lib().orc_quantize_q4_0(_ptr(w), w.size, _ptr(packed), _ptr(scales))
    return packed, scales, int(ties)


def q4_matmul(W, S, x, c_in, c_out, prec=F64, nthreads=None):
    """q4_matmul_vec moe_kernels.mojo:59 / q4_matmul_batchN :254."""
    x = np.ascontiguousarray(x, np.float32)
    batch = x.size // c_in
    out = np.empty((batch, c_out), np.float32)
    lib().orc_q4_matmul(_ptr(W), _ptr(S), _ptr(x), _ptr(out), c_in, c_out, batch, prec,
                        nthreads or nthreads_default())
    return out


def rms_norm(x, w=None):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().orc_rms_norm(_ptr(x), _ptr(w), _ptr(out), x.size)
    return out


def softmax(s):
    s = np.array(s, np.float32, copy=True)
    lib().orc_softmax(_ptr(s), s.size)
    return s


def get_top_k(p, k=8):
    p = np.ascontiguousarray(p, np.float32)
    idx = np.empty(k, np.int64)
    val = np.empty(k, np.float32)
    lib().orc_get_top_k(_ptr(p), p.size, k, _ptr(idx), _ptr(val))
    return idx, val


def compute_moe_lod_weights(top_idx, top_val, per_expert_scale, top_p, top_k=8):
    top_idx = np.ascontiguousarray(top_idx, np.int64)
    top_val = np.ascontiguousarray(top_val, np.float32)
    pes = np.ascontiguousarray(per_expert_scale, np.float32)
    ai = np.zeros(top_k, np.int64)
    aw = np.zeros(top_k, np.float32)
    n = lib().orc_compute_moe_lod_weights(_ptr(top_idx), _ptr(top_val), _ptr(pes), top_p,
                                          _ptr(ai), _ptr(aw), top_k)
    return int(n), ai, aw


def set_cover(all_top_idx, all_top_val, per_expert_scale, top_p, top_k=8,
              core_top_p=0.85, singleton_min_prob=0.068):
    ti = np.ascontiguousarray(all_top_idx, np.int64)
    tv = np.ascontiguousarray(all_top_val, np.float32)
    sub_b = ti.size // top_k
    cnt = np.zeros(sub_b, np.int64)
    idx = np.zeros(sub_b * top_k, np.int64)
    w = np.zeros(sub_b * top_k, np.float32)
    pes = np.ascontiguousarray(per_expert_scale, np.float32)
    lib().orc_compute_subbatch_set_cover_moe_weights(sub_b, _ptr(ti), _ptr(tv), _ptr(pes), top_p,
                                                     _ptr(cnt), _ptr(idx), _ptr(w), pes.size,
                                                     top_k, core_top_p, singleton_min_prob)
    return cnt, idx.reshape(sub_b, top_k), w.reshape(sub_b, top_k)


def apply_moe_lod_and_set_cover(top_idx, top_val, per_expert_scale, B, top_k, active_top_k,
                                top_p, eb_mask=None, active_canvas_idx=None, unaccepted_top_k=8):
    ti = np.ascontiguousarray(top_idx, np.int64)
    tv = np.ascontiguousarray(top_val, np.float32)
    pes = np.ascontiguousarray(per_expert_scale, np.float32)
    tw = np.zeros(B * top_k, np.float32)
    eb = None if eb_mask is None else np.ascontiguousarray(eb_mask, np.uint8)
    ac = None if active_canvas_idx is None else np.ascontiguousarray(active_canvas_idx, np.int64)
    lib().orc_apply_moe_lod_and_set_cover(_ptr(ti), _ptr(tv), _ptr(pes), _ptr(tw), B, top_k,
                                          active_top_k, top_p, _ptr(eb), _ptr(ac), unaccepted_top_k)
    return tw.reshape(B, top_k)


def experts_stage1(gu_p, gu_s, moe_in, act_idx, d, F, act=ACT_SIGMOID1702, prec=F64,
                   nthreads=None):
    act_idx = np.ascontiguousarray(act_idx, np.int64)
    cnt = act_idx.size
    gu = np.zeros((max(cnt, 1), 2 * F), np.float32)
    a = np.zeros((max(cnt, 1), F), np.float32)
    lib().orc_experts_stage1(_ptr(gu_p), _ptr(gu_s), _ptr(np.ascontiguousarray(moe_in, np.float32)),
                             _ptr(act_idx), cnt, _ptr(gu), _ptr(a), d, F, act, prec,
                             nthreads or nthreads_default())
    return gu[:cnt], a[:cnt]


def experts_stage2(dn_p, dn_s, act_all, act_idx, act_w, d, F, prec=F64, nthreads=None):
    act_idx = np.ascontiguousarray(act_idx, np.int64)
    act_w = np.ascontiguousarray(act_w, np.float32)
    out = np.zeros(d, np.float32)
    aa = np.ascontiguousarray(act_all, np.float32)
    lib().orc_experts_stage2(_ptr(dn_p), _ptr(dn_s), _ptr(aa), _ptr(act_idx), _ptr(act_w),
                             act_idx.size, _ptr(out), d, F, prec, nthreads or nthreads_default())
    return out


def make_layer(w: dict, act=ACT_SIGMOID1702, top_p=1.0, r_scale_factor=None, bias=None):
    """Builds an OrcLayer from a dict of numpy arrays (see tests/synth.py).
    `bias` (optional, [E] fp32) is added to the router logits before the
    softmax: the synthetic skew of the prefill workload, not a reference
    feature."""
    d, F, E, K = w["d"], w["F"], w["E"], w["top_k"]
    L = OrcLayer()
    L.d, L.F, L.E, L.top_k = d, F, E, K
    L.act = act
    L.r_scale_factor = float(1.0 / np.sqrt(np.float32(d))) if r_scale_factor is None else r_scale_factor
    L.top_p = top_p
    L.router_p = _ptr(w.get("router_p"))
    L.router_s = _ptr(w.get("router_s"))
    L.router_f32 = _ptr(w.get("router_f32"))
    L.router_scale = _ptr(w["router_scale"])
    L.per_expert_scale = _ptr(w["per_expert_scale"])
    L.pre_norm_w = _ptr(w["pre_norm_w"])
    L.post_norm_w = _ptr(w["post_norm_w"])
    L.gu_p, L.gu_s = _ptr(w["gu_p"]), _ptr(w["gu_s"])
    L.dn_p, L.dn_s = _ptr(w["dn_p"]), _ptr(w["dn_s"])
    if bias is not None:
        bias = np.ascontiguousarray(bias, np.float32)
        L.router_logit_bias = _ptr(bias)
    L._keep = (w, bias)  # keep arrays alive
    return L


def route(L, x, use_set_cover=False):
    M = x.size // L.d
    K, E = L.top_k, L.E
    scores = np.zeros((M, E), np.float32)
    ti = np.zeros((M, K), np.int64)
    tv = np.zeros((M, K), np.float32)
    cnt = np.zeros(M, np.int64)
    idx = np.zeros((M, K), np.int64)
    w = np.zeros((M, K), np.float32)
    moe_in = np.zeros((M, L.d), np.float32)
    lib().orc_route(C.byref(L), M, _ptr(np.ascontiguousarray(x, np.float32)), int(use_set_cover),
                    _ptr(scores), _ptr(ti), _ptr(tv), _ptr(cnt), _ptr(idx), _ptr(w), _ptr(moe_in), F32)
    return dict(scores=scores, top_idx=ti, top_val=tv, count=cnt, idx=idx, w=w, moe_in=moe_in)


def experts_forward(L, moe_in, cnt, idx, w, prec=F64, nthreads=None):
    M = cnt.size
    out = np.zeros((M, L.d), np.float32)
    lib().orc_experts_forward(C.byref(L), M, _ptr(np.ascontiguousarray(moe_in, np.float32)),
                              _ptr(np.ascontiguousarray(cnt, np.int64)),
                              _ptr(np.ascontiguousarray(idx, np.int64)),
                              _ptr(np.ascontiguousarray(w, np.float32)), _ptr(out), prec,
                              nthreads or nthreads_default())
    return out


def layer_forward(L, x, post_norm=True, set_cover=False, prec=F64, nthreads=None):
    M = x.size // L.d
    out = np.zeros((M, L.d), np.float32)
    cnt = np.zeros(M, np.int64)
    idx = np.zeros((M, L.top_k), np.int64)
    w = np.zeros((M, L.top_k), np.float32)
    flags = (1 if post_norm else 0) | (4 if set_cover else 0)
    lib().orc_layer_forward(C.byref(L), M, _ptr(np.ascontiguousarray(x, np.float32)), _ptr(out),
                            flags, prec, nthreads or nthreads_default(), _ptr(cnt), _ptr(idx), _ptr(w))
    return out, cnt, idx, w


def diffusion_experts(gu_p, gu_s, dn_p, dn_s, x_f16, top_idx, top_w, d, F, top_k=8,
                      act=ACT_SIGMOID1702, prec=F64, nthreads=None):
    x_f16 = np.ascontiguousarray(x_f16, np.float16)
    B = x_f16.size // d
    out = np.zeros((B, d), np.float16)
    lib().orc_diffusion_experts(_ptr(gu_p), _ptr(gu_s), _ptr(dn_p), _ptr(dn_s),
                                _ptr(x_f16.view(np.uint16)),
                                _ptr(np.ascontiguousarray(top_idx, np.int64)),
                                _ptr(np.ascontiguousarray(top_w, np.float32)),
                                _ptr(out.view(np.uint16)), B, d, F, top_k, act, prec,
                                nthreads or nthreads_default())
    return out


def router_subspace_ffn_filter(r_curr, r_prev, top_idx, prev_top2, B, num_experts, top_k, step,
                               tau_ffn=0.05, eb_mask=None, active_canvas_idx=None, top_weights=None):
    """diffusion_kernels.mojo:2253-2337.  r_prev, prev_top2 and top_weights
    are updated in place; returns (ffn_keep_b[:count], count)."""
    keep = np.zeros(max(B, 1), np.int64)
    eb = None if eb_mask is None else np.ascontiguousarray(eb_mask, np.uint8)
    ac = None if active_canvas_idx is None else np.ascontiguousarray(active_canvas_idx, np.int64)
    n = lib().orc_router_subspace_ffn_filter(
        _ptr(np.ascontiguousarray(r_curr, np.float32)), _ptr(r_prev),
        _ptr(np.ascontiguousarray(top_idx, np.int64)), _ptr(prev_top2), _ptr(eb), _ptr(ac),
        _ptr(keep), B, num_experts, top_k, step, tau_ffn, _ptr(top_weights))
    return keep[:n], int(n)


def sync_moe_subspace_cache(moe_out, cache, ffn_keep_b, B, ffn_active_len, active_canvas_idx=None):
    """diffusion_kernels.mojo:2345-2381, in place on moe_out / cache (rows of
    any dtype)."""
    ac = None if active_canvas_idx is None else np.ascontiguousarray(active_canvas_idx, np.int64)
    row_bytes = moe_out.nbytes // B
    lib().orc_sync_moe_subspace_cache(_ptr(moe_out), _ptr(cache), _ptr(ac),
                                      _ptr(np.ascontiguousarray(ffn_keep_b, np.int64)), B,
                                      ffn_active_len, row_bytes)


def scatter_and_restore_ffn_subspace(sub_out, cache, full_out, ffn_keep_b, B, ffn_active_len,
                                     active_canvas_idx=None):
    """diffusion_kernels.mojo:2386-2426, in place on cache / full_out."""
    ac = None if active_canvas_idx is None else np.ascontiguousarray(active_canvas_idx, np.int64)
    row_bytes = full_out.nbytes // B
    lib().orc_scatter_and_restore_ffn_subspace(_ptr(np.ascontiguousarray(sub_out)), _ptr(cache),
                                               _ptr(full_out), _ptr(ac),
                                               _ptr(np.ascontiguousarray(ffn_keep_b, np.int64)), B,
                                               ffn_active_len, row_bytes)
