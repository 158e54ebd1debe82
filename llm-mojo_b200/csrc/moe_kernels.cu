// moe_kernels.cu -- CUDA-core kernels of the Q4_0 MoE-FFN path (sm_100a):
// router, expert bucketing, grouped Q4_0 GEMV with fused activation,
// weighted combine (+ post-norm), quantizer and routing helpers.
//
// The grouped GEMV (k_q4_gemv) is the memory-bound decode kernel: weights are
// streamed once with 128-bit non-allocating loads, nibbles are dequantised in
// registers (one shift + one LOP3 per weight, see nib_1p), activations sit in
// shared memory in a bank-conflict-free swizzle and partial sums are reduced
// with warp shuffles.
#include <float.h>

#include <algorithm>

#include "common.cuh"
#include "moe_internal.h"

namespace moe {

// Asks L2 for [p, p + bytes) (128-byte lines spread over the block's threads).
__device__ __forceinline__ void prefetch_l2(const void* p, int64_t bytes) {
    const char* c = static_cast<const char*>(p);
    for (int64_t o = (int64_t)threadIdx.x * 128; o < bytes; o += (int64_t)blockDim.x * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(c + o));
}

// Dot products of one Q4_0 block (16 bytes = 32 weights) with the
// matching 32 activations of T rows, one 32-bit word (8 weights) at a time.
// XS = true: weights as 1 + n/16 (shift + LOP3 per weight, see nib_1p); the
//   caller then uses sum (n-8) x = 16 * (dot - 1.5 * sum x).
// XS = false: exact n - 8 (shift + LOP3 + FADD per weight).
template <bool XS, int T>
__device__ __forceinline__ void block_dot(uint4 q, const float* const (&xp)[T], float (&d)[T]) {
    const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int t = 0; t < T; ++t) d[t] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float f[8];
        if (XS) {
            f[0] = nib_1p<0>(wv[i]);
            f[1] = nib_1p<1>(wv[i]);
            f[2] = nib_1p<2>(wv[i]);
            f[3] = nib_1p<3>(wv[i]);
            f[4] = nib_1p<4>(wv[i]);
            f[5] = nib_1p<5>(wv[i]);
            f[6] = nib_1p<6>(wv[i]);
            f[7] = nib_1p<7>(wv[i]);
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k)
                f[k] = __uint_as_float(0x4B000000u | ((wv[i] >> (4 * k)) & 0xFu)) - 8388616.0f;
        }
#pragma unroll
        for (int t = 0; t < T; ++t) {
            const float4* x4 = reinterpret_cast<const float4*>(xp[t]) + 2 * i;
            const float4 v0 = __ldg(x4), v1 = __ldg(x4 + 1);
            float p0 = f[0] * v0.x;
            float p1 = f[1] * v0.y;
            p0 = fmaf(f[2], v0.z, p0);
            p1 = fmaf(f[3], v0.w, p1);
            p0 = fmaf(f[4], v1.x, p0);
            p1 = fmaf(f[5], v1.y, p1);
            p0 = fmaf(f[6], v1.z, p0);
            p1 = fmaf(f[7], v1.w, p1);
            d[t] += p0 + p1;
        }
    }
}

// ------------------------------------------------------------ grouped GEMV
// Warp-level work item = (unique expert u, row group).  A warp owns 4 rows
// per pass (8 lanes per row; lane l8 takes blocks l8, l8+8, ...) and RPW
// passes.  All weight loads of the item are issued before any math; the
// activations are read through L1 (every lane group of the warp reads the
// same 128-byte block, so each load is a broadcast).  In ACT mode the 4
// rows of a pass are gate a, gate a+1, up a, up a+1 and the activation is
// applied after the 8-lane shuffle reduction.
struct GemvWarp {
    int lane, g, l8;
};

template <int MODE, bool XS, int NBL, int RPW, int T>
__device__ __forceinline__ void gemv_tokens(const GemvArgs& a, const GemvWarp& W, int cb, int nb,
                                            const uint4 (&wq)[RPW][NBL], const float (&sc)[RPW][NBL],
                                            const int64_t (&row)[RPW], const bool (&rv)[RPW],
                                            const int (&arow)[RPW], int p0) {
    const int K = a.K;
    int64_t xr[T];
    int po[T];
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const int p = p0 + t;
        xr[t] = a.pair_row ? a.pair_row[p] : p;
        po[t] = a.out_row ? a.out_row[p] : p;
    }
    float acc[RPW][T];
#pragma unroll
    for (int ip = 0; ip < RPW; ++ip)
#pragma unroll
        for (int t = 0; t < T; ++t) acc[ip][t] = 0.f;
#pragma unroll
    for (int ip = 0; ip < RPW; ++ip)
#pragma unroll
        for (int ib = 0; ib < NBL; ++ib) {
            const int b = W.l8 + 8 * (cb + ib);
            if (rv[ip] && b < nb) {
                const float* xp[T];
#pragma unroll
                for (int t = 0; t < T; ++t) xp[t] = a.X + xr[t] * K + b * 32;
                float dd[T];
                block_dot<XS, T>(wq[ip][ib], xp, dd);
                const float s = XS ? 16.0f * sc[ip][ib] : sc[ip][ib];
#pragma unroll
                for (int t = 0; t < T; ++t)
                    acc[ip][t] = XS ? fmaf(s, dd[t] - __ldg(a.xsum + xr[t] * nb + b), acc[ip][t])
                                    : fmaf(s, dd[t], acc[ip][t]);
            }
        }
#pragma unroll
    for (int ip = 0; ip < RPW; ++ip)
#pragma unroll
        for (int t = 0; t < T; ++t) {
            float v = acc[ip][t];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            if (MODE == GEMV_ACT) {
                const float up = __shfl_down_sync(0xffffffffu, v, 16);
                if (rv[ip]) {
                    if (W.l8 == 0 && a.gu_out) a.gu_out[(int64_t)po[t] * a.gu_stride + row[ip]] = v;
                    if (W.lane == 0 || W.lane == 8)
                        a.out[(int64_t)po[t] * a.out_stride + arow[ip]] = act_fn(v, up, a.act);
                }
            } else if (rv[ip] && W.l8 == 0) {
                a.out[(int64_t)po[t] * a.out_stride + row[ip]] = v;
            }
        }
}

constexpr int DENSE_CHUNK = 4;

template <int MODE, bool XS, int NBL, int RPW>
__global__ void __launch_bounds__(128, 4) k_q4_gemv(GemvArgs a) {
    pdl_wait();
    pdl_trigger();
    GemvWarp W;
    W.lane = threadIdx.x & 31;
    W.g = W.lane >> 3;
    W.l8 = W.lane & 7;
    const int warp = threadIdx.x >> 5;
    const int K = a.K, nb = K >> 5, nbl = (nb + 7) >> 3;
    const int rows_per_item = (MODE == GEMV_ACT) ? 2 * RPW : 4 * RPW;
    const int64_t tile_rows = (MODE == GEMV_ACT) ? a.F : a.rows_per_expert;
    const int n_groups = (int)((tile_rows + rows_per_item - 1) / rows_per_item);
    // dense mode splits the tokens into chunks of DENSE_CHUNK per item, so a
    // small matrix with many tokens (the router) still spreads over the GPU
    const int n_chunks = a.dense_tokens > 0 ? (a.dense_tokens + DENSE_CHUNK - 1) / DENSE_CHUNK : 1;
    const int U = a.dense_tokens > 0 ? n_chunks : a.meta[0];
    const int64_t n_items = (int64_t)U * n_groups;

    for (int64_t item = (int64_t)blockIdx.x * 4 + warp; item < n_items; item += (int64_t)gridDim.x * 4) {
        const int u = (int)(item / n_groups), grp = (int)(item - (int64_t)u * n_groups);
        const int e = a.dense_tokens > 0 ? 0 : a.unique_expert[u];
        const int n = a.dense_tokens > 0 ? min(DENSE_CHUNK, a.dense_tokens - u * DENSE_CHUNK) : a.seg_count[u];
        const int s0 = a.dense_tokens > 0 ? u * DENSE_CHUNK : a.seg_start[u];
        const uint8_t* Wp = a.Wp + (size_t)e * a.rows_per_expert * (K >> 1);
        const float* Ws = a.Ws + (size_t)e * a.rows_per_expert * nb;
        int64_t row[RPW];
        bool rv[RPW];
        int arow[RPW];
#pragma unroll
        for (int ip = 0; ip < RPW; ++ip) {
            if (MODE == GEMV_ACT) {
                const int ar = grp * rows_per_item + ip * 2 + (W.g & 1);
                arow[ip] = ar;
                rv[ip] = ar < a.F;
                row[ip] = (W.g < 2) ? ar : (int64_t)a.F + ar;
            } else {
                const int64_t r = (int64_t)grp * rows_per_item + ip * 4 + W.g;
                arow[ip] = 0;
                rv[ip] = r < a.rows_per_expert;
                row[ip] = r;
            }
        }
        // token chunks outermost; within a chunk, K chunks of NBL blocks per lane
        // (a single K chunk for the layer shapes, so weights are loaded once)
        const bool one_chunk = nbl <= NBL;
        uint4 wq[RPW][NBL];
        float sc[RPW][NBL];
        auto load = [&](int cb) {
#pragma unroll
            for (int ip = 0; ip < RPW; ++ip)
#pragma unroll
                for (int ib = 0; ib < NBL; ++ib) {
                    const int b = W.l8 + 8 * (cb + ib);
                    if (rv[ip] && b < nb) {
                        wq[ip][ib] = ldg_stream(Wp + row[ip] * (K >> 1) + b * 16);
                        sc[ip][ib] = ldg_stream_f(Ws + row[ip] * nb + b);
                    } else {
                        wq[ip][ib] = make_uint4(0, 0, 0, 0);
                        sc[ip][ib] = 0.f;
                    }
                }
        };
        if (one_chunk) {
            load(0);
            int t = 0;
            while (n - t >= 4) {
                gemv_tokens<MODE, XS, NBL, RPW, 4>(a, W, 0, nb, wq, sc, row, rv, arow, s0 + t);
                t += 4;
            }
            if (n - t >= 2) {
                gemv_tokens<MODE, XS, NBL, RPW, 2>(a, W, 0, nb, wq, sc, row, rv, arow, s0 + t);
                t += 2;
            }
            if (n - t >= 1) gemv_tokens<MODE, XS, NBL, RPW, 1>(a, W, 0, nb, wq, sc, row, rv, arow, s0 + t);
        } else {
            // long rows: one token at a time, K chunk by K chunk, partials kept
            // in the output row (first chunk stores, later chunks add)
            for (int t = 0; t < n; ++t) {
                const int p = s0 + t;
                const int64_t xr = a.pair_row ? a.pair_row[p] : p;
                const int64_t po = a.out_row ? a.out_row[p] : p;
                float acc[RPW];
#pragma unroll
                for (int ip = 0; ip < RPW; ++ip) acc[ip] = 0.f;
                for (int cb = 0; cb < nbl; cb += NBL) {
                    load(cb);
#pragma unroll
                    for (int ip = 0; ip < RPW; ++ip)
#pragma unroll
                        for (int ib = 0; ib < NBL; ++ib) {
                            const int b = W.l8 + 8 * (cb + ib);
                            if (rv[ip] && b < nb) {
                                const float* xp[1] = {a.X + xr * K + b * 32};
                                float dd[1];
                                block_dot<XS, 1>(wq[ip][ib], xp, dd);
                                const float s = XS ? 16.0f * sc[ip][ib] : sc[ip][ib];
                                acc[ip] = XS ? fmaf(s, dd[0] - __ldg(a.xsum + xr * nb + b), acc[ip])
                                             : fmaf(s, dd[0], acc[ip]);
                            }
                        }
                }
#pragma unroll
                for (int ip = 0; ip < RPW; ++ip) {
                    float v = acc[ip];
                    v += __shfl_xor_sync(0xffffffffu, v, 1);
                    v += __shfl_xor_sync(0xffffffffu, v, 2);
                    v += __shfl_xor_sync(0xffffffffu, v, 4);
                    if (MODE == GEMV_ACT) {
                        const float up = __shfl_down_sync(0xffffffffu, v, 16);
                        if (rv[ip]) {
                            if (W.l8 == 0 && a.gu_out) a.gu_out[po * a.gu_stride + row[ip]] = v;
                            if (W.lane == 0 || W.lane == 8)
                                a.out[po * a.out_stride + arow[ip]] = act_fn(v, up, a.act);
                        }
                    } else if (rv[ip] && W.l8 == 0) {
                        a.out[po * a.out_stride + row[ip]] = v;
                    }
                }
            }
        }
    }
}

template <int MODE, bool XS, int NBL, int RPW>
static void gemv_launch_t(const GemvArgs& a, int num_sms, cudaStream_t s) {
    const int rows_per_item = (MODE == GEMV_ACT) ? 2 * RPW : 4 * RPW;
    const int64_t tile_rows = (MODE == GEMV_ACT) ? a.F : a.rows_per_expert;
    const int64_t n_groups = (tile_rows + rows_per_item - 1) / rows_per_item;
    const int64_t items =
        n_groups * (a.dense_tokens > 0 ? (a.dense_tokens + DENSE_CHUNK - 1) / DENSE_CHUNK : a.max_unique);
    const int64_t blocks = (items + 3) / 4;
    const int64_t cap = (int64_t)num_sms * 16;
    const int grid = (int)(blocks < cap ? blocks : cap);
    if (grid <= 0) return;
    launch_k(k_q4_gemv<MODE, XS, NBL, RPW>, dim3(grid), dim3(128), 0, s, a);
}

template <int MODE, bool XS>
static void gemv_dispatch(const GemvArgs& a, int num_sms, cudaStream_t s) {
    const int nb = a.K / 32, nbl = (nb + 7) / 8;
    if (nbl == 11)
        gemv_launch_t<MODE, XS, 11, 1>(a, num_sms, s);  // K in (2560, 2816]
    else if (nbl <= 3)
        gemv_launch_t<MODE, XS, 3, 2>(a, num_sms, s);   // K <= 768 (704: down projection)
    else
        gemv_launch_t<MODE, XS, 8, 1>(a, num_sms, s);   // other K, chunked beyond 2048
}

int launch_gemv(int mode, const GemvArgs& a, int num_sms, cudaStream_t s) {
    const bool xs = a.xsum != nullptr;
    if (mode == GEMV_ACT) {
        if (xs) gemv_dispatch<GEMV_ACT, true>(a, num_sms, s);
        else gemv_dispatch<GEMV_ACT, false>(a, num_sms, s);
    } else {
        if (xs) gemv_dispatch<GEMV_PLAIN, true>(a, num_sms, s);
        else gemv_dispatch<GEMV_PLAIN, false>(a, num_sms, s);
    }
    return 1;
}

// fp32 router (the literal reading of the configs' "router weight fp32"):
// out[t][e] = W[e] . X[t]; one warp per (token, expert), float4 loads.
__global__ void __launch_bounds__(128) k_gemv_f32(const float* W, const float* X, float* out,
                                                  int64_t M, int64_t E, int64_t d) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t gw = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (gw >= M * E) return;
    const int64_t t = gw / E, e = gw - t * E;
    const float4* w4 = reinterpret_cast<const float4*>(W + e * d);
    const float4* x4 = reinterpret_cast<const float4*>(X + t * d);
    float acc = 0.f;
    for (int64_t j = lane; j < d / 4; j += 32) {
        const float4 a = __ldg(w4 + j), b = __ldg(x4 + j);
        acc = fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, acc))));
    }
    acc = warp_sum(acc);
    if (lane == 0) out[t * E + e] = acc;
}

int launch_gemv_f32(const float* W, const float* X, float* out, int64_t M, int64_t E, int64_t d,
                    cudaStream_t s) {
    const int64_t warps = M * E;
    if (warps <= 0) return 0;
    launch_k(k_gemv_f32, dim3((unsigned)((warps + 3) / 4)), dim3(128), 0, s, W, X, out, M, E, d);
    return 1;
}

// ------------------------------------------------------------ wide GEMV
// Dense Q4_0 GEMV for few rows and few tokens (the router: 128 rows): one
// warp per (row, chunk of up to 4 tokens), lanes across K (lane takes blocks
// lane, lane+32, ...), exact (n-8) dequant, fp32 FMA, full-warp reduction.
// Token chunks vary slowest so the warps of an SM share the activation rows
// in L1.
template <int T>
__global__ void __launch_bounds__(256) k_gemv_wide(const uint8_t* __restrict__ W, const float* __restrict__ S,
                                                   const float* __restrict__ X, float* __restrict__ out,
                                                   int64_t rows, int K, int ntok, int64_t out_stride) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nb = K >> 5;
    const int64_t chunks = (ntok + T - 1) / T;
    if (gw >= rows * chunks) return;
    const int64_t r = gw % rows;
    const int t0 = (int)(gw / rows) * T;
    const int nt = min(T, ntok - t0);
    float acc[T];
#pragma unroll
    for (int t = 0; t < T; ++t) acc[t] = 0.f;
    const uint8_t* wr = W + r * (K >> 1);
    const float* sr = S + r * nb;
    for (int b = lane; b < nb; b += 32) {
        const uint4 q = ldg_stream(wr + b * 16);
        const float s = __ldg(sr + b);
        const float* xp[T];
#pragma unroll
        for (int t = 0; t < T; ++t) xp[t] = X + (int64_t)(t0 + (t < nt ? t : 0)) * K + b * 32;
        float d[T];
        block_dot<false, T>(q, xp, d);
#pragma unroll
        for (int t = 0; t < T; ++t) acc[t] = fmaf(s, d[t], acc[t]);
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const float v = warp_sum(acc[t]);
        if (lane == 0 && t < nt) out[(int64_t)(t0 + t) * out_stride + r] = v;
    }
}

int launch_gemv_wide(const uint8_t* W, const float* S, const float* X, float* out, int64_t rows, int K,
                     int ntok, int64_t out_stride, cudaStream_t s) {
    if (rows <= 0 || ntok <= 0) return 0;
    const int T = ntok >= 4 ? 4 : (ntok >= 2 ? 2 : 1);
    const int64_t warps = rows * ((ntok + T - 1) / T);
    const unsigned blocks = (unsigned)((warps + 7) / 8);
    if (T == 4) launch_k(k_gemv_wide<4>, dim3(blocks), dim3(256), 0, s, W, S, X, out, rows, K, ntok, out_stride);
    else if (T == 2) launch_k(k_gemv_wide<2>, dim3(blocks), dim3(256), 0, s, W, S, X, out, rows, K, ntok, out_stride);
    else launch_k(k_gemv_wide<1>, dim3(blocks), dim3(256), 0, s, W, S, X, out, rows, K, ntok, out_stride);
    return 1;
}

// ------------------------------------------------------------ router (few tokens)
// Router logits of M <= 16 tokens as partial sums over K slices: CTA c takes
// the slice [c*RS, (c+1)*RS) of every token (staged in shared memory) and
// thread (e, token group) dots router row e's slice with the group's tokens;
// every thread loads its row's blocks before using them, and the 32 threads
// of a warp read the same activations (broadcast).  part[c][t][e] is summed
// over c, in c order, by k_topk.
constexpr int RS = 128;  // K slice per CTA (4 Q4 blocks)
// J: tokens per thread group (4 groups of 128 threads): M <= 4 * J.  `xs`
// holds RS floats per token in shared memory.
template <int J>
__device__ __forceinline__ void router_slice_dot(const uint8_t* __restrict__ W, const float* __restrict__ S, int M,
                                                 int K, int E, float* __restrict__ part, int c, const float* xs) {
    const int k0 = c * RS, tid = threadIdx.x;
    const int tg = tid >> 7, TG = blockDim.x >> 7;
    for (int e0 = 0; e0 < E; e0 += 128) {
        const int e = e0 + (tid & 127);
        if (e >= E) continue;
        uint4 q[RS / 32];
        float sc[RS / 32];
#pragma unroll
        for (int b = 0; b < RS / 32; ++b) {
            q[b] = ldg_stream(W + (int64_t)e * (K / 2) + k0 / 2 + b * 16);
            sc[b] = ldg_stream_f(S + (int64_t)e * (K / 32) + k0 / 32 + b);
        }
        float acc[J];
#pragma unroll
        for (int j = 0; j < J; ++j) acc[j] = 0.f;
#pragma unroll
        for (int b = 0; b < RS / 32; ++b) {
            const uint32_t w4[4] = {q[b].x, q[b].y, q[b].z, q[b].w};
            float wv[32];
#pragma unroll
            for (int w = 0; w < 4; ++w)
#pragma unroll
                for (int n = 0; n < 8; ++n)  // element 8w+n: nibble n of word w
                    wv[8 * w + n] = (float)((int)((w4[w] >> (4 * n)) & 15u) - 8);
#pragma unroll
            for (int j = 0; j < J; ++j) {
                const int t = tg + TG * j;
                if (t < M) {
                    const float4* xp = reinterpret_cast<const float4*>(xs + t * RS + b * 32);
                    float d = 0.f;
#pragma unroll
                    for (int v = 0; v < 8; ++v) {
                        const float4 x4 = xp[v];
                        d = fmaf(wv[4 * v], x4.x, d);
                        d = fmaf(wv[4 * v + 1], x4.y, d);
                        d = fmaf(wv[4 * v + 2], x4.z, d);
                        d = fmaf(wv[4 * v + 3], x4.w, d);
                    }
                    acc[j] = fmaf(sc[b], d, acc[j]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const int t = tg + TG * j;
            if (t < M) part[((int64_t)c * M + t) * E + e] = acc[j];
        }
    }
}

template <int J>
__device__ __forceinline__ void router_slice(const uint8_t* __restrict__ W, const float* __restrict__ S,
                                             const float* __restrict__ X, int M, int K, int E,
                                             float* __restrict__ part, int c, float* xs) {
    const int k0 = c * RS, tid = threadIdx.x;
    for (int i = tid; i < M * RS / 4; i += blockDim.x) {
        const int t = (i * 4) / RS, k = (i * 4) % RS;
        reinterpret_cast<float4*>(xs + t * RS)[k / 4] =
            __ldg(reinterpret_cast<const float4*>(X + (int64_t)t * K + k0 + k));
    }
    __syncthreads();
    router_slice_dot<J>(W, S, M, K, E, part, c, xs);
}

__global__ void __launch_bounds__(512) k_router_part(const uint8_t* __restrict__ W, const float* __restrict__ S,
                                                     const float* __restrict__ X, int M, int K, int E,
                                                     float* __restrict__ part) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) {  // weights: ahead of the dependency wait
        asm volatile("prefetch.global.L2 [%0];" ::"l"(W + (int64_t)e * (K / 2) + blockIdx.x * RS / 2));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(S + (int64_t)e * (K / 32) + blockIdx.x * RS / 32));
    }
    pdl_wait();
    pdl_trigger();
    __shared__ __align__(16) float xs[16 * RS];
    router_slice<4>(W, S, X, M, K, E, part, blockIdx.x, xs);
}

bool router_part_supported(int M, int K) { return M >= 1 && M <= 16 && K % RS == 0; }

int launch_router_part(const uint8_t* W, const float* S, const float* X, int M, int K, int E, float* part,
                       cudaStream_t s) {
    launch_k(k_router_part, dim3(K / RS), dim3(512), 0, s, W, S, X, M, K, E, part);
    return 1;
}

// ------------------------------------------------------------ row prep
// One CTA per row: layout conversion (moe_x_layout), fp16 -> fp32, optional
// rms norms (model_speculative_moe_batched.mojo:857-879): out = x * inv *
// pre_w and scaled = x * inv * router_scale * r_scale_factor; and the
// per-32-block sums (x1.5) the XS GEMV needs.
// One step of a thread's sum of squares over float4 elements (shared by
// every kernel that forms the rms of a row, so that they agree bit for bit).
__device__ __forceinline__ float ss_step(float ss, const float4 v) {
    return ss + (v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
}

// Row t of the prep; `xs` holds K floats of shared memory, `red` 33.
__device__ __forceinline__ void prep_row(const PrepArgs& a, int64_t t, float* xs, float* red) {
    const int64_t K = a.K;
    float ss = 0.f;
    if (a.x_layout == 0 && !a.x_f16 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0) {
        // natural fp32 rows: float4 loads, several in flight per thread
        const float4* x4 = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.x) + t * K);
#pragma unroll 4
        for (int64_t j = threadIdx.x; j < K / 4; j += blockDim.x) {
            const float4 v = __ldg(x4 + j);
            reinterpret_cast<float4*>(xs)[j] = v;
            ss = ss_step(ss, v);
        }
    } else {
#pragma unroll 4
        for (int64_t j = threadIdx.x; j < K; j += blockDim.x) {
            const int64_t si = t * K + x_src_index(j, K, a.x_layout);
            const float v = a.x_f16 ? __half2float(reinterpret_cast<const __half*>(a.x)[si])
                                    : reinterpret_cast<const float*>(a.x)[si];
            xs[j] = v;
            ss += v * v;
        }
    }
    float inv = 1.f;
    if (a.norm) {
        ss = block_sum(ss, red);
        inv = 1.0f / sqrtf(ss / (float)K + 1e-6f);
    } else {
        __syncthreads();
    }
#pragma unroll 4
    for (int64_t j = threadIdx.x; j < K; j += blockDim.x) {
        const float v = xs[j];
        if (a.scaled) a.scaled[t * K + j] = v * inv * __ldg(a.router_scale + j) * a.rsf;
        const float o = a.norm ? v * inv * __ldg(a.pre_w + j) : v;
        xs[j] = o;
        a.out[t * K + j] = o;
        if (a.out_q) a.out_q[t * K + qpos(j)] = o * qscale(j);
    }
    if (a.out_sum) {
        __syncthreads();
        const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
        for (int64_t b = w; b < K / 32; b += nw) {
            const float s = warp_sum(xs[b * 32 + lane]);
            if (lane == 0) a.out_sum[t * (K / 32) + b] = 1.5f * s;
        }
    }
}

__global__ void __launch_bounds__(512) k_prep(PrepArgs a) {
    if (a.norm) prefetch_l2(a.pre_w, a.K * 4);  // weights: ahead of the dependency wait
    if (a.scaled) prefetch_l2(a.router_scale, a.K * 4);
    pdl_wait();
    pdl_trigger();
    extern __shared__ float4 smem4[];
    __shared__ float red[33];
    prep_row(a, blockIdx.x, reinterpret_cast<float*>(smem4), red);
}

int launch_prep(const PrepArgs& a, int64_t M, cudaStream_t s) {
    if (M <= 0) return 0;
    const size_t smem = (size_t)a.K * sizeof(float);
    if (smem > 48 * 1024) cudaFuncSetAttribute(k_prep, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_k(k_prep, dim3((unsigned)M), dim3(512), smem, s, a);
    return 1;
}

// ------------------------------------------------------ softmax + top-k + LOD
// One CTA per token on the router scores: softmax (model_speculative_moe_
// batched.mojo:921-933), top-k with insertion semantics (:936-953; equal
// values keep the lower index first) and, when a.lod,
// compute_moe_lod_weights (moe_kernels.mojo:445-490).
__device__ __forceinline__ void topk_finish(const TopkArgs& a, int64_t t, const float* tval, const int* tidx,
                                            const float* pes);

// Token t: `pr` holds E floats of shared memory, `red` 33, tval / tidx 32.
__device__ __forceinline__ void topk_row(const TopkArgs& a, int64_t t, float* pr, float* red, float* tval,
                                         int* tidx, float* pes_s) {
    const int E = a.E, K = a.K;
    for (int e = threadIdx.x; e < E; e += blockDim.x) pes_s[e] = __ldg(a.pes + e);
    float m = -INFINITY;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        float sc;
        if (a.part_n > 0) {  // router partial sums over K slices, in slice order
            sc = 0.f;
            // up to 32 loads in flight (one L2 round trip for d <= 4096), then
            // the sum in slice order
            for (int c0 = 0; c0 < a.part_n; c0 += 32) {
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    v[j] = c0 + j < a.part_n ? __ldg(a.part + ((int64_t)(c0 + j) * a.M + t) * E + e) : 0.f;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (c0 + j < a.part_n) sc += v[j];
            }
            if (a.scores_out) a.scores_out[t * E + e] = sc;
        } else {
            sc = a.scores[t * E + e];
        }
        const float v = sc + (a.bias ? a.bias[e] : 0.f);
        pr[e] = v;
        m = fmaxf(m, v);
    }
    m = block_max(m, red);
    float se = 0.f;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const float v = expf(pr[e] - m);
        pr[e] = v;
        se += v;
    }
    se = block_sum(se, red);
    const float den = se + 1e-10f;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        pr[e] = pr[e] / den;
        if (a.probs_out) a.probs_out[t * E + e] = pr[e];
    }
    if (threadIdx.x < K) {
        tval[threadIdx.x] = -999999.0f;
        tidx[threadIdx.x] = -1;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
        const float pi = pr[i];
        if (pi == pi) {
            int rank = 0;
            for (int j = 0; j < E; ++j) {
                const float pj = pr[j];
                rank += (pj > pi) || (pj == pi && j < i);
            }
            if (rank < K) {
                tval[rank] = pi;
                tidx[rank] = i;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    topk_finish(a, t, tval, tidx, pes_s);
}

// Outputs of token t from its top-k values and ids (one thread): the top-k
// arrays, then (a.lod) compute_moe_lod_weights (moe_kernels.mojo:445-490)
// into the slot table and the reference's per-token lists.
// `pes` is per_expert_scale, staged in shared memory by the caller: the LOD
// loop below reads it slot by slot, and from global memory each read would
// be a dependent round trip.
__device__ __forceinline__ void topk_finish(const TopkArgs& a, int64_t t, const float* tval, const int* tidx,
                                            const float* pes) {
    const int K = a.K;
    for (int k = 0; k < K; ++k) {
        if (a.top_idx) a.top_idx[t * K + k] = tidx[k];
        if (a.top_val) a.top_val[t * K + k] = tval[k];
        a.ti32[t * K + k] = tidx[k];
        a.tv[t * K + k] = tval[k];
    }
    if (!a.lod) return;
    float sum = 0.f;
    for (int k = 0; k < K; ++k) sum += tval[k];
    const float inv_sum = 1.0f / (sum + 1e-10f);
    const float tp = (a.top_p == a.top_p) ? a.top_p : 1.0f;
    int cnt = 0;
    int oi[32];
    float ow[32];
    if (tp >= 1.0f) {
        for (int k = 0; k < K; ++k) {
            const float np_ = tval[k] * inv_sum;
            if ((np_ >= 0.05f || k == 0) && tidx[k] >= 0) {
                const int e = tidx[k];
                oi[cnt] = e;
                ow[cnt] = np_ * pes[e];
                ++cnt;
            }
        }
    } else {
        float cum = 0.f;
        for (int k = 0; k < K; ++k) {
            const float np_ = tval[k] * inv_sum;
            if (k > 0 && (np_ < 0.05f || cum >= tp)) break;
            if (tidx[k] < 0) break;
            oi[cnt] = tidx[k];
            ow[cnt] = np_;
            cum += np_;
            ++cnt;
        }
        const float rn = 1.0f / (cum + 1e-10f);
        for (int k = 0; k < cnt; ++k) ow[k] = (ow[k] * rn) * pes[oi[k]];
    }
    for (int k = 0; k < K; ++k) {
        const bool on = k < cnt;
        a.slot_expert[t * K + k] = on ? oi[k] : -1;
        a.slot_weight[t * K + k] = on ? ow[k] : 0.f;
        if (a.tok_idx) a.tok_idx[t * K + k] = on ? oi[k] : 0;
        if (a.tok_w) a.tok_w[t * K + k] = on ? ow[k] : 0.f;
    }
    if (a.tok_count) a.tok_count[t] = cnt;
}

__global__ void __launch_bounds__(128) k_topk(TopkArgs a) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ float4 smem4[];
    __shared__ float red[33];
    __shared__ float tval[32];
    __shared__ int tidx[32];
    topk_row(a, blockIdx.x, reinterpret_cast<float*>(smem4), red, tval, tidx,
             reinterpret_cast<float*>(smem4) + a.E);
}

int launch_topk(const TopkArgs& a, int64_t M, cudaStream_t s) {
    if (M <= 0) return 0;
    const size_t smem = (size_t)a.E * 2 * sizeof(float);
    launch_k(k_topk, dim3((unsigned)M), dim3(128), smem, s, a);
    return 1;
}

// ---------------------------------------------------------------- set cover
// compute_subbatch_set_cover_moe_weights (moe_kernels.mojo:493-611), one
// thread per sub-batch of `sub_batch` tokens (5 in the engine).
__global__ void k_set_cover(const int* ti, const float* tv, int64_t M, int K, int E,
                            const float* pes, float top_p, float core_top_p, float smp,
                            int sub_batch, int* slot_expert, float* slot_weight,
                            int64_t* tok_count, int64_t* tok_idx, float* tok_w) {
    pdl_wait();
    pdl_trigger();
    const int64_t t0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * sub_batch;
    if (t0 >= M) return;
    const int sb = (int)min((int64_t)sub_batch, M - t0);
    const float safe = (top_p == top_p) ? top_p : 1.0f;
    int cnt_out[64];
    int oi[64][32];
    float ow[64][32];
    // anchor token: compute_moe_lod_weights
    {
        const int* i0 = ti + t0 * K;
        const float* v0 = tv + t0 * K;
        float sum = 0.f;
        for (int k = 0; k < K; ++k) sum += v0[k];
        const float inv = 1.0f / (sum + 1e-10f);
        int c = 0;
        if (safe >= 1.0f) {
            for (int k = 0; k < K; ++k) {
                const float np_ = v0[k] * inv;
                if ((np_ >= 0.05f || k == 0) && i0[k] >= 0 && i0[k] < E) {
                    oi[0][c] = i0[k];
                    ow[0][c] = np_ * pes[i0[k]];
                    ++c;
                }
            }
        } else {
            float cum = 0.f;
            for (int k = 0; k < K; ++k) {
                const float np_ = v0[k] * inv;
                if (k > 0 && (np_ < 0.05f || cum >= safe)) break;
                if (i0[k] < 0 || i0[k] >= E) break;
                oi[0][c] = i0[k];
                ow[0][c] = np_;
                cum += np_;
                ++c;
            }
            const float rn = 1.0f / (cum + 1e-10f);
            for (int k = 0; k < c; ++k) ow[0][k] = (ow[0][k] * rn) * pes[oi[0][k]];
        }
        cnt_out[0] = c;
    }
    uint8_t in_pool[256], freq[256];
    for (int i = 0; i < 256; ++i) in_pool[i] = freq[i] = 0;
    for (int k = 0; k < cnt_out[0]; ++k) {
        const int e0 = oi[0][k];
        if (e0 >= 0 && e0 < 256) {
            in_pool[e0] = 1;
            freq[e0] = 1;
        }
    }
    float inv_s[64], elig[64];
    for (int b = 1; b < sb; ++b) {
        const int* ib = ti + (t0 + b) * K;
        const float* vb = tv + (t0 + b) * K;
        float s = 0.f;
        for (int k = 0; k < K; ++k) s += vb[k];
        const float is = 1.0f / (s + 1e-10f);
        inv_s[b] = is;
        float cum = 0.f;
        for (int k = 0; k < K; ++k) {
            const float np_ = vb[k] * is;
            if (safe >= 1.0f) {
                if (np_ < 0.05f && k > 0) continue;
            } else if (k > 0 && (np_ < 0.05f || cum >= safe)) {
                break;
            }
            const int e = ib[k];
            if (e >= 0 && e < 256) {
                freq[e] = (uint8_t)(freq[e] + 1);
                if (k < 2 || np_ >= smp || cum < core_top_p) in_pool[e] = 1;
            }
            cum += np_;
        }
        elig[b] = cum;
    }
    for (int b = 1; b < sb; ++b) {
        const int* ib = ti + (t0 + b) * K;
        const float* vb = tv + (t0 + b) * K;
        float cum = 0.f, kept = 0.f;
        int c = 0;
        bool pruned = false;
        for (int k = 0; k < K; ++k) {
            const float np_ = vb[k] * inv_s[b];
            if (safe >= 1.0f) {
                if (np_ < 0.05f && k > 0) continue;
            } else if (k > 0 && (np_ < 0.05f || cum >= safe)) {
                break;
            }
            const int e = ib[k];
            const bool core = (k < 2) || (np_ >= smp) || (cum < core_top_p);
            const bool shared = (e >= 0 && e < 256) && (in_pool[e] != 0 || freq[e] >= 2);
            cum += np_;
            if ((core || shared) && e >= 0 && e < E) {
                oi[b][c] = e;
                ow[b][c] = np_;
                kept += np_;
                ++c;
            } else {
                pruned = true;
            }
        }
        const float target = (safe < 1.0f) ? 1.0f : elig[b];
        const float rn = (pruned || safe < 1.0f) ? (target / (kept + 1e-10f)) : 1.0f;
        for (int k = 0; k < c; ++k) ow[b][k] = (ow[b][k] * rn) * pes[oi[b][k]];
        cnt_out[b] = c;
    }
    for (int b = 0; b < sb; ++b) {
        const int64_t t = t0 + b;
        for (int k = 0; k < K; ++k) {
            const bool on = k < cnt_out[b];
            if (slot_expert) slot_expert[t * K + k] = on ? oi[b][k] : -1;
            if (slot_weight) slot_weight[t * K + k] = on ? ow[b][k] : 0.f;
            if (tok_idx) tok_idx[t * K + k] = on ? oi[b][k] : 0;
            if (tok_w) tok_w[t * K + k] = on ? ow[b][k] : 0.f;
        }
        if (tok_count) tok_count[t] = cnt_out[b];
    }
}

int launch_set_cover(const int* ti32, const float* tv, int64_t M, int K, int E, const float* pes,
                     float top_p, float core_top_p, float smp, int sub_batch, int* slot_expert,
                     float* slot_weight, int64_t* tok_count, int64_t* tok_idx, float* tok_w,
                     cudaStream_t s) {
    if (M <= 0) return 0;
    const int64_t groups = (M + sub_batch - 1) / sub_batch;
    const int threads = 32;
    const int blocks = (int)((groups + threads - 1) / threads);
    launch_k(k_set_cover, dim3(blocks), dim3(threads), 0, s, ti32, tv, M, K, E, pes, top_p, core_top_p, smp,
                                           sub_batch, slot_expert, slot_weight, tok_count,
                                           tok_idx, tok_w);
    return 1;
}

// -------------------------------------------------------- slot conversions
// Compact per-token lists (count + int64 ids, as compute_moe_lod_weights
// returns them) -> internal [M][K] slot table.  Out-of-range ids raise
// err_flag and are dropped.
__global__ void k_slots_from_lists(int64_t M, int K, const int64_t* count, int64_t count_scalar,
                                   const int64_t* idx, const float* w, int* slot_expert,
                                   float* slot_weight, int E, int* err_flag) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= M * K) return;
    const int64_t t = i / K;
    const int k = (int)(i - t * K);
    const int64_t c = count ? count[t] : count_scalar;
    int e = -1;
    float wt = 0.f;
    if (k < c) {
        const int64_t v = idx[i];
        if (v >= 0 && v < E) {
            e = (int)v;
            wt = w ? w[i] : 0.f;
        } else {
            atomicExch(err_flag, 1);
        }
    }
    slot_expert[i] = e;
    slot_weight[i] = wt;
}

int launch_slots_from_lists(int64_t M, int K, const int64_t* count, int64_t count_scalar,
                            const int64_t* idx, const float* w, int* slot_expert,
                            float* slot_weight, int E, int* err_flag, cudaStream_t s) {
    const int64_t n = M * K;
    if (n <= 0) return 0;
    launch_k(k_slots_from_lists, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, 
        M, K, count, count_scalar, idx, w, slot_expert, slot_weight, E, err_flag);
    return 1;
}

// Diffusion convention (diffusion_kernels.mojo:263-266): slot active iff w > 0.
__global__ void k_slots_from_topw(int64_t n, const int64_t* idx, const float* w, int* slot_expert,
                                  float* slot_weight, int E, int* err_flag) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int e = -1;
    float wt = 0.f;
    if (w[i] > 0.0f) {
        const int64_t v = idx[i];
        if (v >= 0 && v < E) {
            e = (int)v;
            wt = w[i];
        } else {
            atomicExch(err_flag, 1);
        }
    }
    slot_expert[i] = e;
    slot_weight[i] = wt;
}

int launch_slots_from_topw(int64_t M, int K, const int64_t* idx, const float* w, int* slot_expert,
                           float* slot_weight, int E, int* err_flag, cudaStream_t s) {
    const int64_t n = M * K;
    if (n <= 0) return 0;
    launch_k(k_slots_from_topw, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, n, idx, w, slot_expert,
                                                                  slot_weight, E, err_flag);
    return 1;
}

// ------------------------------------------------------------------ bucket
// Groups the (token, slot) pairs by expert, ascending expert id, like the
// Hoare bucket sort of moe_kernels.mojo:815-835.  Order inside a bucket is
// not fixed (atomics): every pair's result is computed independently, so
// outputs do not depend on it.  One CTA of 1024 threads; E <= 1024.
__device__ __forceinline__ int block_excl_scan(int v, int* wsum, int* total) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) wsum[wid] = x;
    __syncthreads();
    if (wid == 0) {
        int w = lane < nw ? wsum[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < nw) wsum[lane] = w;
    }
    __syncthreads();
    const int base = wid > 0 ? wsum[wid - 1] : 0;
    const int tot = wsum[nw - 1];
    __syncthreads();
    *total = tot;
    return base + x - v;
}

// Pairs whose expert lies outside [e_lo, e_hi) are left out (expert
// parallelism: this rank holds only those experts); their slots get no pair.
// With tt_prefix, also the exclusive prefix of token tiles of BN tokens per
// unique expert (the tensor-core work list), one launch fewer.
// The bucketing by one CTA of at least E threads; cnt / cur hold blockDim
// ints of shared memory, wsum 32.
__device__ __forceinline__ void bucket_block(const int* slot_expert, int64_t P, int K, int E, int e_lo, int e_hi,
                                             const BucketOut& o, int BN, int* tt_prefix, int* cnt, int* cur,
                                             int* wsum) {
    const int tid = threadIdx.x;
    cnt[tid] = 0;
    __syncthreads();
    for (int64_t p = tid; p < P; p += blockDim.x) {
        const int e = slot_expert[p];
        if (e >= e_lo && e < e_hi) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    const int c = tid < E ? cnt[tid] : 0;
    int total_pairs = 0, total_u = 0;
    const int off = block_excl_scan(c, wsum, &total_pairs);
    const int ui = block_excl_scan(c > 0 ? 1 : 0, wsum, &total_u);
    if (c > 0) {
        o.unique_expert[ui] = tid;
        o.seg_start[ui] = off;
        o.seg_count[ui] = c;
    }
    cur[tid] = off;
    if (tid == 0) {
        o.meta[0] = total_u;
        o.meta[1] = total_pairs;
    }
    if (tt_prefix) {  // unique experts are numbered in thread (expert) order
        int total_t = 0;
        const int toff = block_excl_scan(c > 0 ? (c + BN - 1) / BN : 0, wsum, &total_t);
        if (c > 0) tt_prefix[ui] = toff;
        if (tid == 0) tt_prefix[total_u] = total_t;
    }
    __syncthreads();
    for (int64_t p = tid; p < P; p += blockDim.x) {
        const int e = slot_expert[p];
        if (e >= e_lo && e < e_hi) {
            const int pos = atomicAdd(&cur[e], 1);
            o.pair_token[pos] = (int)(p / K);
            o.pair_slot[pos] = (int)p;
            o.slot_pair[p] = pos;
        } else {
            o.slot_pair[p] = -1;
        }
    }
}

__global__ void __launch_bounds__(1024) k_bucket(const int* slot_expert, int64_t P, int K, int E, int e_lo,
                                                 int e_hi, BucketOut o, int BN, int* tt_prefix) {
    pdl_wait();
    pdl_trigger();
    __shared__ int cnt[1024];
    __shared__ int cur[1024];
    __shared__ int wsum[32];
    bucket_block(slot_expert, P, K, E, e_lo, e_hi, o, BN, tt_prefix, cnt, cur, wsum);
}

int launch_bucket(const int* slot_expert, int64_t P, int K, int E, int e_lo, int e_hi, const BucketOut& o,
                  cudaStream_t s, int BN, int* tt_prefix) {
    launch_k(k_bucket, dim3(1), dim3(1024), 0, s, slot_expert, P, K, E, e_lo, e_hi, o, BN, tt_prefix);
    return 1;
}

// ----------------------------------------------------------------- combine
// moe_out[t][r] = sum over slots k (in slot order) of w_k * y[pair(t,k)][r]
// (moe_kernels.mojo:775-779, diffusion_kernels.mojo:386-399), then optionally
// rms_norm with post_feedforward_layernorm_2 (model_speculative_moe_batched
// .mojo:1144-1150) and fp16 rounding.  float4 per thread, d % 4 == 0.
__global__ void __launch_bounds__(512) k_combine(CombineArgs a) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[33];
    __shared__ int sp[32];
    __shared__ float sw[32];
    const int64_t t = blockIdx.x;
    const int K = a.K;
    if (threadIdx.x < K) {
        sp[threadIdx.x] = a.slot_pair[t * K + threadIdx.x];
        sw[threadIdx.x] = a.slot_weight[t * K + threadIdx.x];
    }
    __syncthreads();
    const int64_t d4 = a.d / 4;
    constexpr int MAXV = 6;  // 512 threads x 6 float4: d <= 12288 kept in registers
    float4 acc[MAXV];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int64_t j = threadIdx.x + (int64_t)i * blockDim.x;
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < d4) {
#pragma unroll 8
            for (int k = 0; k < K; ++k) {
                const int p = sp[k];
                if (p < 0) continue;
                float4 y = __ldg(reinterpret_cast<const float4*>(a.y + (size_t)p * a.d) + j);
                for (int ks = 1; ks < a.ksplit; ++ks) {  // split-K partials, fixed order
                    const float4 z = __ldg(reinterpret_cast<const float4*>(a.y + ks * a.split_stride +
                                                                           (size_t)p * a.d) + j);
                    y.x += z.x; y.y += z.y; y.z += z.z; y.w += z.w;
                }
                const float w = sw[k];
                if (a.fma_mode) {
                    s.x = fmaf(y.x, w, s.x); s.y = fmaf(y.y, w, s.y);
                    s.z = fmaf(y.z, w, s.z); s.w = fmaf(y.w, w, s.w);
                } else {
                    s.x = __fadd_rn(s.x, __fmul_rn(y.x, w)); s.y = __fadd_rn(s.y, __fmul_rn(y.y, w));
                    s.z = __fadd_rn(s.z, __fmul_rn(y.z, w)); s.w = __fadd_rn(s.w, __fmul_rn(y.w, w));
                }
            }
            ss += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
        }
        acc[i] = s;
    }
    float inv = 1.f;
    if (a.post_norm) {
        ss = block_sum(ss, red);
        inv = 1.0f / sqrtf(ss / (float)a.d + 1e-6f);
    }
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int64_t j = threadIdx.x + (int64_t)i * blockDim.x;
        if (j >= d4) continue;
        float4 v = acc[i];
        if (a.post_norm) {
            const float4 w = __ldg(reinterpret_cast<const float4*>(a.post_w) + j);
            v.x = v.x * inv * w.x; v.y = v.y * inv * w.y; v.z = v.z * inv * w.z; v.w = v.w * inv * w.w;
        }
        if (a.out_f16) {
            __half2* o = reinterpret_cast<__half2*>(a.out) + (t * a.d) / 2 + 2 * j;
            o[0] = __floats2half2_rn(v.x, v.y);
            o[1] = __floats2half2_rn(v.z, v.w);
        } else {
            reinterpret_cast<float4*>(a.out)[(t * a.d) / 4 + j] = v;
        }
    }
}

// The same per-token combine with a token's row split over a cluster of
// CW_CL CTAs (more CTAs in flight for small batches); the post-norm's sum of
// squares is added across the cluster through distributed shared memory, in
// cluster-rank order.
constexpr int CW_CL = 4;
__global__ void __launch_bounds__(256) k_combine_cl(CombineArgs a) {
    if (a.post_norm) {  // the norm weights of this CTA's part of the row, ahead of the dependency wait
        const int64_t per = a.d / CW_CL;
        const char* w = reinterpret_cast<const char*>(a.post_w + cl_rank() * per);
        for (int64_t o = (int64_t)threadIdx.x * 128; o < per * 4; o += (int64_t)blockDim.x * 128)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(w + o));
    }
    pdl_wait();
    pdl_trigger();
    __shared__ float red[33];
    __shared__ int sp[32];
    __shared__ float sw[32];
    __shared__ float parts[CW_CL];
    const uint32_t r = cl_rank();
    const int64_t t = blockIdx.x / CW_CL;
    const int K = a.K;
    if (threadIdx.x < K) {
        sp[threadIdx.x] = a.slot_pair[t * K + threadIdx.x];
        sw[threadIdx.x] = a.slot_weight[t * K + threadIdx.x];
    }
    cl_sync();  // every CTA of the cluster runs before shared memory is exchanged
    const int64_t d4 = a.d / 4, per = d4 / CW_CL, j0 = (int64_t)r * per;
    constexpr int MAXV = 3;  // 256 threads x 3 float4 x 4 CTAs: d <= 12288
    float4 acc[MAXV];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int64_t jj = threadIdx.x + (int64_t)i * blockDim.x;
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        if (jj < per) {
            const int64_t j = j0 + jj;
#pragma unroll 8
            for (int k = 0; k < K; ++k) {
                const int p = sp[k];
                if (p < 0) continue;
                float4 y = __ldg(reinterpret_cast<const float4*>(a.y + (size_t)p * a.d) + j);
                for (int ks = 1; ks < a.ksplit; ++ks) {  // split-K partials, fixed order
                    const float4 z = __ldg(reinterpret_cast<const float4*>(a.y + ks * a.split_stride +
                                                                           (size_t)p * a.d) + j);
                    y.x += z.x; y.y += z.y; y.z += z.z; y.w += z.w;
                }
                const float w = sw[k];
                if (a.fma_mode) {
                    s.x = fmaf(y.x, w, s.x); s.y = fmaf(y.y, w, s.y);
                    s.z = fmaf(y.z, w, s.z); s.w = fmaf(y.w, w, s.w);
                } else {
                    s.x = __fadd_rn(s.x, __fmul_rn(y.x, w)); s.y = __fadd_rn(s.y, __fmul_rn(y.y, w));
                    s.z = __fadd_rn(s.z, __fmul_rn(y.z, w)); s.w = __fadd_rn(s.w, __fmul_rn(y.w, w));
                }
            }
            ss += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
        }
        acc[i] = s;
    }
    float inv = 1.f;
    if (a.post_norm) {
        ss = block_sum(ss, red);
        if (threadIdx.x == 0) cl_st(cl_map(&parts[r], 0), ss);
    }
    cl_sync();
    if (a.post_norm) {
        float tot = 0.f;
        for (int i = 0; i < CW_CL; ++i) tot += cl_ldf(cl_map(&parts[i], 0));
        inv = 1.0f / sqrtf(tot / (float)a.d + 1e-6f);
    }
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int64_t jj = threadIdx.x + (int64_t)i * blockDim.x;
        if (jj >= per) continue;
        const int64_t j = j0 + jj;
        float4 v = acc[i];
        if (a.post_norm) {
            const float4 w = __ldg(reinterpret_cast<const float4*>(a.post_w) + j);
            v.x = v.x * inv * w.x; v.y = v.y * inv * w.y; v.z = v.z * inv * w.z; v.w = v.w * inv * w.w;
        }
        if (a.out_f16) {
            __half2* o = reinterpret_cast<__half2*>(a.out) + (t * a.d) / 2 + 2 * j;
            o[0] = __floats2half2_rn(v.x, v.y);
            o[1] = __floats2half2_rn(v.z, v.w);
        } else {
            reinterpret_cast<float4*>(a.out)[(t * a.d) / 4 + j] = v;
        }
    }
    cl_sync();  // CTA 0's shared memory stays alive until every CTA has read it
}

int launch_combine(const CombineArgs& a, int64_t M, cudaStream_t s) {
    if (M <= 0) return 0;
    if (M <= 64 && (a.d / 4) % CW_CL == 0 && a.d <= 12288) {  // small batches: more CTAs per token
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(M * CW_CL));
        cfg.blockDim = dim3(256);
        cfg.stream = s;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = CW_CL;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        cudaLaunchKernelEx(&cfg, k_combine_cl, a);
        return 1;
    }
    launch_k(k_combine, dim3((unsigned)M), dim3(512), 0, s, a);
    return 1;
}

// ---------------------------------------------------------------- quantize
// quantize_fp32_to_q4_0 (moe_kernels.mojo:7-56): one thread per 32-block;
// IEEE division (no fast-math) so scale and 1/scale match the reference bit
// for bit; rint rounds exact ties to even like numpy.
__global__ void k_quantize(const float* src, uint8_t* packed, float* scales, int64_t nblocks) {
    pdl_wait();
    pdl_trigger();
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const float4* s4 = reinterpret_cast<const float4*>(src + b * 32);
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 q = s4[i];
        v[4 * i] = q.x;
        v[4 * i + 1] = q.y;
        v[4 * i + 2] = q.z;
        v[4 * i + 3] = q.w;
    }
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) mx = fmaxf(mx, fabsf(v[i]));
    float scale = __fdiv_rn(mx, 7.0f);
    if (scale < 1e-5f) scale = 1e-5f;
    scales[b] = scale;
    const float inv = __fdiv_rn(1.0f, scale);
    uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        float q0 = rintf(__fmul_rn(v[2 * j], inv));
        float q1 = rintf(__fmul_rn(v[2 * j + 1], inv));
        q0 = fminf(fmaxf(q0, -8.0f), 7.0f);
        q1 = fminf(fmaxf(q1, -8.0f), 7.0f);
        const uint32_t byte = (uint32_t)((int)q0 + 8) | ((uint32_t)((int)q1 + 8) << 4);
        w[j >> 2] |= byte << (8 * (j & 3));
    }
    *reinterpret_cast<uint4*>(packed + b * 16) = make_uint4(w[0], w[1], w[2], w[3]);
}

int launch_quantize(const float* src, uint8_t* packed, float* scales, int64_t nblocks,
                    cudaStream_t s) {
    if (nblocks <= 0) return 0;
    launch_k(k_quantize, dim3((unsigned)((nblocks + 255) / 256)), dim3(256), 0, s, src, packed, scales, nblocks);
    return 1;
}

// ---------------------------------------------------------------- LOD APIs
__global__ void k_lod(int64_t B, const int64_t* top_idx, const float* top_val, const float* pes,
                      float top_p, int64_t* act_idx, float* act_w, int64_t* act_count, int K,
                      int64_t E, int* err_flag) {
    pdl_wait();
    pdl_trigger();
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= B) return;
    const int64_t* ti = top_idx + t * K;
    const float* tv = top_val + t * K;
    int64_t* ai = act_idx + t * K;
    float* aw = act_w + t * K;
    float sum = 0.f;
    for (int k = 0; k < K; ++k) sum += tv[k];
    const float inv = 1.0f / (sum + 1e-10f);
    const float safe = (top_p == top_p) ? top_p : 1.0f;
    int64_t c = 0;
    if (safe >= 1.0f) {
        for (int k = 0; k < K; ++k) {
            const float np_ = tv[k] * inv;
            if (np_ >= 0.05f || k == 0) {
                if (ti[k] < 0 || ti[k] >= E) {
                    atomicExch(err_flag, 1);
                    continue;
                }
                ai[c] = ti[k];
                aw[c] = np_ * pes[ti[k]];
                ++c;
            }
        }
    } else {
        float cum = 0.f;
        for (int k = 0; k < K; ++k) {
            const float np_ = tv[k] * inv;
            if (k > 0 && (np_ < 0.05f || cum >= safe)) break;
            if (ti[k] < 0 || ti[k] >= E) {
                atomicExch(err_flag, 1);
                break;
            }
            ai[c] = ti[k];
            aw[c] = np_;
            cum += np_;
            ++c;
        }
        const float rn = 1.0f / (cum + 1e-10f);
        for (int64_t k = 0; k < c; ++k) aw[k] = (aw[k] * rn) * pes[ai[k]];
    }
    act_count[t] = c;
}

int launch_lod(int64_t B, const int64_t* top_idx, const float* top_val, const float* pes,
               float top_p, int64_t* act_idx, float* act_w, int64_t* act_count, int K,
               int64_t E, int* err_flag, cudaStream_t s) {
    if (B <= 0) return 0;
    launch_k(k_lod, dim3((unsigned)((B + 127) / 128)), dim3(128), 0, s, B, top_idx, top_val, pes, top_p, act_idx,
                                                       act_w, act_count, K, E, err_flag);
    return 1;
}

// apply_moe_lod_and_set_cover (diffusion_kernels.mojo:3607-3664)
__global__ void k_apply_lod(const int64_t* top_idx, const float* top_val, const float* pes,
                            float* top_w, int64_t B, int K, int64_t eff_k, int64_t unacc_k,
                            const uint8_t* eb_mask, const int64_t* active_canvas_idx) {
    pdl_wait();
    pdl_trigger();
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const int64_t orig = active_canvas_idx ? active_canvas_idx[b] : b;
    const bool accepted = eb_mask ? (eb_mask[orig] != 0) : true;
    const int64_t tok_k = accepted ? eff_k : unacc_k;
    const int64_t* ti = top_idx + b * K;
    const float* tv = top_val + b * K;
    float* tw = top_w + b * K;
    float sd = 0.f;
    for (int64_t s = 0; s < tok_k; ++s)
        if (ti[s] >= 0) sd += tv[s];
    const float inv = 1.0f / (sd + 1e-10f);
    for (int s = 0; s < K; ++s) {
        const int64_t e = ti[s];
        const float np_ = tv[s] * inv;
        tw[s] = (s < tok_k && e >= 0 && e < 128 && np_ >= 0.05f) ? np_ * pes[e] : 0.0f;
    }
}

int launch_apply_lod(const int64_t* top_idx, const float* top_val, const float* pes, float* top_w,
                     int64_t B, int K, int64_t active_top_k, const uint8_t* eb_mask,
                     const int64_t* active_canvas_idx, int64_t unaccepted_top_k, cudaStream_t s) {
    if (B <= 0) return 0;
    int64_t eff_k = active_top_k <= K ? active_top_k : K;
    if (eff_k < 1) eff_k = 1;
    int64_t unacc = unaccepted_top_k <= eff_k ? unaccepted_top_k : eff_k;
    if (unacc < 1) unacc = 1;
    launch_k(k_apply_lod, dim3((unsigned)((B + 127) / 128)), dim3(128), 0, s, top_idx, top_val, pes, top_w, B, K,
                                                             eff_k, unacc, eb_mask,
                                                             active_canvas_idx);
    return 1;
}

}  // namespace moe

namespace moe {

// ------------------------------------------------------- expert parallelism
__global__ void k_ep_localize(int* se, int64_t P, int e_lo, int e_hi) {
    pdl_wait();
    pdl_trigger();
    for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < P; p += (int64_t)gridDim.x * blockDim.x) {
        const int e = se[p];
        se[p] = (e >= e_lo && e < e_hi) ? e - e_lo : -1;
    }
}

int launch_ep_localize(int* slot_expert, int64_t P, int e_lo, int e_hi, cudaStream_t s) {
    if (P <= 0) return 0;
    const int grid = (int)std::min<int64_t>((P + 255) / 256, 1184);
    launch_k(k_ep_localize, dim3(grid), dim3(256), 0, s, slot_expert, P, e_lo, e_hi);
    return 1;
}

// One warp per unique expert: its pairs go to rank e / epr as local id e % epr.
__global__ void __launch_bounds__(1024) k_ep_pack(BucketOut b, int epr, int nranks, int* local_e, int* cnt) {
    pdl_wait();
    pdl_trigger();
    for (int j = threadIdx.x; j < nranks; j += blockDim.x) cnt[j] = 0;
    __syncthreads();
    const int U = b.meta[0];
    const int lane = threadIdx.x & 31;
    for (int u = threadIdx.x >> 5; u < U; u += blockDim.x >> 5) {
        const int e = b.unique_expert[u], dest = e / epr, n = b.seg_count[u], s0 = b.seg_start[u];
        for (int i = lane; i < n; i += 32) local_e[s0 + i] = e - dest * epr;
        if (lane == 0) atomicAdd(&cnt[dest], n);
    }
}

int launch_ep_pack(const BucketOut& b, int experts_per_rank, int nranks, int* send_local_e, int* send_cnt,
                   cudaStream_t s) {
    launch_k(k_ep_pack, dim3(1), dim3(1024), 0, s, b, experts_per_rank, nranks, send_local_e, send_cnt);
    return 1;
}

__global__ void __launch_bounds__(256) k_gather_rows(const float* src, const int* map, const int* n_rows,
                                                     int64_t max_rows, int64_t d, float* dst) {
    pdl_wait();
    pdl_trigger();
    const int64_t n = min((int64_t)*n_rows, max_rows), d4 = d / 4;
    for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
        const float4* a = reinterpret_cast<const float4*>(src + (int64_t)map[r] * d);
        float4* o = reinterpret_cast<float4*>(dst + r * d);
        for (int64_t j = threadIdx.x; j < d4; j += blockDim.x) o[j] = __ldg(a + j);
    }
}

int launch_gather_rows(const float* src, const int* map, const int* n_rows, int64_t max_rows, int64_t d, float* dst,
                       cudaStream_t s) {
    if (max_rows <= 0) return 0;
    const int grid = (int)std::min<int64_t>(max_rows, 1184);
    launch_k(k_gather_rows, dim3(grid), dim3(256), 0, s, src, map, n_rows, max_rows, d, dst);
    return 1;
}

__global__ void k_ep_slots(const int* le, int64_t P, int E, int* se, float* sw, int* err) {
    pdl_wait();
    pdl_trigger();
    for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < P; p += (int64_t)gridDim.x * blockDim.x) {
        const int e = le[p];
        const bool ok = e >= 0 && e < E;
        if (!ok) atomicExch(err, 1);
        se[p] = ok ? e : -1;
        sw[p] = 1.0f;
    }
}

int launch_ep_slots(const int* local_e, int64_t P, int E, int* slot_expert, float* slot_weight, int* err_flag,
                    cudaStream_t s) {
    if (P <= 0) return 0;
    const int grid = (int)std::min<int64_t>((P + 255) / 256, 1184);
    launch_k(k_ep_slots, dim3(grid), dim3(256), 0, s, local_e, P, E, slot_expert, slot_weight, err_flag);
    return 1;
}

}  // namespace moe


namespace moe {

// ------------------------------------------ routing of a small batch, 2 launches
// k_route_rt, one launch of (d/128 router CTAs) + (M prep CTAs):
//  - prep CTA t writes the expert input of token t (prep_row: moe_in, its
//    block sums, the q layout of the CUDA-core kernels);
//  - router CTA c forms the rms of every token with prep_row's arithmetic
//    (per-thread sums of squares, then block_sum's reduction order), scales
//    its 128-wide K slice as prep_row does (x * inv * router_scale * rsf),
//    and writes the slice's router partial sums as k_router_part does;
//  - the router CTA that finishes last (a ticket taken after a threadfence,
//    as in the classic threadfence reduction: no CTA waits for another) adds
//    the partials of every token in slice order, runs softmax, top-k and the
//    LOD weights with one warp per token, reproducing k_topk's 128-thread
//    sums exactly, then buckets the pairs (bucket_block) and resets the
//    ticket.
// The routing outputs are therefore bit-identical to the separate kernels'.
// The fp16 gather of the pair rows follows as its own launch.
namespace {

// block_sum of R values per thread at once: warp xor trees, then the warps'
// sums as block_sum adds them.  red holds R * 33 floats.
template <int R>
__device__ __forceinline__ void block_sum_rows(float (&v)[R], int nrows, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = warp_sum(v[r]);
    __syncthreads();
    if (lane == 0)
        for (int r = 0; r < nrows; ++r) red[r * 33 + wid] = v[r];
    __syncthreads();
    for (int r = wid; r < nrows; r += nw) {
        float t = lane < nw ? red[r * 33 + lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) red[r * 33 + 32] = t;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = r < nrows ? red[r * 33 + 32] : 0.f;
}

// Softmax, top-k and LOD of token t by one warp, with the arithmetic of
// topk_row run by 128 threads: virtual thread v = 32 w + lane (w = 0..3)
// owns experts v, v + 128, ...; the sums are that thread's sequential sums,
// each warp's xor tree, then the tree of the four warp sums, (S0 + S2) +
// (S1 + S3).  pr holds E floats, tval / tidx 32 (this warp's).
// `lg` holds the token's logits (the partials summed in slice order).
__device__ __forceinline__ void topk_warp(const TopkArgs& a, int t, const float* lg, float* pr, float* tval,
                                          int* tidx, const float* pes) {
    const int lane = threadIdx.x & 31, E = a.E, K = a.K;
    float m = -INFINITY;
    for (int e = lane; e < E; e += 32) {
        const float v = lg[e] + (a.bias ? a.bias[e] : 0.f);
        pr[e] = v;
        m = fmaxf(m, v);
    }
    m = warp_max(m);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int e0 = 0; e0 < E; e0 += 128)
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const int e = e0 + 32 * w + lane;
            if (e < E) {
                const float v = expf(pr[e] - m);
                pr[e] = v;
                acc[w] += v;
            }
        }
#pragma unroll
    for (int w = 0; w < 4; ++w) acc[w] = warp_sum(acc[w]);
    const float se = (acc[0] + acc[2]) + (acc[1] + acc[3]);
    const float den = se + 1e-10f;
    __syncwarp();
    for (int e = lane; e < E; e += 32) {
        pr[e] = pr[e] / den;
        if (a.probs_out) a.probs_out[(int64_t)t * E + e] = pr[e];
    }
    __syncwarp();
    // top-k: k rounds of the largest remaining probability, the lower index
    // first on equal values (the rank order of topk_row); NaNs never enter,
    // and a chosen entry is set to NaN in pr (it is not read again)
    for (int k = 0; k < K; ++k) {
        float bv = 0.f;
        int be = -1;
        for (int e = lane; e < E; e += 32) {
            const float p = pr[e];
            if (p != p) continue;
            if (be < 0 || p > bv) {
                bv = p;
                be = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (oe >= 0 && (be < 0 || ov > bv || (ov == bv && oe < be))) {
                bv = ov;
                be = oe;
            }
        }
        if (lane == 0) {
            tval[k] = be >= 0 ? bv : -999999.0f;
            tidx[k] = be;
        }
        if (be >= 0 && lane == (be & 31)) pr[be] = __int_as_float(0x7fc00000);
        __syncwarp();
    }
    __syncwarp();
    if (lane == 0) topk_finish(a, t, tval, tidx, pes);
}

template <int J>
__global__ void __launch_bounds__(512, 1) k_route_rt(RouteRtArgs a) {
    extern __shared__ float4 sm4[];
    float* sm = reinterpret_cast<float*>(sm4);
    __shared__ float red[33];
    __shared__ int is_last;
    const int M = a.ta.M, d = (int)a.pa.K, E = a.ta.E, nsl = d / RS;
    // Weights are no product of the previous kernel: their L2 prefetch is
    // issued before the dependency wait and overlaps that kernel's tail.
    if ((int)blockIdx.x >= nsl) {  // expert input of one token
        prefetch_l2(a.pa.pre_w, d * 4);
        prefetch_l2(a.pa.router_scale, d * 4);
        pdl_wait();
        pdl_trigger();
        prep_row(a.pa, blockIdx.x - nsl, sm, red);
        return;
    }
    const int c = blockIdx.x, k0 = c * RS;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {  // this slice's router rows and scales
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a.rp + (int64_t)e * (d / 2) + k0 / 2));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a.rs + (int64_t)e * (d / 32) + k0 / 32));
    }
    if (threadIdx.x < RS / 32) asm volatile("prefetch.global.L2 [%0];" ::"l"(a.pa.router_scale + k0 + 32 * threadIdx.x));
    if (threadIdx.x == 0 && a.ta.pes) asm volatile("prefetch.global.L2 [%0];" ::"l"(a.ta.pes));
    pdl_wait();
    pdl_trigger();
    // rms of every token: prep_row's per-thread sums, block_sum's order
    float* red_rows = sm;                 // [16][33] per pass
    float* inv_s = sm + 16 * 33;          // [M]
    float* xs = inv_s + 64;               // [M][RS] scaled slice
    const float4* x4 = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.pa.x));
    for (int t0 = 0; t0 < M; t0 += 16) {
        const int nr = min(16, M - t0);
        float ss[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) ss[r] = 0.f;
        // each row's elements in prep_row's order; the rows' loads in flight together
        for (int j = threadIdx.x; j < d / 4; j += blockDim.x) {
            float4 v[16];
#pragma unroll
            for (int r = 0; r < 16; ++r)
                if (r < nr) v[r] = __ldg(x4 + (int64_t)(t0 + r) * (d / 4) + j);
#pragma unroll
            for (int r = 0; r < 16; ++r)
                if (r < nr) ss[r] = ss_step(ss[r], v[r]);
        }
        block_sum_rows<16>(ss, nr, red_rows);
        if (threadIdx.x < nr) inv_s[t0 + threadIdx.x] = 1.0f / sqrtf(ss[threadIdx.x] / (float)d + 1e-6f);
        __syncthreads();
    }
    // this CTA's slice of the router input, as prep_row writes `scaled`
    const float* xin = reinterpret_cast<const float*>(a.pa.x);
    for (int i = threadIdx.x; i < M * RS; i += blockDim.x) {
        const int t = i / RS, k = i % RS;
        const float v = __ldg(xin + (int64_t)t * d + k0 + k);
        xs[t * RS + k] = v * inv_s[t] * __ldg(a.pa.router_scale + k0 + k) * a.pa.rsf;
    }
    __syncthreads();
    router_slice_dot<J>(a.rp, a.rs, M, d, E, a.ta.part_out, c, xs);
    // the last router CTA to finish routes every token
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        is_last = atomicAdd(a.ticket, 1u) == (unsigned)(nsl - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // logits of every token: the partials of each 4 experts summed in slice
    // order by one thread, every slice's load in flight at once
    float* lg = sm;                                  // [M][E]
    const int E4 = E / 4, nsum = M * E4;
    for (int i = threadIdx.x; i < nsum; i += blockDim.x) {
        const int t = i / E4, e4 = i - t * E4;
        float4 sc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c0 = 0; c0 < nsl; c0 += 12) {
            float4 v[12];
#pragma unroll
            for (int j = 0; j < 12; ++j)
                if (c0 + j < nsl)
                    v[j] = __ldcg(reinterpret_cast<const float4*>(a.ta.part + ((int64_t)(c0 + j) * M + t) * E) + e4);
#pragma unroll
            for (int j = 0; j < 12; ++j)
                if (c0 + j < nsl) {
                    sc.x += v[j].x;
                    sc.y += v[j].y;
                    sc.z += v[j].z;
                    sc.w += v[j].w;
                }
        }
        reinterpret_cast<float4*>(lg + t * E)[e4] = sc;
        if (a.ta.scores_out) reinterpret_cast<float4*>(a.ta.scores_out + (int64_t)t * E)[e4] = sc;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
    float* pr = lg + M * E + warp * E;                       // [nwarp][E]
    float* tv_s = lg + M * E + nwarp * E + warp * 32;        // [nwarp][32]
    int* ti_s = reinterpret_cast<int*>(lg + M * E + nwarp * E + nwarp * 32) + warp * 32;
    float* pes_s = lg + M * E + nwarp * E + 2 * nwarp * 32;  // [E]
    for (int e = threadIdx.x; e < E; e += blockDim.x) pes_s[e] = __ldg(a.ta.pes + e);
    __syncthreads();
    for (int t = warp; t < M; t += nwarp) topk_warp(a.ta, t, lg + t * E, pr, tv_s, ti_s, pes_s);
    __syncthreads();
    __threadfence_block();
    int* cnt = reinterpret_cast<int*>(sm);
    __shared__ int wsum[32];
    bucket_block(a.ta.slot_expert, (int64_t)M * a.ta.K, a.ta.K, E, a.e_lo, a.e_hi, a.b, a.BN, a.tt_prefix, cnt,
                 cnt + blockDim.x, wsum);
    if (threadIdx.x == 0) atomicExch(a.ticket, 0u);
}

}  // namespace

bool route_rt_supported(int M, int E, int K, int d) {
    return M >= 1 && M <= 64 && E >= 4 && E <= 512 && E % 4 == 0 && K >= 1 && K <= 32 && d % RS == 0 &&
           d <= 12288 && d / RS >= 1;
}

int launch_route_rt(const RouteRtArgs& a, cudaStream_t s) {
    const int M = a.ta.M, d = (int)a.pa.K, E = a.ta.E;
    if (!route_rt_supported(M, E, a.ta.K, d)) return -1;
    const int nsl = d / RS;
    size_t smem = (size_t)d * 4;                                             // prep CTAs
    smem = std::max(smem, (size_t)(16 * 33 + 64 + M * RS) * 4);              // router CTAs
    smem = std::max(smem, (size_t)(M * E + 16 * E + 16 * 64 + E) * 4);       // logits + top-k (16 warps)
    smem = std::max(smem, (size_t)2 * 512 * 4);                              // bucketing
    auto kern = M <= 16 ? k_route_rt<4> : k_route_rt<16>;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return -1;
    launch_k(kern, dim3(nsl + M), dim3(512), smem, s, a);
    return 1;
}

}  // namespace moe
