// moe_gemv.cu -- grouped Q4_0 GEMV on CUDA cores for experts with few
// routed tokens (decode): stage 1 (gate/up + activation) and stage 2 (down)
// of moe_kernels.mojo:614-781 over the bucketed (expert, token) pairs.
//
// With one or two tokens per expert the tensor-core path is bound by its MMA
// issue rate (an M=128, N=16, K=16 tcgen05.mma per 2048 weights); here each
// weight costs about two CUDA-core instructions:
//  - a warp owns 4 weight rows (PLAIN) or 2 activation rows = 2 gate + 2 up
//    rows (ACT) over the whole K; lane l takes the 16-byte Q4 chunks
//    (32 weights, one block and its scale) l, l+32, ...; the 4 rows share
//    every activation value the lane loads;
//  - nibble i (0..3) of a 16-bit half-word becomes the float 2^23 + n*16^i
//    with one LOP3 ((w & 0xF<<4i) | 0x4B000000); one packed subtract
//    (add.rn.f32x2) gives n*16^i exactly, and the activation is used
//    pre-scaled by 16^-i (exact powers of two), so sum_k n_k x_k needs one
//    packed fma.rn.f32x2 per two weights and token;
//  - the -8 offset of Q4_0 is applied per block: sum (n-8) x = sum n x - 8 X
//    with X the block sum of x; then times the block scale, in fp32;
//  - a CTA (8 warps) covers 32 consecutive rows of one expert, so the
//    expert's activation rows stay in the SM's L1; the next work item's rows
//    and scales are prefetched into L2 as contiguous blocks.
#include "common.cuh"
#include "moe_internal.h"

namespace moe {

namespace {

constexpr int DG_WARPS = 8;

__device__ __forceinline__ unsigned long long pk2(uint32_t lo, uint32_t hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ unsigned long long pkf(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 upk(unsigned long long v) {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
    return make_float2(lo, hi);
}
__device__ __forceinline__ unsigned long long fadd2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long ffma2(unsigned long long a, unsigned long long b,
                                                    unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__device__ __forceinline__ void l2_prefetch(const void* p, int64_t bytes) {
    uintptr_t b = (reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15);
    const uintptr_t e = (reinterpret_cast<uintptr_t>(p) + (uintptr_t)bytes) & ~uintptr_t(15);
    while (b < e) {
        const uint32_t n = (uint32_t)((e - b) < 65536u ? (e - b) : 65536u);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(b), "r"(n) : "memory");
        b += n;
    }
}

// rows of a warp: PLAIN 4 consecutive rows; ACT act rows j, j+1 -> weight
// rows j, j+1 (gate) and F+j, F+j+1 (up)
template <int MODE>
struct Rows {
    static constexpr int RW = 4;                         // weight rows per warp
    static constexpr int ITEM = (MODE == GEMV_ACT) ? 16 : 32;  // act rows / rows per CTA item
};

// dot products of the warp's 4 rows with NT tokens over the whole K;
// res[r][t] is complete in every lane afterwards.
template <int NT>
__device__ __forceinline__ void rows_dot(const uint8_t* const (&wrow)[4], const float* const (&srow)[4],
                                         const bool (&rv)[4], const float* const (&xrow)[NT], int K,
                                         float (&res)[4][NT]) {
    const int lane = threadIdx.x & 31;
    const int nc = K >> 5;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) res[r][t] = 0.f;
    const unsigned long long neg_magic = pkf(-8388608.0f, -8388608.0f);
    for (int c = lane; c < nc; c += 32) {
        uint4 q[4];
        float s[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            if (rv[r]) {
                q[r] = ldg_stream(wrow[r] + c * 16);
                s[r] = ldg_stream_f(srow[r] + c);
            } else {
                q[r] = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
                s[r] = 0.f;
            }
        }
        unsigned long long acc[4][NT];
        float xs[NT];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[r][t] = 0ull;
#pragma unroll
        for (int t = 0; t < NT; ++t) xs[t] = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            // activations 8w .. 8w+7 of the chunk, pre-scaled by 16^-(k % 4)
            unsigned long long xp[NT][4];
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float4* xv = reinterpret_cast<const float4*>(xrow[t] + c * 32 + 8 * w);
                const float4 f0 = __ldg(xv), f1 = __ldg(xv + 1);
                xs[t] += ((f0.x + f0.y) + (f0.z + f0.w)) + ((f1.x + f1.y) + (f1.z + f1.w));
                xp[t][0] = pkf(f0.x, f0.y * 0.0625f);
                xp[t][1] = pkf(f0.z * 0.00390625f, f0.w * 0.000244140625f);
                xp[t][2] = pkf(f1.x, f1.y * 0.0625f);
                xp[t][3] = pkf(f1.z * 0.00390625f, f1.w * 0.000244140625f);
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const uint32_t word = w == 0 ? q[r].x : w == 1 ? q[r].y : w == 2 ? q[r].z : q[r].w;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t u = h ? (word >> 16) : word;
                    // elements 8w+4h+i, i = 0..3, as 2^23 + n * 16^i, minus 2^23
                    const unsigned long long v01 =
                        fadd2(pk2((u & 0xFu) | 0x4B000000u, (u & 0xF0u) | 0x4B000000u), neg_magic);
                    const unsigned long long v23 =
                        fadd2(pk2((u & 0xF00u) | 0x4B000000u, (u & 0xF000u) | 0x4B000000u), neg_magic);
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        acc[r][t] = ffma2(v01, xp[t][2 * h], acc[r][t]);
                        acc[r][t] = ffma2(v23, xp[t][2 * h + 1], acc[r][t]);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float2 a2 = upk(acc[r][t]);
                res[r][t] = fmaf(s[r], (a2.x + a2.y) - 8.0f * xs[t], res[r][t]);
            }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) res[r][t] = warp_sum(res[r][t]);
}

}  // namespace

template <int MODE>
__global__ void __launch_bounds__(DG_WARPS * 32, 2) k_dgemv(GemvArgs a) {
    pdl_wait();
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = a.K, nb = K >> 5;
    const int64_t rows_tile = (MODE == GEMV_ACT) ? a.F : a.rows_per_expert;
    const int n_groups = (int)((rows_tile + Rows<MODE>::ITEM - 1) / Rows<MODE>::ITEM);
    const int U = a.meta[0];
    const int64_t n_items = (int64_t)U * n_groups;
    auto item_rows = [&](int64_t item, int* e, int* r0) {
        const int u = (int)(item / n_groups), g = (int)(item - (int64_t)u * n_groups);
        *e = a.unique_expert[u];
        *r0 = g * Rows<MODE>::ITEM;
        return u;
    };
    for (int64_t item = blockIdx.x; item < n_items; item += gridDim.x) {
        int e, r0;
        const int u = item_rows(item, &e, &r0);
        if (threadIdx.x == 0 && item + gridDim.x < n_items) {  // next item's rows into L2
            int e2, r2;
            item_rows(item + gridDim.x, &e2, &r2);
            const int64_t base = (int64_t)e2 * a.rows_per_expert;
            const int64_t nr = (MODE == GEMV_ACT) ? min((int64_t)Rows<MODE>::ITEM, (int64_t)a.F - r2)
                                                  : min((int64_t)Rows<MODE>::ITEM, a.rows_per_expert - r2);
            for (int h = 0; h < ((MODE == GEMV_ACT) ? 2 : 1); ++h) {
                const int64_t row = base + r2 + (h ? a.F : 0);
                l2_prefetch(a.Wp + row * (K >> 1), nr * (K >> 1));
                l2_prefetch(a.Ws + row * nb, nr * nb * 4);
            }
        }
        const int n = a.seg_count[u], s0 = a.seg_start[u];
        const uint8_t* We = a.Wp + (size_t)e * a.rows_per_expert * (K >> 1);
        const float* Se = a.Ws + (size_t)e * a.rows_per_expert * nb;
        int64_t row[4];
        bool rv[4];
        if (MODE == GEMV_ACT) {
            const int j = r0 + warp * 2;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                rv[i] = rv[2 + i] = j + i < a.F;
                row[i] = j + i;
                row[2 + i] = (int64_t)a.F + j + i;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                row[i] = (int64_t)r0 + warp * 4 + i;
                rv[i] = row[i] < a.rows_per_expert;
            }
        }
        if (!(rv[0] || rv[1] || rv[2] || rv[3])) continue;
        const uint8_t* wrow[4];
        const float* srow[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t rr = rv[i] ? row[i] : 0;
            wrow[i] = We + rr * (K >> 1);
            srow[i] = Se + rr * nb;
        }
        auto emit = [&](int p, const float (&v)[4]) {
            if (MODE == GEMV_ACT) {
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    if (!rv[i]) continue;
                    if (a.gu_out) {
                        a.gu_out[(int64_t)p * a.gu_stride + row[i]] = v[i];
                        a.gu_out[(int64_t)p * a.gu_stride + row[2 + i]] = v[2 + i];
                    }
                    a.out[(int64_t)p * a.out_stride + row[i]] = act_fn(v[i], v[2 + i], a.act);
                }
            } else {
                const int64_t orow = a.out_row ? a.out_row[p] : p;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (rv[i]) a.out[orow * a.out_stride + row[i]] = v[i];
            }
        };
        int t = 0;
        for (; t + 2 <= n; t += 2) {
            const float* xr[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int p = s0 + t + i;
                xr[i] = a.X + (int64_t)(a.pair_row ? a.pair_row[p] : p) * K;
            }
            float res[4][2];
            rows_dot<2>(wrow, srow, rv, xr, K, res);
            if (lane == 0) {
                for (int i = 0; i < 2; ++i) {
                    const float v[4] = {res[0][i], res[1][i], res[2][i], res[3][i]};
                    emit(s0 + t + i, v);
                }
            }
        }
        if (t < n) {
            const int p = s0 + t;
            const float* xr[1] = {a.X + (int64_t)(a.pair_row ? a.pair_row[p] : p) * K};
            float res[4][1];
            rows_dot<1>(wrow, srow, rv, xr, K, res);
            if (lane == 0) {
                const float v[4] = {res[0][0], res[1][0], res[2][0], res[3][0]};
                emit(p, v);
            }
        }
    }
}

bool dgemv_supported(const GemvArgs& a) {
    return a.dense_tokens == 0 && a.K % 32 == 0 && (reinterpret_cast<uintptr_t>(a.Wp) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(a.X) & 15) == 0;
}

int launch_dgemv(int mode, const GemvArgs& a, int num_sms, cudaStream_t s) {
    const int64_t rows_tile = mode == GEMV_ACT ? a.F : a.rows_per_expert;
    const int item = mode == GEMV_ACT ? Rows<GEMV_ACT>::ITEM : Rows<GEMV_PLAIN>::ITEM;
    const int64_t items = ((rows_tile + item - 1) / item) * a.max_unique;
    const int64_t cap = (int64_t)num_sms * 2;
    const int grid = (int)(items < cap ? items : cap);
    if (grid <= 0) return 0;
    if (mode == GEMV_ACT) launch_k(k_dgemv<GEMV_ACT>, dim3(grid), dim3(DG_WARPS * 32), 0, s, a);
    else launch_k(k_dgemv<GEMV_PLAIN>, dim3(grid), dim3(DG_WARPS * 32), 0, s, a);
    return 1;
}

}  // namespace moe
