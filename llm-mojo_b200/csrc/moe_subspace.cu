// moe_subspace.cu -- the diffusion engine's router-subspace FFN bypass on
// the GPU (diffusion_kernels.mojo:2253-2426), and the check of the bounded
// device-side wait that every pipelined kernel of the library uses.
//
// Bypass.  Between denoising steps most canvas tokens barely move.  The
// reference uses the 128 router logits a token already has as a cheap
// monitor: a token whose two top experts are unchanged since it was last
// evaluated, and whose logits moved by at most tau relative to that
// evaluation, skips the MoE FFN and reuses its cached output.
//  - k_subspace_filter (one CTA): eight lanes per token compute the drift
//    sums in the reference's SIMD order (lane l takes experts e = l mod 8
//    with fused multiply-adds; the lanes are added as a halving tree; a
//    tail of E % 8 experts is added one by one), so every bypass decision is
//    bit-identical to the reference's.  The evaluated tokens are compacted
//    into ffn_keep_b in ascending b with a block scan; their logits and top-2
//    ids become the new reference point, the bypassed ones get zero routing
//    weights;
//  - k_keep_map + k_subspace_rows: the reference walks b in order with a
//    cursor into ffn_keep_b.  That walk matches exactly the longest strictly
//    increasing prefix of ffn_keep_b whose values are valid rows (an entry
//    that breaks it is never reached again), so k_keep_map marks those
//    entries in a row map in parallel, and the row kernel then copies each
//    row (16-byte vectors when the row size and pointers allow): evaluated
//    rows go to the cache (and, for the scatter form, first from the
//    compacted sub-batch output to the full output), bypassed rows come back
//    from the cache.  Both are pure HBM traffic, 2-3 row copies per token.
#include "common.cuh"
#include "moe_internal.h"
#include "tc_ptx.cuh"

namespace moe {

namespace {

constexpr int kFilterThreads = 1024;
constexpr int kLanes = 8;                           // lanes per token (the reference's SIMD width)
constexpr int kTokPerPass = kFilterThreads / kLanes;  // 128 tokens per pass

__global__ void __launch_bounds__(kFilterThreads) k_subspace_filter(SubspaceFilterArgs a) {
    __shared__ int keep_s[kTokPerPass];
    __shared__ int pos_s[kTokPerPass];
    __shared__ int total_s;
    pdl_wait();
    pdl_trigger();
    const int g = threadIdx.x / kLanes, l = threadIdx.x % kLanes;
    const unsigned gmask = 0xFFu << (threadIdx.x & 24);  // this token's 8 lanes
    const int E = a.E, K = a.K;
    const float tau_sq = a.tau * a.tau;
    int64_t running = 0;
    for (int64_t b0 = 0; b0 < a.B; b0 += kTokPerPass) {
        const int64_t b = b0 + g;
        const bool valid = b < a.B;
        int64_t ot = 0;
        bool bypass = false;
        if (valid) {
            ot = a.active_idx ? a.active_idx[b] : b;
            const bool accepted = a.eb_mask ? (a.eb_mask[ot] != 0) : true;
            if (a.step >= 1 && accepted && K >= 2 && E > 0) {
                const int64_t e0 = a.top_idx[b * K], e1 = a.top_idx[b * K + 1];
                const int64_t p0 = a.prev_top2[ot * 2], p1 = a.prev_top2[ot * 2 + 1];
                if (p0 >= 0 && p1 >= 0 && e0 == p0 && e1 == p1) {
                    const float* cr = a.r_curr + b * E;
                    const float* pr = a.r_prev + ot * E;
                    float vd = 0.f, vn = 0.f;
                    const int full = E / kLanes * kLanes;
                    for (int e = l; e < full; e += kLanes) {
                        const float c = cr[e], p = pr[e];
                        const float d = __fsub_rn(c, p);
                        vd = __fmaf_rn(d, d, vd);
                        vn = __fmaf_rn(p, p, vn);
                    }
                    // halving tree over the 8 lanes: (0+4, 1+5, 2+6, 3+7), then (.+2), then (.+1)
#pragma unroll
                    for (int o = 4; o > 0; o >>= 1) {
                        vd = __fadd_rn(vd, __shfl_xor_sync(gmask, vd, o, kLanes));
                        vn = __fadd_rn(vn, __shfl_xor_sync(gmask, vn, o, kLanes));
                    }
                    for (int e = full; e < E; ++e) {  // the reference's scalar tail
                        const float d = __fsub_rn(cr[e], pr[e]);
                        vd = __fadd_rn(vd, __fmul_rn(d, d));
                        vn = __fadd_rn(vn, __fmul_rn(pr[e], pr[e]));
                    }
                    bypass = vn > 1e-12f ? (vd <= __fmul_rn(tau_sq, vn)) : (vd <= 1e-12f);
                }
            }
        }
        if (l == 0) keep_s[g] = (valid && !bypass) ? 1 : 0;
        __syncthreads();
        if (threadIdx.x < 32) {  // exclusive scan of 128 flags, 4 per lane
            const int t0 = threadIdx.x * 4;
            const int c = keep_s[t0] + keep_s[t0 + 1] + keep_s[t0 + 2] + keep_s[t0 + 3];
            int inc = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, inc, o);
                if ((int)threadIdx.x >= o) inc += v;
            }
            int ex = inc - c;
            for (int j = 0; j < 4; ++j) {
                pos_s[t0 + j] = ex;
                ex += keep_s[t0 + j];
            }
            if (threadIdx.x == 31) total_s = inc;
        }
        __syncthreads();
        if (valid) {
            if (!bypass) {
                if (l == 0) {
                    a.keep_out[running + pos_s[g]] = b;
                    if (K >= 1) a.prev_top2[ot * 2] = a.top_idx[b * K];
                    if (K >= 2) a.prev_top2[ot * 2 + 1] = a.top_idx[b * K + 1];
                }
                for (int e = l; e < E; e += kLanes) a.r_prev[ot * E + e] = a.r_curr[b * E + e];
            } else if (a.top_w) {
                for (int s = l; s < K; s += kLanes) a.top_w[b * K + s] = 0.f;
            }
        }
        running += total_s;
        __syncthreads();  // keep_s / pos_s / total_s are reused by the next pass
    }
    if (threadIdx.x == 0) *a.count_out = running;
}

// map[b] = index j of ffn_keep_b that the reference's in-order walk matches
// at row b, else -1.  Those j are the longest prefix of ffn_keep_b (at most
// len entries) that is strictly increasing with values in [0, B).
__global__ void __launch_bounds__(1024) k_keep_map(const int64_t* keep, int64_t len, int64_t B, int* map) {
    __shared__ int64_t first_bad;
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) first_bad = len;
    for (int64_t b = threadIdx.x; b < B; b += blockDim.x) map[b] = -1;
    __syncthreads();
    for (int64_t j = threadIdx.x; j < len; j += blockDim.x) {
        const int64_t v = keep[j];
        const bool bad = v < 0 || v >= B || (j > 0 && v <= keep[j - 1]);
        if (bad) atomicMin(reinterpret_cast<unsigned long long*>(&first_bad), (unsigned long long)j);
    }
    __syncthreads();
    const int64_t n = first_bad;
    for (int64_t j = threadIdx.x; j < n; j += blockDim.x) map[keep[j]] = (int)j;
}

template <typename V>
__device__ __forceinline__ void copy_row(uint8_t* dst, const uint8_t* src, int64_t bytes) {
    const int64_t n = bytes / (int64_t)sizeof(V);
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x)
        reinterpret_cast<V*>(dst)[i] = reinterpret_cast<const V*>(src)[i];
}
template <typename V>
__device__ __forceinline__ void copy_row2(uint8_t* d0, uint8_t* d1, const uint8_t* src, int64_t bytes) {
    const int64_t n = bytes / (int64_t)sizeof(V);
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const V v = reinterpret_cast<const V*>(src)[i];
        reinterpret_cast<V*>(d0)[i] = v;
        reinterpret_cast<V*>(d1)[i] = v;
    }
}

// One CTA per row.  sub == nullptr: sync_moe_subspace_cache (out is read
// for evaluated rows); else scatter_and_restore_ffn_subspace.
template <typename V>
__global__ void __launch_bounds__(256) k_subspace_rows(SubspaceRowsArgs a) {
    pdl_wait();
    pdl_trigger();
    const int64_t b = blockIdx.x;
    const int64_t ot = a.active_idx ? a.active_idx[b] : b;
    const int j = a.map[b];
    uint8_t* row = a.out + b * a.row_bytes;
    uint8_t* cache = a.cache + ot * a.row_bytes;
    if (j < 0)
        copy_row<V>(row, cache, a.row_bytes);
    else if (!a.sub)
        copy_row<V>(cache, row, a.row_bytes);
    else
        copy_row2<V>(row, cache, a.sub + (int64_t)j * a.row_bytes, a.row_bytes);
}

// One CTA of two warps, each waiting on an mbarrier that nothing completes:
// warp 0 with the bounded poll the pipelined kernels use for their data
// hand-offs (it gives up at the deadline, raises the abort flag and the
// error word), warp 1 with the back-off poll of their epilogues (it leaves
// when it sees the abort flag).
__global__ void k_wait_check(int* err_flag, uint64_t timeout_ns) {
    __shared__ __align__(8) uint64_t bar[2];
    __shared__ volatile int abort_flag;
    if (threadIdx.x == 0) {
        tc::mbar_init(tc::smem_u32(&bar[0]), 1);
        tc::mbar_init(tc::smem_u32(&bar[1]), 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const tc::Guard G{&abort_flag, err_flag, tc::globaltimer() + timeout_ns};
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        if (warp == 0) {
            tc::mbar_wait(tc::smem_u32(&bar[0]), 0, G);
        } else {
            for (uint32_t it = 0;; ++it) {
                if (tc::mbar_try(tc::smem_u32(&bar[1]), 0)) break;
                if (abort_flag) break;
                if (tc::globaltimer() > G.deadline + 1000000000ull) break;  // backstop
                __nanosleep(1024);
            }
        }
    }
    __syncthreads();
}

}  // namespace

int launch_subspace_filter(const SubspaceFilterArgs& a, cudaStream_t s) {
    if (a.B <= 0) return 0;
    launch_k(k_subspace_filter, dim3(1), dim3(kFilterThreads), 0, s, a);
    return 1;
}

int launch_subspace_rows(const SubspaceRowsArgs& a, const int64_t* keep, int64_t len, cudaStream_t s) {
    if (a.B <= 0 || a.row_bytes <= 0) return 0;
    launch_k(k_keep_map, dim3(1), dim3(1024), 0, s, keep, len, a.B, a.map);
    const uintptr_t al = reinterpret_cast<uintptr_t>(a.out) | reinterpret_cast<uintptr_t>(a.cache) |
                         reinterpret_cast<uintptr_t>(a.sub) | (uintptr_t)a.row_bytes;
    const dim3 grid((unsigned)a.B);
    if ((al & 15u) == 0)
        launch_k(k_subspace_rows<uint4>, grid, dim3(256), 0, s, a);
    else if ((al & 3u) == 0)
        launch_k(k_subspace_rows<uint32_t>, grid, dim3(256), 0, s, a);
    else
        launch_k(k_subspace_rows<uint8_t>, grid, dim3(256), 0, s, a);
    return 2;
}

int launch_wait_check(int* err_flag, uint64_t timeout_ns, cudaStream_t s) {
    k_wait_check<<<1, 64, 0, s>>>(err_flag, timeout_ns);
    return 1;
}

}  // namespace moe
