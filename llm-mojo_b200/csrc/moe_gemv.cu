// moe_gemv.cu -- grouped Q4_0 products on CUDA cores for experts with few
// routed tokens (decode): stage 1 (gate/up + activation) and stage 2 (down)
// of moe_kernels.mojo:614-781 over the bucketed (expert, token) pairs.
//
// With a handful of tokens per expert the work is a weight stream: every
// weight byte is read once from HBM and used for each of the expert's
// tokens.  Layout of the work:
//  - one CTA per SM: 8 compute warps and one copy warp.  A work item is 32
//    consecutive weight rows of one expert (ACT: 16 act rows = 16 gate + 16
//    up rows), i.e. one or two contiguous blocks of rows x K/2 bytes plus
//    their scale rows, which the copy warp brings into a shared-memory slot
//    with one bulk copy (cp.async.bulk) each: long sequential DRAM reads, no
//    per-thread load tracking.  As many slots as fit keep the next items in
//    flight while the warps work on one;
//  - the tokens' activations arrive the same way, one bulk copy per token
//    row, in passes of up to QT tokens (two pass slots); an item's weights
//    stay in their slot for all of its passes;
//  - a compute warp takes 4 rows; lane l takes the 16-byte Q4 chunks (32
//    weights, one block and its scale) l, l+32, ... of each;
//  - the CTAs split the expert-major item list into contiguous ranges, so
//    consecutive items of a CTA mostly share one activation pass;
//  - nibble i (0..3) of a 16-bit half-word becomes the float 2^23 + n*16^i
//    with one LOP3 ((w & 0xF<<4i) | 0x4B000000); one packed subtraction of
//    2^23 + 8*16^i (add.rn.f32x2) leaves (n - 8) * 16^i exactly, and the
//    activations are kept pre-scaled by 16^-i (exact powers of two), so
//    sum_k (n_k - 8) x_k takes one packed fma.rn.f32x2 per two weights and
//    token; the block sum is then scaled by the block's fp32 scale.
//
// Activation rows are read in the "q layout": within each row, element j is
// stored pre-scaled by 16^-(j % 4) at float position 4 * xunit(j / 4) + j % 4,
// where xunit XOR-swizzles the eight float4 units of each 32-element chunk so
// that the lanes' shared-memory reads spread over all banks.  k_to_qlayout
// writes the gate/up input that way and the ACT epilogue writes its output
// (the down projection's input) that way.
//
// Every mbarrier wait is bounded; on expiry the kernel raises err_flag = 2
// and every role stops.
#include <type_traits>

#include "common.cuh"
#include "moe_internal.h"
#include "tc_ptx.cuh"

namespace moe {

namespace {

constexpr int QW = 8;                    // compute warps
constexpr int RW = 4;                    // weight rows per compute warp
constexpr int QT = 4;                    // tokens per pass (at most)
constexpr int IROWS = QW * RW;           // weight rows per item (ACT: half gate, half up)
constexpr int NXS = 2;                   // activation pass slots
constexpr int MAX_SLOTS = 6;             // weight item slots (as many as fit, at least 2)
constexpr int QTHREADS = (QW + 1) * 32;  // + the copy warp

struct QLay {
    int qt;          // tokens per pass: min(QT, most tokens any expert has)
    int xbytes;      // one pass: qt rows of K floats
    int qbytes;      // IROWS rows x K/2 bytes
    int slot_bytes;  // packed rows, then their scales; 128-aligned
    int nslot;
    int off_slot, off_bar, total;
};
// Passes only as wide as the batch can fill: a one-token batch leaves the
// activation slots small and the weight ring deeper.
__host__ __device__ inline QLay qlay(int K, int max_tokens) {
    QLay L;
    L.qt = max_tokens < 1 ? 1 : (max_tokens < QT ? max_tokens : QT);
    L.xbytes = L.qt * K * 4;
    L.qbytes = IROWS * (K / 2);
    L.slot_bytes = (L.qbytes + IROWS * (K / 32) * 4 + 127) & ~127;
    const int budget = 225 * 1024 - NXS * L.xbytes - 256;
    L.nslot = budget / L.slot_bytes;
    if (L.nslot > MAX_SLOTS) L.nslot = MAX_SLOTS;
    L.off_slot = NXS * L.xbytes;
    L.off_bar = L.off_slot + L.nslot * L.slot_bytes;
    L.total = L.off_bar + 8 * (2 * MAX_SLOTS + 2 * NXS) + 16;
    return L;
}

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

// bytes (a multiple of 16) from global to shared memory, completing on `bar`
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     tc::smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// every lane waits (the data the barrier guards is read by all of them)
__device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity, const tc::Guard& g) {
    const bool ok = tc::mbar_wait(bar, parity, g);
    return __all_sync(0xffffffffu, ok) != 0;
}

template <int MODE>
struct QRows {
    static constexpr int ITEM = (MODE == GEMV_ACT) ? IROWS / 2 : IROWS;  // act rows / rows per item
};

// Dot products of the warp's RW rows (slot rows lr[], packed rows sq, scale
// rows ss; every row of an item exists) with NT staged tokens over the whole
// K.  res[r][t] is complete in every lane afterwards.
template <int NT>
__device__ __forceinline__ void rows_dot(const uint8_t* sq, const float* ss, const int (&lr)[RW],
                                         const float4* xs, int K, float (&res)[RW][NT]) {
    const int lane = threadIdx.x & 31;
    const int nc = K >> 5, ku = K >> 2, k2 = K >> 1;
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) res[r][t] = 0.f;
    // -(2^23 + 8 * 16^i) for the nibble pairs (0, 1) and (2, 3)
    const unsigned long long m01 = pkf(-8388616.0f, -8388736.0f);
    const unsigned long long m23 = pkf(-8390656.0f, -8421376.0f);
    // masks and the magic exponent live in registers (see and_or)
    uint32_t mk[4] = {0xFu, 0xF0u, 0xF00u, 0xF000u}, magic = 0x4B000000u;
    asm volatile("" : "+r"(mk[0]), "+r"(mk[1]), "+r"(mk[2]), "+r"(mk[3]), "+r"(magic));
    const uint8_t* qrow[RW];
    const float* srow[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        qrow[r] = sq + lr[r] * k2 + lane * 16;
        srow[r] = ss + lr[r] * nc + lane;
    }
    // every lane runs the same number of chunks; a lane past the row's end
    // reads finite data (chunk 0's activations) and weights it by 0
    const int iters = (nc + 31) >> 5;
    for (int it = 0; it < iters; ++it) {
        const int c = lane + 32 * it;
        const bool live = c < nc;
        uint4 q[RW];
        float s[RW];
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            q[r] = *reinterpret_cast<const uint4*>(qrow[r] + it * 512);
            s[r] = live ? srow[r][it * 32] : 0.f;
        }
        // this chunk's activation units: xunit(8c + k) = 8c + (k ^ (c % 8))
        const float4* xc = xs + (live ? (c << 3) : 0);
        const int sw = live ? (c & 7) : 0;
        unsigned long long acc[RW][NT];
#pragma unroll
        for (int r = 0; r < RW; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[r][t] = 0ull;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                // elements 8w+4h+i, i = 0..3, of every row as (n - 8) * 16^i
                unsigned long long v01[RW], v23[RW];
#pragma unroll
                for (int r = 0; r < RW; ++r) {
                    const uint32_t word = w == 0 ? q[r].x : w == 1 ? q[r].y : w == 2 ? q[r].z : q[r].w;
                    const uint32_t u = h ? (word >> 16) : word;
                    v01[r] = fadd2(pk2(tc::and_or(u, mk[0], magic), tc::and_or(u, mk[1], magic)), m01);
                    v23[r] = fadd2(pk2(tc::and_or(u, mk[2], magic), tc::and_or(u, mk[3], magic)), m23);
                }
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const float4 f = xc[t * ku + ((2 * w + h) ^ sw)];  // pre-scaled activations
                    const unsigned long long x01 = pkf(f.x, f.y), x23 = pkf(f.z, f.w);
#pragma unroll
                    for (int r = 0; r < RW; ++r) {
                        acc[r][t] = ffma2(v01[r], x01, acc[r][t]);
                        acc[r][t] = ffma2(v23[r], x23, acc[r][t]);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < RW; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float2 a2 = upk(acc[r][t]);
                res[r][t] = fmaf(s[r], a2.x + a2.y, res[r][t]);
            }
    }
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) res[r][t] = warp_sum(res[r][t]);
}

__global__ void k_to_qlayout(const float* __restrict__ x, float* __restrict__ xq, int64_t rows, int K) {
    pdl_wait();
    pdl_trigger();
    const int64_t n = rows * K;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / K, j = i - r * K;
        xq[r * K + qpos(j)] = x[i] * qscale(j);
    }
}

}  // namespace

template <int MODE>
__global__ void __launch_bounds__(QTHREADS, 1) k_dgemv(GemvArgs a) {
    extern __shared__ __align__(128) uint8_t qsm[];
    const int K = a.K, nb = K >> 5;
    const QLay L = qlay(K, a.max_tokens);
    const uint32_t bar0 = tc::smem_u32(qsm + L.off_bar);
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto empty = [&](int s) { return bar0 + 8u * (MAX_SLOTS + s); };
    auto xfull = [&](int s) { return bar0 + 8u * (2 * MAX_SLOTS + s); };
    auto xempty = [&](int s) { return bar0 + 8u * (2 * MAX_SLOTS + NXS + s); };
    volatile int* abort_flag = reinterpret_cast<volatile int*>(qsm + L.off_bar + 8 * (2 * MAX_SLOTS + 2 * NXS));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < L.nslot; ++s) {
            tc::mbar_init(full(s), 1);
            tc::mbar_init(empty(s), QW);
        }
        for (int s = 0; s < NXS; ++s) {
            tc::mbar_init(xfull(s), 1);
            tc::mbar_init(xempty(s), QW);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_wait();  // barrier setup overlaps the previous kernel
    pdl_trigger();
    const tc::Guard G{abort_flag, a.err_flag, tc::globaltimer() + a.timeout_ns};

    const int64_t R = a.rows_per_expert;
    const int64_t rows_tile = (MODE == GEMV_ACT) ? a.F : R;
    const int n_groups = (int)((rows_tile + QRows<MODE>::ITEM - 1) / QRows<MODE>::ITEM);
    const int64_t n_items = (int64_t)a.meta[0] * n_groups;
    const int64_t beg = (int64_t)blockIdx.x * n_items / gridDim.x;
    const int64_t end = (int64_t)(blockIdx.x + 1) * n_items / gridDim.x;

    if (warp == QW) {
        // ------------------------------------------------ copy warp (one thread)
        if (lane == 0) {
            uint32_t armed = 0, par = 0, xarmed = 0, xpar = 0;
            int xs_u = -1, xs_t0 = -1;
            uint32_t k = 0, xk = 0;
            bool ok = true;
            for (int64_t item = beg; ok && item < end; ++item, ++k) {
                const int u = (int)(item / n_groups), g = (int)(item - (int64_t)u * n_groups);
                const int64_t ebase = (int64_t)a.unique_expert[u] * R;
                const int r0 = g * QRows<MODE>::ITEM;
                const int slot = (int)(k % (uint32_t)L.nslot);
                const uint32_t ph = (k / (uint32_t)L.nslot) & 1u;
                if (!(ok = tc::mbar_wait(empty(slot), ph ^ 1u, G))) break;
                uint8_t* dq = qsm + L.off_slot + slot * L.slot_bytes;
                float* ds = reinterpret_cast<float*>(dq + L.qbytes);
                // one (PLAIN) or two (ACT: gate, up) blocks of whole rows
                const int nblk = (MODE == GEMV_ACT) ? 2 : 1;
                const int brows = QRows<MODE>::ITEM;
                const int nr = (int)min((int64_t)brows, rows_tile - r0);
                const uint32_t qb = (uint32_t)nr * (K / 2), sb = (uint32_t)nr * nb * 4;
                tc::mbar_expect_tx(full(slot), nblk * (qb + sb));
                for (int b = 0; b < nblk; ++b) {
                    const int64_t grow = ebase + (b ? a.F : 0) + r0;
                    bulk_g2s(dq + (size_t)b * brows * (K / 2), a.Wp + grow * (K / 2), qb, full(slot));
                    bulk_g2s(ds + (size_t)b * brows * nb, a.Ws + grow * nb, sb, full(slot));
                }
                armed |= 1u << slot;
                par = (par & ~(1u << slot)) | (ph << slot);
                // the item's activation passes, each once per run of items that share it
                const int n = a.seg_count[u], s0 = a.seg_start[u];
                for (int t0 = 0; t0 < n; t0 += L.qt) {
                    if (u == xs_u && t0 == xs_t0) continue;
                    const int xsl = (int)(xk % NXS);
                    const uint32_t xph = (xk / NXS) & 1u;
                    if (!(ok = tc::mbar_wait(xempty(xsl), xph ^ 1u, G))) break;
                    const int nt = min(L.qt, n - t0);
                    tc::mbar_expect_tx(xfull(xsl), (uint32_t)nt * K * 4);
                    for (int t = 0; t < nt; ++t) {
                        const int p = s0 + t0 + t;
                        const int64_t xr = a.pair_row ? a.pair_row[p] : p;
                        bulk_g2s(qsm + xsl * L.xbytes + (size_t)t * K * 4, a.X + xr * K, (uint32_t)K * 4, xfull(xsl));
                    }
                    xarmed |= 1u << xsl;
                    xpar = (xpar & ~(1u << xsl)) | (xph << xsl);
                    xs_u = u;
                    xs_t0 = t0;
                    ++xk;
                }
            }
            // every armed copy lands before the CTA may exit
            tc::Guard Gd{abort_flag, a.err_flag, tc::globaltimer() + 2000000000ull};
            volatile int no_abort = 0;
            Gd.abort = &no_abort;
            for (int s = 0; s < L.nslot; ++s)
                if (armed & (1u << s)) tc::mbar_wait(full(s), (par >> s) & 1u, Gd);
            for (int s = 0; s < NXS; ++s)
                if (xarmed & (1u << s)) tc::mbar_wait(xfull(s), (xpar >> s) & 1u, Gd);
        }
        return;
    }

    // ---------------------------------------------------- compute warps
    uint32_t k = 0, xk = 0;
    int xs_u = -1, xs_t0 = -1, xsl = -1;
    bool ok = true;
    for (int64_t item = beg; ok && item < end; ++item, ++k) {
        const int u = (int)(item / n_groups), g = (int)(item - (int64_t)u * n_groups);
        const int r0 = g * QRows<MODE>::ITEM;
        const int n = a.seg_count[u], s0 = a.seg_start[u];
        const int slot = (int)(k % (uint32_t)L.nslot);
        if (!(ok = wait_warp(full(slot), (k / (uint32_t)L.nslot) & 1u, G))) break;
        const uint8_t* sq = qsm + L.off_slot + slot * L.slot_bytes;
        const float* ss = reinterpret_cast<const float*>(sq + L.qbytes);
        int lr[RW];   // rows of the slot
        int64_t row[RW];  // rows of the expert
        bool rv[RW];
        if (MODE == GEMV_ACT) {  // act rows j, j+1: gate rows j, j+1, up rows F+j, F+j+1
            const int j = r0 + warp * 2;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                rv[i] = rv[2 + i] = j + i < a.F;
                lr[i] = warp * 2 + i;
                lr[2 + i] = IROWS / 2 + warp * 2 + i;
                row[i] = j + i;
                row[2 + i] = (int64_t)a.F + j + i;
            }
        } else {
#pragma unroll
            for (int i = 0; i < RW; ++i) {
                lr[i] = warp * RW + i;
                row[i] = (int64_t)r0 + lr[i];
                rv[i] = row[i] < R;
            }
        }
        for (int t0 = 0; ok && t0 < n; t0 += L.qt) {
            if (u != xs_u || t0 != xs_t0) {  // next activation pass
                if (xsl >= 0) {
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(xempty(xsl));
                }
                xsl = (int)(xk % NXS);
                if (!(ok = wait_warp(xfull(xsl), (xk / NXS) & 1u, G))) break;
                xs_u = u;
                xs_t0 = t0;
                ++xk;
            }
            const float4* xs = reinterpret_cast<const float4*>(qsm + xsl * L.xbytes);
            const int nt = min(L.qt, n - t0);
            auto emit = [&](int t, const float (&v)[RW]) {
                const int p = s0 + t0 + t;
                if (MODE == GEMV_ACT) {
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        if (!rv[i]) continue;
                        if (a.gu_out) {
                            a.gu_out[(int64_t)p * a.gu_stride + row[i]] = v[i];
                            a.gu_out[(int64_t)p * a.gu_stride + row[2 + i]] = v[2 + i];
                        }
                        const float y = act_fn(v[i], v[2 + i], a.act);
                        if (a.out_qlayout)
                            a.out[(int64_t)p * a.out_stride + qpos(row[i])] = y * qscale(row[i]);
                        else
                            a.out[(int64_t)p * a.out_stride + row[i]] = y;
                    }
                } else {
                    const int64_t orow = a.out_row ? a.out_row[p] : p;
#pragma unroll
                    for (int i = 0; i < RW; ++i)
                        if (rv[i]) a.out[orow * a.out_stride + row[i]] = v[i];
                }
            };
            // one instantiation per token count keeps missing tokens out of the FMAs
            auto pass = [&](auto ntc) {
                constexpr int NT = decltype(ntc)::value;
                float res[RW][NT];
                rows_dot<NT>(sq, ss, lr, xs, K, res);
                if (lane == 0)
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        const float v[RW] = {res[0][t], res[1][t], res[2][t], res[3][t]};
                        emit(t, v);
                    }
            };
            if (nt == 1) pass(std::integral_constant<int, 1>{});
            else if (nt == 2) pass(std::integral_constant<int, 2>{});
            else if (nt == 3) pass(std::integral_constant<int, 3>{});
            else pass(std::integral_constant<int, 4>{});
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(empty(slot));
    }
}

// ------------------------------------------------------------ one token
// k_gemv1: the expert GEMV when every expert has at most one token (a
// one-token batch).  One warp per output row (ACT: per activation row, i.e.
// gate row j and up row F + j), no shared-memory staging: each lane streams
// its 16-byte chunks of the row straight from HBM (all of them requested
// before the first is used) and reads the token's q-layout activations
// through L1 (every warp of the expert reads the same row).  Without a ring
// or a copy warp the kernel needs few registers, so many warps per SM hide
// the latency that bounds k_dgemv at one token.  The per-chunk arithmetic,
// the order of the chunk sums in a lane and the warp reduction are
// rows_dot's, so the results equal k_dgemv's bit for bit.
namespace {

constexpr int G1_WARPS = 8;     // warps per CTA
constexpr int G1_MAXIT = 4;     // chunks per lane and row (K <= 4096)
constexpr int G1_MAXU = 1024;   // experts staged in shared memory

// UR: row units per task (ACT: activation rows, each a gate and an up row;
// PLAIN: rows), IT: 16-byte chunks per lane and row (ceil(K / 1024)).
template <int MODE, int UR, int IT>
__global__ void __launch_bounds__(G1_WARPS * 32) k_gemv1(GemvArgs a) {
    __shared__ int s_base[G1_MAXU];  // expert id of unique expert u
    __shared__ int s_pair[G1_MAXU];
    __shared__ int s_xrow[G1_MAXU];
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int K = a.K, nc = K >> 5;
    const int R = (int)a.rows_per_expert;
    const int rows_tile = (MODE == GEMV_ACT) ? a.F : R;
    const int U = a.meta[0];
    // the experts' indices once per CTA: no dependent index loads per task
    for (int u = threadIdx.x; u < U; u += blockDim.x) {
        const int p = a.seg_start[u];
        s_base[u] = a.unique_expert[u];
        s_pair[u] = p;
        s_xrow[u] = a.pair_row ? a.pair_row[p] : p;
    }
    __syncthreads();
    const unsigned long long m01 = pkf(-8388616.0f, -8388736.0f);
    const unsigned long long m23 = pkf(-8390656.0f, -8421376.0f);
    uint32_t mk[4] = {0xFu, 0xF0u, 0xF00u, 0xF000u}, magic = 0x4B000000u;
    asm volatile("" : "+r"(mk[0]), "+r"(mk[1]), "+r"(mk[2]), "+r"(mk[3]), "+r"(magic));
    constexpr int NR = (MODE == GEMV_ACT) ? 2 * UR : UR;  // weight rows per task
    const int tasks_per_expert = (rows_tile + UR - 1) / UR;
    const int ntask = U * tasks_per_expert;
    for (int task = blockIdx.x * G1_WARPS + (threadIdx.x >> 5); task < ntask; task += gridDim.x * G1_WARPS) {
        const int u = task / tasks_per_expert;
        const int j0 = (task - u * tasks_per_expert) * UR;
        const int64_t ebase = (int64_t)s_base[u] * R;
        const int p = s_pair[u];
        // every chunk of the task's rows in flight before the first is used
        uint4 q[NR][IT];
        float sc[NR][IT];
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            const int ju = j0 + (MODE == GEMV_ACT ? r / 2 : r);
            const int64_t row = (MODE == GEMV_ACT && (r & 1)) ? (int64_t)a.F + ju : ju;
            const bool rv = ju < rows_tile;
            const uint8_t* wr = a.Wp + (ebase + row) * (K / 2);
            const float* sr = a.Ws + (ebase + row) * nc;
#pragma unroll
            for (int it = 0; it < IT; ++it) {
                const int c = lane + 32 * it;
                const bool live = rv && c < nc;
                q[r][it] = live ? ldg_stream(wr + (int64_t)c * 16) : make_uint4(0, 0, 0, 0);
                sc[r][it] = live ? ldg_stream_f(sr + c) : 0.f;
            }
        }
        const float4* xs = reinterpret_cast<const float4*>(a.X + (int64_t)s_xrow[u] * K);
        float res[NR];
#pragma unroll
        for (int r = 0; r < NR; ++r) res[r] = 0.f;
#pragma unroll
        for (int it = 0; it < IT; ++it) {
            const int c = lane + 32 * it;
            const bool live = c < nc;
            const float4* xc = xs + (live ? (c << 3) : 0);
            const int sw = live ? (c & 7) : 0;
            unsigned long long acc[NR];
#pragma unroll
            for (int r = 0; r < NR; ++r) acc[r] = 0ull;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float4 f = __ldg(xc + ((2 * w + h) ^ sw));  // pre-scaled activations
                    const unsigned long long x01 = pkf(f.x, f.y), x23 = pkf(f.z, f.w);
#pragma unroll
                    for (int r = 0; r < NR; ++r) {
                        const uint4 qq = q[r][it];
                        const uint32_t word = w == 0 ? qq.x : w == 1 ? qq.y : w == 2 ? qq.z : qq.w;
                        const uint32_t uu = h ? (word >> 16) : word;
                        const unsigned long long v01 =
                            fadd2(pk2(tc::and_or(uu, mk[0], magic), tc::and_or(uu, mk[1], magic)), m01);
                        const unsigned long long v23 =
                            fadd2(pk2(tc::and_or(uu, mk[2], magic), tc::and_or(uu, mk[3], magic)), m23);
                        acc[r] = ffma2(v01, x01, acc[r]);
                        acc[r] = ffma2(v23, x23, acc[r]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const float2 a2 = upk(acc[r]);
                res[r] = fmaf(sc[r][it], a2.x + a2.y, res[r]);
            }
        }
#pragma unroll
        for (int r = 0; r < NR; ++r) res[r] = warp_sum(res[r]);
        if (lane == 0) {
#pragma unroll
            for (int uu = 0; uu < UR; ++uu) {
                const int j = j0 + uu;
                if (j >= rows_tile) break;
                if (MODE == GEMV_ACT) {
                    const float g = res[2 * uu], up = res[2 * uu + 1];
                    if (a.gu_out) {
                        a.gu_out[(int64_t)p * a.gu_stride + j] = g;
                        a.gu_out[(int64_t)p * a.gu_stride + a.F + j] = up;
                    }
                    const float y = act_fn(g, up, a.act);
                    if (a.out_qlayout)
                        a.out[(int64_t)p * a.out_stride + qpos(j)] = y * qscale(j);
                    else
                        a.out[(int64_t)p * a.out_stride + j] = y;
                } else {
                    const int64_t orow = a.out_row ? a.out_row[p] : p;
                    a.out[orow * a.out_stride + j] = res[uu];
                }
            }
        }
    }
}

}  // namespace

bool gemv1_supported(const GemvArgs& a) {
    return a.dense_tokens == 0 && a.max_tokens == 1 && a.x_qlayout && a.K % 32 == 0 && a.K <= 32 * 32 * G1_MAXIT &&
           a.max_unique <= G1_MAXU && a.rows_per_expert < (1LL << 30) &&
           (reinterpret_cast<uintptr_t>(a.Wp) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.Ws) & 3) == 0 &&
           (reinterpret_cast<uintptr_t>(a.X) & 15) == 0 && (a.K / 2) % 16 == 0;
}

int launch_gemv1(int mode, const GemvArgs& a, int num_sms, cudaStream_t s) {
    // rows per task: enough 16-byte chunks in flight per warp (about 8 per
    // lane) to cover the HBM latency with the warps an SM holds
    const int it = (a.K / 32 + 31) / 32;
    const int ur = mode == GEMV_ACT ? (it >= 3 ? 2 : 4) : (it >= 3 ? 2 : (it == 2 ? 4 : 8));
    const int64_t rows_tile = mode == GEMV_ACT ? a.F : a.rows_per_expert;
    const int64_t tasks = (rows_tile + ur - 1) / ur * a.max_unique;
    int64_t grid = (tasks + G1_WARPS - 1) / G1_WARPS;
    if (grid > (int64_t)num_sms * 8) grid = (int64_t)num_sms * 8;  // the CTAs stride over the rest
    if (grid <= 0) return 0;
    const dim3 g((unsigned)grid), b(G1_WARPS * 32);
    auto go = [&](auto kern) { launch_k(kern, g, b, 0, s, a); };
    if (mode == GEMV_ACT) {
        if (it == 1) go(k_gemv1<GEMV_ACT, 4, 1>);
        else if (it == 2) go(k_gemv1<GEMV_ACT, 4, 2>);
        else if (it == 3) go(k_gemv1<GEMV_ACT, 2, 3>);
        else go(k_gemv1<GEMV_ACT, 2, 4>);
    } else {
        if (it == 1) go(k_gemv1<GEMV_PLAIN, 8, 1>);
        else if (it == 2) go(k_gemv1<GEMV_PLAIN, 4, 2>);
        else if (it == 3) go(k_gemv1<GEMV_PLAIN, 2, 3>);
        else go(k_gemv1<GEMV_PLAIN, 2, 4>);
    }
    return 1;
}

// Whole blocks of rows only (every bulk copy a multiple of 16 bytes at a
// 16-byte aligned address), activations in the q layout, two item slots fit.
bool dgemv_supported(const GemvArgs& a, int mode) {
    if (a.dense_tokens != 0 || a.K % 32 != 0 || !a.x_qlayout) return false;
    const int64_t nb = a.K / 32;
    const int64_t tile = mode == GEMV_ACT ? a.F : a.rows_per_expert;
    const int64_t item = mode == GEMV_ACT ? QRows<GEMV_ACT>::ITEM : QRows<GEMV_PLAIN>::ITEM;
    if (tile % item != 0 || (a.rows_per_expert * nb) % 4 != 0 || (mode == GEMV_ACT && (a.F * nb) % 4 != 0))
        return false;
    if (qlay(a.K, a.max_tokens).nslot < 2) return false;
    return (reinterpret_cast<uintptr_t>(a.Wp) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.Ws) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(a.X) & 15) == 0;
}

int launch_dgemv(int mode, const GemvArgs& a, int num_sms, cudaStream_t s) {
    const int64_t rows_tile = mode == GEMV_ACT ? a.F : a.rows_per_expert;
    const int item = mode == GEMV_ACT ? QRows<GEMV_ACT>::ITEM : QRows<GEMV_PLAIN>::ITEM;
    const int64_t items = ((rows_tile + item - 1) / item) * a.max_unique;
    const int64_t cap = num_sms;
    const int grid = (int)(items < cap ? items : cap);
    if (grid <= 0) return 0;
    const int smem = qlay(a.K, a.max_tokens).total;
    if (mode == GEMV_ACT) {
        if (cudaFuncSetAttribute(k_dgemv<GEMV_ACT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return -1;
        launch_k(k_dgemv<GEMV_ACT>, dim3(grid), dim3(QTHREADS), (size_t)smem, s, a);
    } else {
        if (cudaFuncSetAttribute(k_dgemv<GEMV_PLAIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return -1;
        launch_k(k_dgemv<GEMV_PLAIN>, dim3(grid), dim3(QTHREADS), (size_t)smem, s, a);
    }
    return 1;
}

int launch_to_qlayout(const float* x, float* xq, int64_t rows, int K, int num_sms, cudaStream_t s) {
    const int64_t n = rows * K;
    int64_t blocks = (n + 255) / 256;
    if (blocks > (int64_t)num_sms * 4) blocks = (int64_t)num_sms * 4;
    if (blocks <= 0) return 0;
    launch_k(k_to_qlayout, dim3((unsigned)blocks), dim3(256), 0, s, x, xq, rows, K);
    return 1;
}

}  // namespace moe
