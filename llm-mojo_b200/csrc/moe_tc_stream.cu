// moe_tc_stream.cu -- streaming variant of the tcgen05 grouped Q4_0 GEMM
// for token tiles of 16..64 tokens and K % 128 == 0 (MOE_OPT_TC_STREAM:
// by default the expert GEMMs whose K allows it, i.e. gate/up).
//
// Same contraction, work list, K order and epilogues as k_tc_gemm
// (moe_tc.cu), organised as one CTA per SM with all 512 TMEM columns
// (measured 12-18 % faster than k_tc_gemm on the gate/up GEMM at 16-256
// tokens):
//  - a stage covers 256 K: the 128 weight rows' 128 packed bytes (two TMA
//    boxes of 128 B x 64 rows, SWIZZLE_128B), their eight block scales (two
//    TMA boxes of 8 fp32 x 64 rows) and the token tile's activations (one 3-D
//    TMA box that lands in the UMMA no-swizzle K-major layout);
//  - the producer prefetches the CTA's next work item into L2 as whole
//    contiguous row blocks (cp.async.bulk.prefetch.L2);
//  - two groups of four dequant warps take alternate stages; the thread that
//    owns A-tile row t turns the row's 256 weights into fp16 in TMEM with
//    tcgen05.st.32x32b.x32 (128-K A slots).  (w & 0x000F000F) | 0x64006400
//    is 1024 + n and (w & 0x00F000F0) | 0x54005400 is 64 + n, so (n - 8) is
//    one exact fp16 subtraction, then one multiply by the fp16 scale;
//  - epilogue warps wait with back-off.
//  - with the A operand in TMEM a tcgen05.mma of M=128, N=16, K=16 holds
//    its issuing thread for about 100 cycles, so two threads (warps 1 and
//    14) issue the MMAs of alternate stages into separate accumulators,
//    which the epilogue adds.
//
// Every mbarrier wait is bounded (globaltimer deadline); on expiry the kernel
// raises err_flag = 2, every role drains what it issued and the CTA frees
// its TMEM and returns.
#include <cuda.h>

#include "common.cuh"
#include "moe_tc.h"
#include "tc_ptx.cuh"

namespace moe {
namespace tc {

constexpr int ST_K = 256;                       // K per stage
constexpr int ST_Q = 128 * ST_K / 2;            // packed bytes per stage (16384)
constexpr int ST_S = 128 * 32;                  // scale bytes per stage (8 fp32 per row)
constexpr int ST_DQ0 = 2;                       // warps 2-9: dequant, two groups of four
constexpr int ST_EPI0 = ST_DQ0 + 8;             // warps 10-13: epilogue
constexpr int ST_MMA2 = ST_EPI0 + 4;            // warp 14: second MMA issuer
constexpr int ST_NMMA = 2;                      // MMA issuers: warp 1 (even stages), warp 14 (odd)
constexpr int ST_THREADS = 32 * (ST_MMA2 + 1);  // 480

template <int BN>
struct StLayout {
    static constexpr int ACC = ((2 * ST_NMMA * BN + 31) / 32) * 32;  // two buffers x two issuers
    static constexpr int SA = (512 - ACC) / 64 > 7 ? 7 : (512 - ACC) / 64;  // 128-K fp16 A slots in TMEM
    static constexpr int B_BYTES = BN * ST_K * 2;
    static constexpr int SLOT = ST_Q + B_BYTES + ST_S;
    static constexpr int SQ = (227 * 1024 - 2048) / SLOT > 8 ? 8 : (227 * 1024 - 2048) / SLOT;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_B = OFF_Q + SQ * ST_Q;
    static constexpr int OFF_S = OFF_B + SQ * B_BYTES;
    static constexpr int OFF_BAR = OFF_S + SQ * ST_S;
    static constexpr int N_BAR = 2 * SQ + 2 * SA + 4 + ST_NMMA;
    static constexpr int OFF_MISC = OFF_BAR + N_BAR * 8;
    static constexpr int TOTAL = OFF_MISC + 16 + 1024;  // + alignment slack
};

// L2 prefetch of [p, p + bytes), trimmed inwards to 16-byte boundaries, in
// pieces of at most 64 KB.
__device__ __forceinline__ void l2_prefetch_range(const uint8_t* p, int64_t bytes) {
    uintptr_t b = (reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15);
    const uintptr_t e = (reinterpret_cast<uintptr_t>(p) + (uintptr_t)bytes) & ~uintptr_t(15);
    while (b < e) {
        const uint32_t n = (uint32_t)((e - b) < 65536u ? (e - b) : 65536u);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(b), "r"(n) : "memory");
        b += n;
    }
}
// Whole-warp wait: every lane waits, and the warp leaves together (a lane
// that saw the deadline makes all of them give up), so .sync.aligned
// instructions after it always run with the full warp.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t a, uint32_t parity, const Guard& g) {
    const bool ok = mbar_wait(a, parity, g);
    return __all_sync(0xffffffffu, ok) != 0;
}

// Wait with back-off for roles that are far from the critical path.
__device__ __forceinline__ bool mbar_wait_sleep(uint32_t a, uint32_t parity, const Guard& g) {
    for (uint32_t it = 0;; ++it) {
        if (mbar_try(a, parity)) return true;
        if (it >= 2) __nanosleep(256);
        if ((it & 31u) == 31u) {
            if (*g.abort) return false;
            if (globaltimer() > g.deadline) {
                *g.abort = 1;
                atomicExch(g.err, 2);
                return false;
            }
        }
    }
}

// fp16 pair (lo = element p, hi = element p + 4 of the word's 8-group) of
// (nibble - 8) * scale; P selects the nibble pair 0..3 of the 32-bit word.
template <int P>
__device__ __forceinline__ uint32_t deq_pair(uint32_t w, __half2 sc) {
    const uint32_t v = (P < 2 ? w : (w >> 8));
    uint32_t m;
    if (P % 2 == 0) m = (v & 0x000F000Fu) | 0x64006400u;  // 1024 + n
    else m = (v & 0x00F000F0u) | 0x54005400u;             // 64 + n
    const __half2 off = (P % 2 == 0) ? __half2(__float2half(1032.0f), __float2half(1032.0f))
                                     : __half2(__float2half(72.0f), __float2half(72.0f));
    const __half2 x = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&m), off), sc);
    return *reinterpret_cast<const uint32_t*>(&x);
}

template <int MODE, int BN>
__global__ void __launch_bounds__(ST_THREADS, 1)
    k_tc_stream(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap bmap,
                const __grid_constant__ CUtensorMap smap, TcArgs a, const uint8_t* wp, int64_t total_rows) {
    using L = StLayout<BN>;
    constexpr int SQ = L::SQ;
    constexpr int SA = L::SA;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t bar0 = smem_u32(smem + L::OFF_BAR);
    auto q_full = [&](int s) { return bar0 + 8u * s; };
    auto q_empty = [&](int s) { return bar0 + 8u * (SQ + s); };
    auto a_full = [&](int s) { return bar0 + 8u * (2 * SQ + s); };
    auto a_empty = [&](int s) { return bar0 + 8u * (2 * SQ + SA + s); };
    auto acc_full = [&](int s) { return bar0 + 8u * (2 * SQ + 2 * SA + s); };
    auto acc_empty = [&](int s) { return bar0 + 8u * (2 * SQ + 2 * SA + 2 + s); };
    auto drain_bar = [&](int j) { return bar0 + 8u * (2 * SQ + 2 * SA + 4 + j); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = a.K, nb = K / 32, nst = (K + ST_K - 1) / ST_K;
    auto s_begin = [&](const Item& it) { return (int)((int64_t)it.ks * nst / a.ksplit); };
    auto s_end = [&](const Item& it) { return (int)((int64_t)(it.ks + 1) * nst / a.ksplit); };
    const int row_tiles = (MODE == TC_ACT) ? (a.F / 64) : (int)((a.R + 127) / 128);
    // TMA rows of the two 64-row boxes of an item
    auto box_rows = [&](const Item& it, int& ra, int& rb) {
        if (MODE == TC_ACT) {
            ra = (int)((int64_t)it.e * a.R + it.rt * 64);
            rb = (int)((int64_t)it.e * a.R + a.F + it.rt * 64);
        } else {
            ra = (int)((int64_t)it.e * a.R + it.rt * 128);
            rb = ra + 64;
        }
    };
    constexpr uint32_t ACOL = (uint32_t)L::ACC;
    // long deadline for draining work that is already in flight (it always ends)
    const uint64_t drain_ns = a.timeout_ns > 2000000000ull ? a.timeout_ns : 2000000000ull;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SQ; ++s) {
            mbar_init(q_full(s), 1);       // TMA: Q4 tile, its scales, activations
            mbar_init(q_empty(s), 4 + 1);  // the dequant group's four warps + the MMAs reading the activations
        }
        for (int s = 0; s < SA; ++s) {
            mbar_init(a_full(s), 4);
            mbar_init(a_empty(s), 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(acc_full(s), ST_NMMA);
            mbar_init(acc_empty(s), 4);
        }
        for (int j = 0; j < ST_NMMA; ++j) mbar_init(drain_bar(j), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        prefetch_tmap(&qmap);
        prefetch_tmap(&bmap);
        prefetch_tmap(&smap);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512u)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();  // barrier init, TMEM allocation and tensor-map prefetch overlap the previous kernel
    pdl_trigger();
    Guard G{abort_flag, a.err_flag, globaltimer() + a.timeout_ns};

    if (warp == 0) {
        // ------------------------------------------------ TMA producer (one thread)
        // An item's weight rows are one (PLAIN) or two (ACT: gate and up)
        // contiguous blocks of rows x K/2 bytes, plus their scale rows;
        // prefetching the next item into L2 in one piece keeps DRAM accesses
        // long and sequential while the ring's TMA boxes (128 bytes of each
        // of 128 rows per stage) read from L2.
        auto prefetch_item = [&](int64_t item) {
            Item pi;
            if (!decode_item(a, item, row_tiles, BN, pi) || pi.ks != 0) return;
            int ra, rb;
            box_rows(pi, ra, rb);
            const int64_t nrow = (MODE == TC_ACT) ? 64 : 128;
            const int nblk = (MODE == TC_ACT) ? 2 : 1;
            for (int b = 0; b < nblk; ++b) {
                const int64_t r0 = (b == 0) ? ra : rb;
                const int64_t r1 = (r0 + nrow < total_rows) ? r0 + nrow : total_rows;
                if (r1 <= r0) continue;
                l2_prefetch_range(wp + r0 * (K / 2), (r1 - r0) * (K / 2));
                l2_prefetch_range(reinterpret_cast<const uint8_t*>(a.Ws + r0 * nb), (r1 - r0) * nb * 4);
            }
        };
        if (lane == 0) {
            prefetch_item(blockIdx.x);
            uint32_t st = 0;
            uint32_t q_armed = 0;  // stages armed in their current phase
            uint32_t q_par = 0;    // their parity, one bit per stage
            Item it;
            bool ok = true;
            for (int64_t item = blockIdx.x; ok && decode_item(a, item, row_tiles, BN, it); item += gridDim.x) {
                int row_a, row_b;
                box_rows(it, row_a, row_b);
                prefetch_item(item + gridDim.x);
                const int tok_row = it.s0 + it.tt * BN;
                for (int s = s_begin(it); s < s_end(it); ++s, ++st) {
                    const int qs = (int)(st % SQ);
                    const uint32_t qp = (st / SQ) & 1u;
                    if (!(ok = mbar_wait(q_empty(qs), qp ^ 1u, G))) break;
                    const uint32_t qd = smem_u32(smem + L::OFF_Q + qs * ST_Q);
                    const uint32_t sd = smem_u32(smem + L::OFF_S + qs * ST_S);
                    mbar_expect_tx(q_full(qs), ST_Q + ST_S + L::B_BYTES);
                    tma_load_2d(qd, &qmap, q_full(qs), s * (ST_K / 2), row_a);
                    tma_load_2d(qd + ST_Q / 2, &qmap, q_full(qs), s * (ST_K / 2), row_b);
                    tma_load_2d(sd, &smap, q_full(qs), s * (ST_K / 32), row_a);
                    tma_load_2d(sd + ST_S / 2, &smap, q_full(qs), s * (ST_K / 32), row_b);
                    tma_load_3d(smem_u32(smem + L::OFF_B + qs * L::B_BYTES), &bmap, q_full(qs), 0, tok_row,
                                s * (ST_K / 8));
                    q_armed |= 1u << qs;
                    q_par = (q_par & ~(1u << qs)) | (qp << qs);
                }
            }
            // every armed stage's bytes must have landed before exit
            Guard Gd{abort_flag, a.err_flag, globaltimer() + drain_ns};
            volatile int no_abort = 0;
            Gd.abort = &no_abort;
            for (int s = 0; s < SQ; ++s)
                if (q_armed & (1u << s)) mbar_wait(q_full(s), (q_par >> s) & 1u, Gd);
        }
        __syncwarp();
    } else if (warp == 1 || warp == ST_MMA2) {
        // ------------------------------------------------ MMA issuers
        // A tcgen05.mma of N <= 64 with A in TMEM holds its issuing thread for
        // about 100 cycles, so two threads issue: stage st goes to issuer
        // st % 2, each into its own accumulator, summed by the epilogue.
        const int me = (warp == 1) ? 0 : 1;
        if (lane == 0) {
            uint32_t st = 0;
            int ab = 0;
            uint32_t accp = 0;
            constexpr uint32_t IDESC = f16_idesc(128, BN);
            Item it;
            bool ok = true, issued = false;
            for (int64_t item = blockIdx.x; ok && decode_item(a, item, row_tiles, BN, it); item += gridDim.x) {
                if (!(ok = mbar_wait(acc_empty(ab), accp ^ 1u, G))) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)((ab * ST_NMMA + me) * BN);
                bool first = true;
                const int sb = s_begin(it), se = s_end(it);
                for (int s = sb; s < se && ok; ++s, ++st) {
                    if ((int)(st % ST_NMMA) != me) continue;
                    const int qs = (int)(st % SQ);
                    if (!(ok = mbar_wait(q_full(qs), (st / SQ) & 1u, G))) break;  // activations landed
                    const uint32_t bd = smem_u32(smem + L::OFF_B + qs * L::B_BYTES);
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t ag = 2u * st + (uint32_t)h;
                        const int as = (int)(ag % SA);
                        if (!(ok = mbar_wait(a_full(as), (ag / SA) & 1u, G))) break;
                        tc_fence_after();
                        const int kv = K - s * ST_K - 128 * h;
                        const int nk = kv >= 128 ? 8 : (kv > 0 ? kv / 16 : 0);
                        const uint32_t ta = tmem_base + ACOL + (uint32_t)(as * 64);
                        for (int k = 0; k < nk; ++k)
                            tc_mma_ts(d_tmem, ta + 8u * k,
                                      kmajor_plain_desc(bd + (uint32_t)((16 * h + 2 * k) * BN * 16), BN * 16, 128),
                                      IDESC, (!first) || h || k);
                        issued = true;
                        tc_commit(a_empty(as));
                    }
                    first = false;
                    if (!ok) break;
                    tc_commit(q_empty(qs));
                }
                if (!ok) break;
                tc_commit(acc_full(ab));
                if (++ab == 2) {
                    ab = 0;
                    accp ^= 1u;
                }
            }
            if (issued) {  // all of this thread's MMAs complete before TMEM is released
                tc_commit(drain_bar(me));
                Guard Gd{abort_flag, a.err_flag, globaltimer() + drain_ns};
                volatile int no_abort = 0;
                Gd.abort = &no_abort;
                mbar_wait(drain_bar(me), 0, Gd);
            }
        }
        __syncwarp();
    } else if (warp < ST_EPI0) {
        // ------------------------------------------------ dequant
        const int grp = (warp - ST_DQ0) >> 2;  // 0: even stages, 1: odd stages
        const int q = warp & 3;                // TMEM lane quarter
        const int t = q * 32 + lane;           // A-tile row = TMEM lane
        const int sr = (MODE == TC_ACT) ? ((lane < 16) ? 16 * q + lane : 64 + 16 * q + (lane - 16)) : t;
        const int swz = sr & 7;                // SWIZZLE_128B: 16-byte chunk ^= row % 8
        const uint32_t tl = tmem_base + ((uint32_t)(q * 32) << 16) + ACOL;
        uint32_t st = 0;
        Item it;
        bool ok = true;
        for (int64_t item = blockIdx.x; ok && decode_item(a, item, row_tiles, BN, it); item += gridDim.x) {
            const int ns = s_end(it) - s_begin(it);
            for (int i = (int)((uint32_t)(grp - (int)st) & 1u); i < ns && ok; i += 2) {
                const uint32_t gs = st + (uint32_t)i;
                const int qs = (int)(gs % SQ);
                if (!(ok = mbar_wait_warp(q_full(qs), (gs / SQ) & 1u, G))) break;
                const uint8_t* qrow = smem + L::OFF_Q + qs * ST_Q + sr * 128;
                const float4* sp = reinterpret_cast<const float4*>(smem + L::OFF_S + qs * ST_S + sr * 32);
                const float4 s0 = sp[0], s1 = sp[1];
                const float scl[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t ag = 2u * gs + (uint32_t)h;
                    const int as = (int)(ag % SA);
                    if (!(ok = mbar_wait_warp(a_empty(as), ((ag / SA) & 1u) ^ 1u, G))) break;
                    tc_fence_after();
#pragma unroll
                    for (int p2 = 0; p2 < 2; ++p2) {
                        uint32_t hv[32];
#pragma unroll
                        for (int cc = 0; cc < 2; ++cc) {
                            const int c = 4 * h + 2 * p2 + cc;  // chunk = Q4 block 8s + c
                            const uint4 wv = *reinterpret_cast<const uint4*>(qrow + ((c ^ swz) << 4));
                            const __half2 sc = __float2half2_rn(scl[c]);
                            const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                            for (int w = 0; w < 4; ++w) {
                                hv[16 * cc + 4 * w + 0] = deq_pair<0>(w4[w], sc);
                                hv[16 * cc + 4 * w + 1] = deq_pair<1>(w4[w], sc);
                                hv[16 * cc + 4 * w + 2] = deq_pair<2>(w4[w], sc);
                                hv[16 * cc + 4 * w + 3] = deq_pair<3>(w4[w], sc);
                            }
                        }
                        // store and wait in one statement: the 32 source registers stay untouched
                        // until the store has completed
                        asm volatile(
                            "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
                            "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n\t"
                            "tcgen05.wait::st.sync.aligned;" ::"r"(tl + (uint32_t)(as * 64 + 32 * p2)),
                            "r"(hv[0]), "r"(hv[1]), "r"(hv[2]), "r"(hv[3]), "r"(hv[4]), "r"(hv[5]), "r"(hv[6]),
                            "r"(hv[7]), "r"(hv[8]), "r"(hv[9]), "r"(hv[10]), "r"(hv[11]), "r"(hv[12]), "r"(hv[13]),
                            "r"(hv[14]), "r"(hv[15]), "r"(hv[16]), "r"(hv[17]), "r"(hv[18]), "r"(hv[19]),
                            "r"(hv[20]), "r"(hv[21]), "r"(hv[22]), "r"(hv[23]), "r"(hv[24]), "r"(hv[25]),
                            "r"(hv[26]), "r"(hv[27]), "r"(hv[28]), "r"(hv[29]), "r"(hv[30]), "r"(hv[31])
                            : "memory");
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(a_full(as));
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(q_empty(qs));
            }
            st += (uint32_t)ns;
        }
    } else if (warp < ST_MMA2) {
        // ------------------------------------------------ epilogue
        const int q = warp & 3;       // TMEM lane quarter this warp may access
        const int i = q * 32 + lane;  // accumulator row (A-tile row)
        constexpr int CW = BN < 32 ? BN : 32;
        uint32_t est = 0;             // global stage counter at the item's first stage
        int ab = 0;
        uint32_t accp = 0;
        Item it;
        bool ok = true;
        for (int64_t item = blockIdx.x; ok && decode_item(a, item, row_tiles, BN, it); item += gridDim.x) {
            ok = __all_sync(0xffffffffu, mbar_wait_sleep(acc_full(ab), accp, G)) != 0;
            if (!ok) break;
            tc_fence_after();
            const int nv = min(BN, it.n - it.tt * BN);
            const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * ST_NMMA * BN);
            const int ns = s_end(it) - s_begin(it);
            for (int c0 = 0; c0 < nv; c0 += CW) {
                float v[CW];
#pragma unroll
                for (int cc = 0; cc < CW; ++cc) v[cc] = 0.f;
                for (int j = 0; j < ST_NMMA; ++j) {  // the issuers that had a stage of this item
                    if ((j - (int)(est % ST_NMMA) + ST_NMMA) % ST_NMMA >= ns) continue;
                    float v2[CW];
                    tmem_ld<CW>(tbase + (uint32_t)(j * BN) + c0, v2);
#pragma unroll
                    for (int cc = 0; cc < CW; ++cc) v[cc] += v2[cc];
                }
                if (MODE == TC_ACT) {
                    const int j = it.rt * 64 + 16 * q + (lane & 15);  // act row
                    const int jp = (j & ~7) | kpos(j & 7);
#pragma unroll
                    for (int cc = 0; cc < CW; ++cc) {
                        const float up = __shfl_down_sync(0xffffffffu, v[cc], 16);
                        if (lane < 16 && c0 + cc < nv) {
                            const int p = it.s0 + it.tt * BN + c0 + cc;
                            a.act_out[(int64_t)p * a.F + jp] = __float2half_rn(act_fn(v[cc], up, a.act));
                        }
                    }
                } else {
                    const int64_t r = (int64_t)it.rt * 128 + i;
                    if (r < a.R) {
#pragma unroll
                        for (int cc = 0; cc < CW; ++cc) {
                            if (c0 + cc < nv) {
                                const int p = it.s0 + it.tt * BN + c0 + cc;
                                const int64_t orow = a.out_row ? a.out_row[p] : p;
                                a.y_out[it.ks * a.split_stride + orow * a.y_stride + r] = v[cc];
                            }
                        }
                    }
                }
            }
            est += (uint32_t)(s_end(it) - s_begin(it));
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty(ab));
            if (++ab == 2) {
                ab = 0;
                accp ^= 1u;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(512u) : "memory");
}

}  // namespace tc

namespace {

template <int MODE, int BN>
int launch_st(const TcLaunch& L, int num_sms, cudaStream_t s) {
    CUtensorMap qmap, bmap;
    if (!tc_make_map(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.Wp, (uint64_t)L.a.K / 2, (uint64_t)L.total_rows,
                     (uint64_t)L.a.K / 2, tc::ST_K / 2, 64, CU_TENSOR_MAP_SWIZZLE_128B))
        return -1;
    // activations as [K/8 chunks][rows][8 fp16]: one box per stage lands in the
    // UMMA no-swizzle K-major layout (8x8 core matrices of 128 contiguous bytes)
    const uint64_t bdims[3] = {8, (uint64_t)L.b_rows, (uint64_t)L.a.K / 8};
    const uint64_t bstr[2] = {(uint64_t)L.a.K * 2, 16};
    const uint32_t bbox[3] = {8, (uint32_t)BN, tc::ST_K / 8};
    if (!tc_make_map_nd(&bmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, L.B, 3, bdims, bstr, bbox, CU_TENSOR_MAP_SWIZZLE_NONE))
        return -1;
    // scales [rows][K/32] fp32: 8 blocks (one stage) of 64 rows per box
    CUtensorMap smap;
    if (!tc_make_map(&smap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, L.a.Ws, (uint64_t)L.a.K / 32, (uint64_t)L.total_rows,
                     (uint64_t)L.a.K / 32 * 4, tc::ST_K / 32, 64, CU_TENSOR_MAP_SWIZZLE_NONE))
        return -1;
    const int smem = tc::StLayout<BN>::TOTAL;
    auto kern = tc::k_tc_stream<MODE, BN>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -1;
    int grid = num_sms;  // one CTA per SM: it owns all 512 TMEM columns
    if (L.max_items > 0 && L.max_items < grid) grid = (int)L.max_items;
    if (grid <= 0) return 0;
    launch_k(kern, dim3(grid), dim3(tc::ST_THREADS), smem, s, qmap, bmap, smap, L.a, L.Wp, L.total_rows);
    return 1;
}

template <int MODE>
int launch_st_mode(const TcLaunch& L, int num_sms, cudaStream_t s) {
    switch (L.BN) {
        case 16: return launch_st<MODE, 16>(L, num_sms, s);
        case 32: return launch_st<MODE, 32>(L, num_sms, s);
        case 64: return launch_st<MODE, 64>(L, num_sms, s);
        default: return -1;
    }
}

}  // namespace

int launch_tc_stream(int mode, const TcLaunch& L, int num_sms, cudaStream_t s) {
    const int nst = (L.a.K + tc::ST_K - 1) / tc::ST_K;
    // the scale rows are read by TMA: their stride (K/8 bytes) must be a multiple of 16
    if (L.a.K < 128 || L.a.K % 128 != 0 || L.a.ksplit > nst) return -1;
    if ((reinterpret_cast<uintptr_t>(L.a.Ws) & 15u) != 0) return -1;
    return mode == TC_ACT ? launch_st_mode<TC_ACT>(L, num_sms, s) : launch_st_mode<TC_PLAIN>(L, num_sms, s);
}

}  // namespace moe
