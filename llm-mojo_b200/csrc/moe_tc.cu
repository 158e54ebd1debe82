// moe_tc.cu -- tensor-core grouped Q4_0 GEMM for sm_100a (tcgen05 + TMA).
//
// D[rows][tokens] = W_e[rows][K] . X[tokens][K]^T for every (expert, row
// tile, token tile) work item of a device-side list, "swap-AB": the weight
// rows are the MMA's M = 128, the tokens its N = BN.
//
// Warp roles (448 threads):
//   warp 0     TMA producer: packed Q4 tiles (SWIZZLE_32B) and fp16
//              activation tiles (SWIZZLE_128B) into smem rings.
//   warp 1     TMEM owner and single-thread tcgen05.mma issuer; fp32
//              accumulators live in TMEM, double-buffered across items.
//   warps 2-9  dequant: two warps per TMEM lane quarter; the thread owning
//              A-tile row t and K half h turns the row's 32 nibbles of that
//              half of a k-tile into fp16.  Two variants of the A operand:
//              A_TMEM (token tiles <= 64, memory-bound): (n-8) exact in fp16
//                via one LOP3 per nibble pair, times the fp16 scale (HMUL2),
//                stored with tcgen05.st straight into TMEM; the MMA reads A
//                from TMEM, so shared memory carries only the Q4 and
//                activation tiles.
//              A in shared memory (large token tiles, compute-bound):
//                (n-8)*scale in fp32, one rounding to fp16, stored in the UMMA
//                K-major SWIZZLE_128B layout.
//   warps 10-13 epilogue: tcgen05.ld of the accumulator; ACT mode pairs gate
//              and up rows with a warp shuffle and writes the activated
//              result as fp16, PLAIN mode writes fp32 rows.
//
// ACT tiles cover 64 act rows: TMA brings the 64 gate rows and the 64 up
// rows as two boxes; A-tile row t = 32q + l holds gate row 16q + l (l < 16)
// or up row 16q + l - 16 (l >= 16), so each TMEM lane quarter q (the lanes
// one epilogue warp may read) has a gate row and its up row 16 lanes apart.
//
// Inside every 8-element group of K, both operands are stored in the order
// [0,4,1,5,2,6,3,7]: the dequantiser produces nibble pairs (k, k+4) of a
// 32-bit word with one mask, and the activations are written in the same
// order (k_gather_f16 and the ACT epilogue), so the contraction is unchanged.
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

// ---------------------------------------------------------------- layout
constexpr int SA = 3;             // fp16 A ring stages (16 KB in smem, or 32 TMEM columns)
constexpr int KT = 64;            // K per k-tile
constexpr int THREADS = 448;
constexpr int DQ_WARPS = 8;        // warps 2-9: two per TMEM lane quarter, one K half each
constexpr int EPI_WARP0 = 2 + DQ_WARPS;

// Ring depths.  The producer issues a Q4 tile and an activation tile per
// k-tile and waits for a free slot in each ring, so the activation ring is at
// least as deep as the Q4 ring; small token tiles (memory-bound) keep 12 Q4
// tiles (48 KB) per CTA in flight.
template <int BN, bool A_TMEM>
struct Smem {
    static constexpr int SQ = A_TMEM ? (BN <= 32 ? 12 : 8) : 8;
    static constexpr int SB = A_TMEM ? (BN <= 32 ? 14 : 9) : 4;
    static constexpr int A_BYTES = 128 * KT * 2;          // 16384
    static constexpr int B_BYTES = BN * KT * 2;
    static constexpr int Q_BYTES = 128 * KT / 2;          // 4096
    static constexpr int OFF_A = 0;
    static constexpr int OFF_B = OFF_A + (A_TMEM ? 0 : SA * A_BYTES);
    static constexpr int OFF_Q = OFF_B + SB * B_BYTES;
    static constexpr int OFF_BAR = OFF_Q + SQ * Q_BYTES;
    static constexpr int N_BAR = 2 * SQ + 2 * SA + 2 * SB + 4 + 1;
    static constexpr int OFF_MISC = OFF_BAR + N_BAR * 8;
    static constexpr int OFF_WL = OFF_MISC + 16;          // the work list (stage_worklist)
    static constexpr int TOTAL = OFF_WL + WL_SMEM + 1024; // + alignment slack
};

__host__ __device__ constexpr uint32_t pow2_cols(int n) {
    return n <= 32 ? 32u : n <= 64 ? 64u : n <= 128 ? 128u : n <= 256 ? 256u : 512u;
}
// TMEM columns: two fp32 accumulator buffers of BN columns, then (A_TMEM)
// SA stages of the fp16 A tile, 32 columns (64 fp16 per lane) each.
__host__ __device__ constexpr int a_col0(int BN) { return ((2 * BN + 31) / 32) * 32; }
__host__ __device__ constexpr uint32_t tmem_cols(int BN, bool A_TMEM) {
    return pow2_cols(A_TMEM ? a_col0(BN) + SA * 32 : 2 * BN);
}

// -------------------------------------------------------------- kernel
// EXACT (shared-memory A only; the router's logits): fp32 dequant, one
// rounding of (n - 8) * scale.  A template parameter, so that the fp16 path's
// hot loop carries no second copy of the arithmetic.
template <int MODE, int BN, bool A_TMEM, bool EXACT>
__global__ void __launch_bounds__(THREADS, A_TMEM ? 2 : 1)
    k_tc_gemm(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap bmap, TcArgs a) {
    using L = Smem<BN, A_TMEM>;
    constexpr int SQ = L::SQ;
    constexpr int SB = L::SB;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned by pointer arithmetic on the __shared__ array: through
    // an integer cast the compiler loses the address space and every read of
    // the rings becomes a generic load (the L1TEX path, long-scoreboard waits)
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    const uint32_t bar0 = smem_u32(bars);
    auto q_full = [&](int s) { return bar0 + 8u * s; };
    auto q_empty = [&](int s) { return bar0 + 8u * (SQ + s); };
    auto a_full = [&](int s) { return bar0 + 8u * (2 * SQ + s); };
    auto a_empty = [&](int s) { return bar0 + 8u * (2 * SQ + SA + s); };
    auto b_full = [&](int s) { return bar0 + 8u * (2 * SQ + 2 * SA + s); };
    auto b_empty = [&](int s) { return bar0 + 8u * (2 * SQ + 2 * SA + SB + s); };
    auto acc_full = [&](int s) { return bar0 + 8u * (2 * SQ + 2 * SA + 2 * SB + s); };
    auto acc_empty = [&](int s) { return bar0 + 8u * (2 * SQ + 2 * SA + 2 * SB + 2 + s); };
    const uint32_t drain_bar = bar0 + 8u * (2 * SQ + 2 * SA + 2 * SB + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = a.K, nk = K / KT, nb = K / 32;
    auto k_begin = [&](const Item& it) { return (int)((int64_t)it.ks * nk / a.ksplit); };
    auto k_end = [&](const Item& it) { return (int)((int64_t)(it.ks + 1) * nk / a.ksplit); };
    const int row_tiles = (MODE == TC_ACT) ? (a.F / 64) : (int)((a.R + 127) / 128);
    constexpr uint32_t NCOL = tmem_cols(BN, A_TMEM);
    constexpr uint32_t ACOL = (uint32_t)a_col0(BN);

    if (threadIdx.x == 0) {
        for (int s = 0; s < SQ; ++s) {
            mbar_init(q_full(s), 1);
            mbar_init(q_empty(s), DQ_WARPS);
        }
        for (int s = 0; s < SA; ++s) {
            mbar_init(a_full(s), DQ_WARPS);
            mbar_init(a_empty(s), 1);
        }
        for (int s = 0; s < SB; ++s) {
            mbar_init(b_full(s), 1);
            mbar_init(b_empty(s), 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(acc_full(s), 1);
            mbar_init(acc_empty(s), 4);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        prefetch_tmap(&qmap);
        prefetch_tmap(&bmap);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(NCOL)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();  // barrier init, TMEM allocation and tensor-map prefetch overlap the previous kernel
    pdl_trigger();
    const WorkList wl = stage_worklist(a, reinterpret_cast<int*>(smem + L::OFF_WL));
    Guard G{abort_flag, a.err_flag, globaltimer() + a.timeout_ns};
    // draining work already in flight always ends: it gets at least 2 s,
    // whatever the (possibly much shorter) deadline of the work itself
    const uint64_t drain_ns = a.timeout_ns > 2000000000ull ? a.timeout_ns : 2000000000ull;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            int qs = 0, bs = 0;
            uint32_t qp = 0, bp = 0;
            uint32_t q_armed = 0, b_armed = 0;  // stages armed in their current phase
            uint32_t q_par[SQ], b_par[SB];
            Item it;
            bool ok = true;
            for (int64_t item = blockIdx.x; ok && decode_item(wl, item, row_tiles, BN, it); item += gridDim.x) {
                int row_a, row_b;  // first weight rows of the two 64-row halves
                if (MODE == TC_ACT) {
                    row_a = (int)((int64_t)it.e * a.R + it.rt * 64);
                    row_b = (int)((int64_t)it.e * a.R + a.F + it.rt * 64);
                } else {
                    row_a = (int)((int64_t)it.e * a.R + it.rt * 128);
                    row_b = row_a + 64;
                }
                const int tok_row = it.s0 + it.tt * BN;
                for (int kt = k_begin(it); kt < k_end(it); ++kt) {
                    if (!(ok = mbar_wait(q_empty(qs), qp ^ 1, G))) break;
                    uint8_t* qd = smem + L::OFF_Q + qs * L::Q_BYTES;
                    mbar_expect_tx(q_full(qs), L::Q_BYTES);
                    tma_load_2d(smem_u32(qd), &qmap, q_full(qs), kt * (KT / 2), row_a);
                    tma_load_2d(smem_u32(qd + L::Q_BYTES / 2), &qmap, q_full(qs), kt * (KT / 2), row_b);
                    q_armed |= 1u << qs;
                    q_par[qs] = qp;
                    if (++qs == SQ) { qs = 0; qp ^= 1; }
                    if (!(ok = mbar_wait(b_empty(bs), bp ^ 1, G))) break;
                    uint8_t* bd = smem + L::OFF_B + bs * L::B_BYTES;
                    mbar_expect_tx(b_full(bs), L::B_BYTES);
                    tma_load_2d(smem_u32(bd), &bmap, b_full(bs), kt * KT, tok_row);
                    b_armed |= 1u << bs;
                    b_par[bs] = bp;
                    if (++bs == SB) { bs = 0; bp ^= 1; }
                }
            }
            // drain: every armed stage's bytes must have landed before exit
            Guard Gd{abort_flag, a.err_flag, globaltimer() + drain_ns};
            volatile int no_abort = 0;
            Gd.abort = &no_abort;
            for (int s = 0; s < SQ; ++s)
                if (q_armed & (1u << s)) mbar_wait(q_full(s), q_par[s], Gd);
            for (int s = 0; s < SB; ++s)
                if (b_armed & (1u << s)) mbar_wait(b_full(s), b_par[s], Gd);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            int as = 0, bs = 0, ab = 0;
            uint32_t ap = 0, bp = 0, accp = 0;
            constexpr uint32_t IDESC = f16_idesc(128, BN);
            Item it;
            bool ok = true, issued = false;
            for (int64_t item = blockIdx.x; ok && decode_item(wl, item, row_tiles, BN, it); item += gridDim.x) {
                if (!(ok = mbar_wait(acc_empty(ab), accp ^ 1, G))) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(ab * BN);
                const int kb = k_begin(it);
                for (int kt = kb; kt < k_end(it); ++kt) {
                    if (!(ok = mbar_wait(a_full(as), ap, G))) break;
                    if (!(ok = mbar_wait(b_full(bs), bp, G))) break;
                    tc_fence_after();
                    // descriptors built once per k-tile: a K step of 16 fp16 is 32 bytes,
                    // i.e. 2 in the descriptor's 16-byte address field
                    const uint64_t bdesc = sw128_desc(smem_u32(smem + L::OFF_B + bs * L::B_BYTES));
                    if (A_TMEM) {
                        const uint32_t ta = tmem_base + ACOL + (uint32_t)(as * 32);
#pragma unroll
                        for (int k = 0; k < KT / 16; ++k)
                            tc_mma_ts(d_tmem, ta + 8u * k, bdesc + 2u * k, IDESC, (kt != kb) || k);
                    } else {
                        const uint64_t adesc = sw128_desc(smem_u32(smem + L::OFF_A + as * L::A_BYTES));
#pragma unroll
                        for (int k = 0; k < KT / 16; ++k)
                            tc_mma(d_tmem, adesc + 2u * k, bdesc + 2u * k, IDESC, (kt != kb) || k);
                    }
                    issued = true;
                    tc_commit(a_empty(as));
                    tc_commit(b_empty(bs));
                    if (++as == SA) { as = 0; ap ^= 1; }
                    if (++bs == SB) { bs = 0; bp ^= 1; }
                }
                if (!ok) break;
                tc_commit(acc_full(ab));
                if (++ab == 2) { ab = 0; accp ^= 1; }
            }
            if (issued) {  // all MMAs complete before TMEM is released
                tc_commit(drain_bar);
                Guard Gd{abort_flag, a.err_flag, globaltimer() + drain_ns};
                volatile int no_abort = 0;
                Gd.abort = &no_abort;
                mbar_wait(drain_bar, 0, Gd);
            }
        }
    } else if (warp < EPI_WARP0) {
        // ------------------------------------------------ dequant
        // A-tile row t follows the warp's TMEM lane quarter (warp % 4); the two
        // warps of a quarter take K half h = 0 / 1 of every k-tile (one 16-byte
        // Q4 chunk = one 32-weight block with its own scale).
        const int h = (warp - 2) >> 2;
        const int t = (warp & 3) * 32 + lane;
        int qs = 0, as = 0;
        uint32_t qp = 0, ap = 0;
        Item it;
        bool ok = true;
        for (int64_t item = blockIdx.x; ok && decode_item(wl, item, row_tiles, BN, it); item += gridDim.x) {
            int64_t grow;  // global weight row of this thread
            int sr;        // its row in the Q4 stage (gate box rows 0-63, up box 64-127)
            if (MODE == TC_ACT) {
                const int qq = t >> 5, l = t & 31;
                const int g = 16 * qq + (l & 15);
                sr = (l < 16) ? g : 64 + g;
                grow = (int64_t)it.e * a.R + (l < 16 ? it.rt * 64 + g : a.F + it.rt * 64 + g);
            } else {
                sr = t;
                grow = (int64_t)it.e * a.R + it.rt * 128 + t;
            }
            const bool row_ok = (MODE == TC_ACT) || (it.rt * 128 + t < a.R);
            const float* srow = a.Ws + grow * nb + h;  // scale of block 2*kt + h
            const int kb = k_begin(it), ke = k_end(it);
            // the scales PF k-tiles ahead in a shift register; the k-tile loop
            // is not unrolled (one copy of the body for the instruction cache)
            constexpr int PF = 8;
            float sreg[PF];
#pragma unroll
            for (int j = 0; j < PF; ++j) sreg[j] = (row_ok && kb + j < ke) ? __ldg(srow + 2 * (kb + j)) : 0.f;
#pragma unroll 1
            for (int kt = kb; kt < ke && ok; ++kt) {
                {
                    const float s = sreg[0];
#pragma unroll
                    for (int j = 0; j < PF - 1; ++j) sreg[j] = sreg[j + 1];
                    sreg[PF - 1] = (row_ok && kt + PF < ke) ? __ldg(srow + 2 * (kt + PF)) : 0.f;
                    if (!(ok = mbar_wait(q_full(qs), qp, G))) break;
                    // the A slot guards no data these lanes read: lane 0 waits
                    if (!(ok = mbar_wait_warp1(a_empty(as), ap ^ 1, G))) break;
                    const int sw = ((sr >> 2) & 1) << 4;  // SWIZZLE_32B: chunk ^= row bit 2
                    const uint4 c = *reinterpret_cast<const uint4*>(smem + L::OFF_Q + qs * L::Q_BYTES + sr * 32 +
                                                                     ((h << 4) ^ sw));
                    const uint32_t wv[4] = {c.x, c.y, c.z, c.w};
                    if (A_TMEM) {
                        tc_fence_after();
                        // (n-8) exact in fp16: (0x6400 | n) is 1024 + n; times the fp16 scale
                        const __half2 sc = __float2half2_rn(s);
                        const __half2 off = __float2half2_rn(1032.0f);
                        uint32_t hv[16];
#pragma unroll
                        for (int w = 0; w < 4; ++w)
#pragma unroll
                            for (int p = 0; p < 4; ++p) {
                                const uint32_t v = ((wv[w] >> (4 * p)) & 0x000F000Fu) | 0x64006400u;
                                const __half2 x = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&v), off), sc);
                                hv[4 * w + p] = *reinterpret_cast<const uint32_t*>(&x);
                            }
                        tmem_st16(tmem_base + ((uint32_t)((warp & 3) * 32) << 16) + ACOL + (uint32_t)(as * 32 + 16 * h),
                                  hv);
                        tc_fence_before();
                    } else {
                        // the same fp16 arithmetic as the tensor-memory variant:
                        // (0x6400 | n) is 1024 + n, minus 1032, times the fp16 scale
                        // (one LOP3, one HSUB2, one HMUL2 per pair)
                        // (a.exact_a: the router's logits, which decide the routing, keep
                        // fp32 arithmetic and one rounding of (n - 8) * scale)
                        uint8_t* arow = smem + L::OFF_A + as * L::A_BYTES + (t >> 3) * 1024 + (t & 7) * 128;
                        const __half2 sc = __float2half2_rn(s);
                        const __half2 off = __float2half2_rn(1032.0f);
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            uint32_t hh[4];
#pragma unroll
                            for (int p = 0; p < 4; ++p) {
                                const uint32_t v = ((wv[w] >> (4 * p)) & 0x000F000Fu) | 0x64006400u;
                                __half2 x;
                                if (EXACT) {
                                    const float lo = (__uint_as_float(0x4B000000u | (v & 0xFu)) - 8388616.0f) * s;
                                    const float hi = (__uint_as_float(0x4B000000u | ((v >> 16) & 0xFu)) - 8388616.0f) * s;
                                    x = __floats2half2_rn(lo, hi);
                                } else {
                                    x = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&v), off), sc);
                                }
                                hh[p] = *reinterpret_cast<const uint32_t*>(&x);
                            }
                            const int cw = 4 * h + w;  // 16-byte chunk of the 128-byte row
                            *reinterpret_cast<uint4*>(arow + ((cw ^ (t & 7)) << 4)) = make_uint4(hh[0], hh[1], hh[2], hh[3]);
                        }
                        fence_async_smem();
                    }
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(a_full(as));
                        mbar_arrive(q_empty(qs));
                    }
                    if (++qs == SQ) { qs = 0; qp ^= 1; }
                    if (++as == SA) { as = 0; ap ^= 1; }
                }
            }
        }
    } else {
        // ------------------------------------------------ epilogue
        const int q = warp & 3;       // TMEM lane quarter this warp may access
        const int i = q * 32 + lane;  // accumulator row (A-tile row)
        constexpr int CW = BN < 32 ? BN : 32;
        int ab = 0;
        uint32_t accp = 0;
        Item it;
        bool ok = true;
        for (int64_t item = blockIdx.x; ok && decode_item(wl, item, row_tiles, BN, it); item += gridDim.x) {
            ok = mbar_wait_warp1(acc_full(ab), accp, G);  // lane 0 waits; the fence orders the TMEM loads
            tc_fence_after();
            const int nv = min(BN, it.n - it.tt * BN);
            const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BN);
            for (int c0 = 0; ok && c0 < nv; c0 += CW) {
                float v[CW];
                tmem_ld<CW>(tbase + c0, v);
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
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty(ab));
            if (++ab == 2) { ab = 0; accp ^= 1; }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(NCOL) : "memory");
}

// ---------------------------------------------------------- helpers
// Token tiles per unique expert -> exclusive prefix (one CTA, U <= 1024).
__global__ void __launch_bounds__(1024) k_tt_prefix(const int* meta, const int* seg_count, int BN,
                                                    int* tt_prefix) {
    pdl_wait();
    pdl_trigger();
    __shared__ int wsum[32];
    const int U = meta[0];
    const int tid = threadIdx.x;
    const int v = tid < U ? (seg_count[tid] + BN - 1) / BN : 0;
    const int lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
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
    const int excl = (wid > 0 ? wsum[wid - 1] : 0) + x - v;
    if (tid < U) tt_prefix[tid] = excl;
    if (tid == 0) tt_prefix[U] = wsum[nw - 1];
}

// out[p][.] = fp16(X[row(p)][.]) with every 8-group of K in [0,4,1,5,2,6,3,7]
// order; rows p >= meta[1] (no pair) are skipped.
__global__ void __launch_bounds__(256) k_gather_f16(const float* X, int64_t K, const int* pair_row,
                                                    const int* meta, int dense_rows, __half* out) {
    pdl_wait();
    pdl_trigger();
    const int64_t p = blockIdx.x;
    const int64_t P = dense_rows > 0 ? dense_rows : meta[1];
    if (p >= P) return;
    const int64_t src = pair_row ? pair_row[p] : p;
    const float4* x4 = reinterpret_cast<const float4*>(X + src * K);
    uint4* o = reinterpret_cast<uint4*>(out + p * K);
    for (int64_t g = threadIdx.x; g < K / 8; g += blockDim.x) {
        const float4 a = __ldg(x4 + 2 * g), b = __ldg(x4 + 2 * g + 1);
        const __half2 h0 = __floats2half2_rn(a.x, b.x);  // elements 0,4
        const __half2 h1 = __floats2half2_rn(a.y, b.y);  // 1,5
        const __half2 h2 = __floats2half2_rn(a.z, b.z);  // 2,6
        const __half2 h3 = __floats2half2_rn(a.w, b.w);  // 3,7
        o[g] = make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                          *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
    }
}

}  // namespace tc

// ------------------------------------------------------------------ host
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn encode_fn() {
    static EncodeFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeFn>(p);
    }
    return fn;
}

bool tc_make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t rows,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
    EncodeFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


bool tc_make_map_nd(CUtensorMap* m, CUtensorMapDataType dt, const void* base, int rank, const uint64_t* dims,
                    const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle sw) {
    EncodeFn fn = encode_fn();
    if (!fn || rank < 1 || rank > 5) return false;
    cuuint64_t d[5], st[4];
    cuuint32_t b[5], es[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        es[i] = 1;
        if (i + 1 < rank) st[i] = strides[i];
    }
    return fn(m, dt, (cuuint32_t)rank, const_cast<void*>(base), d, st, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

template <int MODE, int BN, bool A_TMEM, bool EXACT = false>
int launch_t(const TcLaunch& L, int num_sms, cudaStream_t s) {
    CUtensorMap qmap, bmap;
    if (!tc_make_map(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.Wp, (uint64_t)L.a.K / 2, (uint64_t)L.total_rows,
                  (uint64_t)L.a.K / 2, 32, 64, CU_TENSOR_MAP_SWIZZLE_32B))
        return -1;
    if (!tc_make_map(&bmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, L.B, (uint64_t)L.a.K, (uint64_t)L.b_rows,
                  (uint64_t)L.a.K * 2, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B))
        return -1;
    const int smem = tc::Smem<BN, A_TMEM>::TOTAL;
    auto kern = tc::k_tc_gemm<MODE, BN, A_TMEM, EXACT>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -1;
    int per_sm = (227 * 1024) / smem;
    const int by_tmem = 512 / (int)tc::tmem_cols(BN, A_TMEM);
    if (per_sm > by_tmem) per_sm = by_tmem;
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) == cudaSuccess && fa.numRegs > 0) {
        const int by_regs = 65536 / (fa.numRegs * tc::THREADS);
        if (per_sm > by_regs) per_sm = by_regs;
    }
    if (per_sm > 2) per_sm = 2;
    if (per_sm < 1) per_sm = 1;
    int grid = num_sms * per_sm;
    if (L.max_items > 0 && L.max_items < grid) grid = (int)L.max_items;
    if (grid <= 0) return 0;
    launch_k(kern, dim3(grid), dim3(tc::THREADS), smem, s, qmap, bmap, L.a);
    return 1;
}

template <int MODE>
int launch_mode(const TcLaunch& L, int num_sms, cudaStream_t s) {
    if (MODE == TC_PLAIN && L.a.exact_a && (L.a_in_smem || L.BN >= 128)) {
        switch (L.BN) {  // the router's dense GEMM: shared-memory A, fp32 dequant
            case 16: return launch_t<MODE, 16, false, true>(L, num_sms, s);
            case 32: return launch_t<MODE, 32, false, true>(L, num_sms, s);
            case 64: return launch_t<MODE, 64, false, true>(L, num_sms, s);
            case 128: return launch_t<MODE, 128, false, true>(L, num_sms, s);
            case 256: return launch_t<MODE, 256, false, true>(L, num_sms, s);
            default: return -1;
        }
    }
    if (L.a_in_smem) {
        switch (L.BN) {
            case 16: return launch_t<MODE, 16, false>(L, num_sms, s);
            case 32: return launch_t<MODE, 32, false>(L, num_sms, s);
            case 64: return launch_t<MODE, 64, false>(L, num_sms, s);
            case 128: return launch_t<MODE, 128, false>(L, num_sms, s);
            case 256: return launch_t<MODE, 256, false>(L, num_sms, s);
            default: return -1;
        }
    }
    switch (L.BN) {  // A in TMEM: token tiles up to 64 (accumulators + A stages fit 256 columns)
        case 16: return launch_t<MODE, 16, true>(L, num_sms, s);
        case 32: return launch_t<MODE, 32, true>(L, num_sms, s);
        case 64: return launch_t<MODE, 64, true>(L, num_sms, s);
        case 128: return launch_t<MODE, 128, false>(L, num_sms, s);
        case 256: return launch_t<MODE, 256, false>(L, num_sms, s);
        default: return -1;
    }
}

}  // namespace

int launch_tc_gemm(int mode, const TcLaunch& L, int num_sms, cudaStream_t s) {
    if (L.stream && !L.a_in_smem && L.BN <= 64) {
        const int r = launch_tc_stream(mode, L, num_sms, s);
        if (r >= 0) return r;
    }
    return mode == TC_ACT ? launch_mode<TC_ACT>(L, num_sms, s) : launch_mode<TC_PLAIN>(L, num_sms, s);
}

// out[i] = sum over s < splits of part[s * stride + i] (fixed order)
__global__ void k_reduce_splits(const float* part, int64_t stride, int splits, float* out, int64_t n) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float v = part[i];
    for (int s = 1; s < splits; ++s) v += part[s * stride + i];
    out[i] = v;
}

int launch_reduce_splits(const float* part, int64_t stride, int splits, float* out, int64_t n,
                         cudaStream_t s) {
    if (n <= 0) return 0;
    launch_k(k_reduce_splits, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, part, stride, splits, out, n);
    return 1;
}

int launch_tt_prefix(const int* meta, const int* seg_count, int BN, int* tt_prefix, cudaStream_t s) {
    launch_k(tc::k_tt_prefix, dim3(1), dim3(1024), 0, s, meta, seg_count, BN, tt_prefix);
    return 1;
}

int launch_gather_f16(const float* X, int64_t K, const int* pair_row, const int* meta, int64_t rows,
                      int dense_rows, __half* out, cudaStream_t s) {
    if (rows <= 0) return 0;
    launch_k(tc::k_gather_f16, dim3((unsigned)rows), dim3(256), 0, s, X, K, pair_row, meta, dense_rows, out);
    return 1;
}

bool tc_supported(int64_t K, int64_t R, int act_mode, int64_t F) {
    if (K % 64 != 0 || K > 65536) return false;
    if (act_mode) return F % 64 == 0;
    return R > 0;
}

}  // namespace moe
