// moe_tc_stream.cu -- streaming variant of the tcgen05 grouped Q4_0 GEMM
// for token tiles of 16..64 tokens and K % 64 == 0 (MOE_OPT_TC_STREAM: by
// default the expert GEMMs).
//
// Same contraction, work list, K order and epilogues as k_tc_gemm
// (moe_tc.cu), organised as one CTA per SM with all 512 TMEM columns:
//  - a stage covers 256 K: the 128 weight rows' 128 packed bytes (two TMA
//    boxes of 128 B x 64 rows, SWIZZLE_128B), their eight block scales (two
//    TMA boxes of 8 fp32 x 64 rows) and the token tile's activations (one 3-D
//    TMA box of four K-major SWIZZLE_128B tiles, BN rows x 64 K each);
//  - when K % 128 == 64 a scale row (K/8 bytes) is no multiple of 16 bytes
//    and no tensor map can describe it: the producer then copies each work
//    item's scale rows, which are contiguous, with one or two bulk copies;
//  - NG groups of four dequant warps (three for 16-token tiles, two for
//    wider ones) take the stages in turn; the thread that owns A-tile row t
//    reads the row's 128 bytes of the stage into registers,
//    hands the slot back to the producer, and turns the 256 weights into
//    fp16 in TMEM with tcgen05.st.32x32b.x32 (128-K A slots).
//    (w & 0x000F000F) | 0x64006400 is 1024 + n and (w & 0x00F000F0) |
//    0x54005400 is 64 + n, so (n - 8) is one exact fp16 subtraction, then
//    one multiply by the fp16 scale;
//  - the activation tile has its own barriers: it stays until the stage's
//    MMAs have read it, while the weight bytes go back as soon as they are in
//    registers;
//  - a tcgen05.mma holds its issuing thread for ~55 cycles whatever N is,
//    so NG threads (warp 1 and the warps after the epilogue) issue the MMAs
//    of their stages into separate accumulators, which the epilogue adds;
//  - every ring (stages, TMEM A slots) has one producer order and one
//    consumer order: stage st belongs to dequant group and issuer st % NG,
//    the stage ring is a multiple of NG slots and each group has its own A
//    slots.  An mbarrier parity wait cannot tell phase p from p - 2, so a
//    consumer that could reach a slot before its previous user had filled it
//    would pass the wait early.
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
constexpr int ST_DQ0 = 2;  // warp 0: TMA producer, warp 1: MMA issuer 0, then the dequant groups

template <int BN>
struct StLayout {
    // NG dequant groups of four warps and NG MMA issuers; stage st belongs to
    // group and issuer st % NG.  Three for 16-token tiles (the dequant warps
    // are latency-bound, 2 groups ran 1.36x faster than one); TMEM holds the
    // accumulators of only two issuers at wider tiles.
    static constexpr int NG = BN <= 16 ? 3 : 2;
    static constexpr int EPI0 = ST_DQ0 + 4 * NG;  // four epilogue warps
    static constexpr int MMAX = EPI0 + 4;         // MMA issuers 1 .. NG-1
    static constexpr int THREADS = 32 * (MMAX + NG - 1);
    static constexpr int ACC = ((2 * NG * BN + 31) / 32) * 32;  // two buffers x NG issuers
    static constexpr int SA = (512 - ACC) / 64 > 7 ? 7 : (512 - ACC) / 64;  // 128-K fp16 A slots in TMEM
    // The slots form one ring per dequant group / MMA issuer pair, SAG slots
    // each: a ring shared by two groups lets an issuer wait on a slot whose
    // previous writer (the other group) has not arrived yet, where the
    // mbarrier parity test matches the phase before and passes.
    static constexpr int SAG = SA / NG;
    static_assert(SAG >= 2, "each group needs two A slots");
    static constexpr int B_BYTES = BN * ST_K * 2;
    static constexpr int SLOT = ST_Q + B_BYTES + ST_S;
    // a multiple of NG, so that stage slot qs is always used by the same
    // dequant group and MMA issuer: each ring then has one producer and one
    // consumer order, which the mbarrier parity waits rely on
    static constexpr int SQ0 = (227 * 1024 - 2048) / SLOT > 8 ? 8 : (227 * 1024 - 2048) / SLOT;
    static constexpr int SQ = (SQ0 / NG) * NG;
    static_assert(SQ >= NG, "stage ring must split evenly between the issuers");
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_B = OFF_Q + SQ * ST_Q;
    static constexpr int OFF_S = OFF_B + SQ * B_BYTES;
    // item-scale mode (K % 128 == 64): the scale area holds NIB item buffers
    // of 128 rows x K/32 fp32 (K <= 768), as many as fit up to four: with two,
    // the producer could not copy an item's scales (nor issue its stages)
    // before the item two back was fully dequantised
    static constexpr int ISCALE_BYTES = 12288;
    static constexpr int NIB0 = (227 * 1024 - 3072 - WL_SMEM - 1024 - OFF_S) / ISCALE_BYTES;
    static constexpr int NIB = NIB0 > 4 ? 4 : NIB0;
    static_assert(NIB >= 2, "two item-scale buffers at least");
    static constexpr int S_AREA = SQ * ST_S > NIB * ISCALE_BYTES ? SQ * ST_S : NIB * ISCALE_BYTES;
    static constexpr int OFF_BAR = OFF_S + S_AREA;
    static constexpr int BAR_IS = 2 * SQ + 2 * SA + 4 + NG;  // first item-scale barrier
    static constexpr int N_BAR = BAR_IS + 2 * NIB + 2 * SQ;
    static constexpr int OFF_MISC = OFF_BAR + N_BAR * 8;
    static constexpr int OFF_WL = OFF_MISC + 16;        // the work list (stage_worklist)
    static constexpr int TOTAL = OFF_WL + WL_SMEM + 1024;  // + alignment slack
    static_assert(TOTAL <= 227 * 1024, "shared memory");
};

// fp16 pair (lo = element p, hi = element p + 4 of the word's 8-group) of
// (nibble - 8) * scale; P selects the nibble pair 0..3 of the 32-bit word.
template <int P>
__device__ __forceinline__ uint32_t deq_pair(uint32_t w, __half2 sc) {
    const uint32_t v = (P < 2 ? w : (w >> 8));
    // one LOP3 each (and_or): 1024 + n, or 64 + n
    const uint32_t m = (P % 2 == 0) ? and_or(v, 0x000F000Fu, 0x64006400u) : and_or(v, 0x00F000F0u, 0x54005400u);
    const __half2 off = (P % 2 == 0) ? __half2(__float2half(1032.0f), __float2half(1032.0f))
                                     : __half2(__float2half(72.0f), __float2half(72.0f));
    const __half2 x = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&m), off), sc);
    return *reinterpret_cast<const uint32_t*>(&x);
}

template <int MODE, int BN>
__global__ void __launch_bounds__(StLayout<BN>::THREADS, 1)
    k_tc_stream(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap bmap,
                const __grid_constant__ CUtensorMap smap, TcArgs a, int64_t total_rows,
                int iscale) {
    using L = StLayout<BN>;
    constexpr int NG = L::NG;
    constexpr int SQ = L::SQ;
    constexpr int SA = L::SA;
    constexpr int SAG = L::SAG;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned by pointer arithmetic on the __shared__ array: through
    // an integer cast the compiler loses the address space and every read of
    // the rings becomes a generic load (the L1TEX path, long-scoreboard waits)
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t bar0 = smem_u32(smem + L::OFF_BAR);
    auto q_full = [&](int s) { return bar0 + 8u * s; };
    auto q_empty = [&](int s) { return bar0 + 8u * (SQ + s); };
    auto a_full = [&](int s) { return bar0 + 8u * (2 * SQ + s); };
    auto a_empty = [&](int s) { return bar0 + 8u * (2 * SQ + SA + s); };
    auto acc_full = [&](int s) { return bar0 + 8u * (2 * SQ + 2 * SA + s); };
    auto acc_empty = [&](int s) { return bar0 + 8u * (2 * SQ + 2 * SA + 2 + s); };
    auto drain_bar = [&](int j) { return bar0 + 8u * (2 * SQ + 2 * SA + 4 + j); };
    // item scales: all of an item's scale rows in one bulk copy (K % 128 == 64,
    // where the 2-D scale tensor map cannot exist); buffers b = 0 .. NIB-1
    constexpr int NIB = L::NIB;
    auto is_full = [&](int b) { return bar0 + 8u * (L::BAR_IS + b); };
    auto is_empty = [&](int b) { return bar0 + 8u * (L::BAR_IS + NIB + b); };
    // activation tiles: same slot index as the stage, own barriers, so a
    // stage's weight bytes are released by the dequant group alone and the
    // tile stays until the stage's MMAs have read it
    auto b_full = [&](int s) { return bar0 + 8u * (L::BAR_IS + 2 * NIB + s); };
    auto b_empty = [&](int s) { return bar0 + 8u * (L::BAR_IS + 2 * NIB + SQ + s); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = a.K, nb = K / 32, nst = (K + ST_K - 1) / ST_K;
    // 32-bit: every role evaluates these per item (ks < ksplit <= 16, nst < 2^16)
    auto s_begin = [&](const Item& it) { return it.ks * nst / a.ksplit; };
    auto s_end = [&](const Item& it) { return (it.ks + 1) * nst / a.ksplit; };
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
            mbar_init(q_full(s), 1);   // TMA: Q4 tile and its scales
            mbar_init(q_empty(s), 4);  // the dequant group's four warps
            mbar_init(b_full(s), 1);   // TMA: activation tile
            mbar_init(b_empty(s), 1);  // the MMAs that read it
        }
        for (int s = 0; s < SA; ++s) {
            mbar_init(a_full(s), 4);
            mbar_init(a_empty(s), 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(acc_full(s), NG);
            mbar_init(acc_empty(s), 4);
        }
        for (int j = 0; j < NG; ++j) mbar_init(drain_bar(j), 1);
        for (int b = 0; b < NIB; ++b) {
            mbar_init(is_full(b), 1);
            mbar_init(is_empty(b), 4 * NG);  // every dequant warp
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        prefetch_tmap(&qmap);
        prefetch_tmap(&bmap);
        if (!iscale) prefetch_tmap(&smap);
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
    const WorkList wl = stage_worklist(a, reinterpret_cast<int*>(smem + L::OFF_WL));
    Guard G{abort_flag, a.err_flag, globaltimer() + a.timeout_ns};

    if (warp == 0) {
        // ------------------------------------------------ TMA producer (one thread)
        // (a whole-item L2 prefetch ahead of the ring, tried here, cost 10-12 %:
        // the TMA ring alone keeps enough bytes in flight)
        if (lane == 0) {
            uint32_t st = 0;
            uint32_t q_armed = 0;  // stages armed in their current phase
            uint32_t q_par = 0;    // their parity, one bit per stage (activation tiles: the same)
            uint32_t b_armed = 0;
            uint32_t is_armed = 0, is_par = 0;
            uint32_t ii = 0;       // items of this CTA so far
            Item it;
            bool ok = true;
            for (int64_t item = blockIdx.x; ok && decode_item(wl, item, row_tiles, BN, it); item += gridDim.x, ++ii) {
                int row_a, row_b;
                box_rows(it, row_a, row_b);
                const int tok_row = it.s0 + it.tt * BN;
                if (iscale) {
                    const int b = (int)(ii % NIB);
                    const uint32_t ph = (ii / NIB) & 1u;
                    if (!(ok = mbar_wait(is_empty(b), ph ^ 1u, G))) break;
                    const uint32_t dst = smem_u32(smem + L::OFF_S + b * L::ISCALE_BYTES);
                    const uint32_t blk = (MODE == TC_ACT ? 64u : 128u) * (uint32_t)nb * 4u;
                    mbar_expect_tx(is_full(b), (MODE == TC_ACT ? 2u : 1u) * blk);
                    asm volatile(
                        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                        "l"(a.Ws + (int64_t)row_a * nb), "r"(blk), "r"(is_full(b))
                        : "memory");
                    if (MODE == TC_ACT)
                        asm volatile(
                            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                                dst + blk),
                            "l"(a.Ws + (int64_t)row_b * nb), "r"(blk), "r"(is_full(b))
                            : "memory");
                    is_armed |= 1u << b;
                    is_par = (is_par & ~(1u << b)) | (ph << b);
                }
                for (int s = s_begin(it); s < s_end(it); ++s, ++st) {
                    const int qs = (int)(st % SQ);
                    const uint32_t qp = (st / SQ) & 1u;
                    if (!(ok = mbar_wait(q_empty(qs), qp ^ 1u, G))) break;
                    const uint32_t qd = smem_u32(smem + L::OFF_Q + qs * ST_Q);
                    const uint32_t sd = smem_u32(smem + L::OFF_S + qs * ST_S);
                    mbar_expect_tx(q_full(qs), ST_Q + (iscale ? 0 : ST_S));
                    // one copy for the 128 rows' bytes and one for their scales: in ACT
                    // mode the maps see the weights as [2E][F][.] (gate and up halves),
                    // a box takes 64 rows of the gate half and the same 64 of the up half
                    if (MODE == TC_ACT) {
                        tma_load_3d(qd, &qmap, q_full(qs), s * (ST_K / 2), it.rt * 64, 2 * it.e);
                        if (!iscale) tma_load_3d(sd, &smap, q_full(qs), s * (ST_K / 32), it.rt * 64, 2 * it.e);
                    } else {
                        tma_load_2d(qd, &qmap, q_full(qs), s * (ST_K / 2), row_a);
                        if (!iscale) tma_load_2d(sd, &smap, q_full(qs), s * (ST_K / 32), row_a);
                    }
                    q_armed |= 1u << qs;
                    q_par = (q_par & ~(1u << qs)) | (qp << qs);
                    if (!(ok = mbar_wait(b_empty(qs), qp ^ 1u, G))) break;
                    mbar_expect_tx(b_full(qs), L::B_BYTES);
                    tma_load_3d(smem_u32(smem + L::OFF_B + qs * L::B_BYTES), &bmap, b_full(qs), 0, tok_row,
                                s * (ST_K / 64));
                    b_armed |= 1u << qs;
                }
            }
            // every armed stage's bytes must have landed before exit
            Guard Gd{abort_flag, a.err_flag, globaltimer() + drain_ns};
            volatile int no_abort = 0;
            Gd.abort = &no_abort;
            for (int s = 0; s < SQ; ++s) {
                if (q_armed & (1u << s)) mbar_wait(q_full(s), (q_par >> s) & 1u, Gd);
                if (b_armed & (1u << s)) mbar_wait(b_full(s), (q_par >> s) & 1u, Gd);
            }
            for (int b = 0; b < NIB; ++b)
                if (is_armed & (1u << b)) mbar_wait(is_full(b), (is_par >> b) & 1u, Gd);
        }
        __syncwarp();
    } else if (warp == 1 || (warp >= L::MMAX && warp < L::MMAX + NG - 1)) {
        // ------------------------------------------------ MMA issuers
        // A tcgen05.mma of N <= 64 with A in TMEM holds its issuing thread for
        // about 100 cycles, so two threads issue: stage st goes to issuer
        // st % 2, each into its own accumulator, summed by the epilogue.
        const int me = (warp == 1) ? 0 : warp - L::MMAX + 1;
        if (lane == 0) {
            uint32_t st = 0;
            int ab = 0;
            uint32_t accp = 0;
            constexpr uint32_t IDESC = f16_idesc(128, BN);
            Item it;
            bool ok = true, issued = false;
            for (int64_t item = blockIdx.x; ok && decode_item(wl, item, row_tiles, BN, it); item += gridDim.x) {
                if (!(ok = mbar_wait(acc_empty(ab), accp ^ 1u, G))) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)((ab * NG + me) * BN);
                bool first = true;
                const int sb = s_begin(it), se = s_end(it);
                for (int s = sb; s < se && ok; ++s, ++st) {
                    if ((int)(st % NG) != me) continue;
                    const int qs = (int)(st % SQ);
                    if (!(ok = mbar_wait(b_full(qs), (st / SQ) & 1u, G))) break;  // activations landed
                    // One thread issues every MMA, so the loop is unrolled with the
                    // descriptors as constant offsets of one base: computed per MMA,
                    // they held the issuer ~190 cycles per tcgen05.mma instead of ~55.
                    const uint64_t bdesc = sw128_desc(smem_u32(smem + L::OFF_B + qs * L::B_BYTES));
#pragma unroll 1
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t la = 2u * (st / NG) + (uint32_t)h;  // place in this issuer's ring
                        const int as = me * SAG + (int)(la % SAG);
                        if (!(ok = mbar_wait(a_full(as), (la / SAG) & 1u, G))) break;
                        tc_fence_after();
                        const int kv = K - s * ST_K - 128 * h;
                        const uint32_t ta = tmem_base + ACOL + (uint32_t)(as * 64);
                        const uint32_t acc = (!first || h) ? 1u : 0u;
                        // B sub-tile of k: 64-K chunk 2h + k/4, 32 bytes per 16 K inside its rows
                        auto boff = [&](int k) { return (uint64_t)(((2 * h + k / 4) * BN * 128 + 32 * (k % 4)) >> 4); };
                        if (kv >= 128) {
#pragma unroll
                            for (int k = 0; k < 8; ++k)
                                tc_mma_ts(d_tmem, ta + 8u * k, bdesc + boff(k), IDESC, acc | (k > 0 ? 1u : 0u));
                        } else {  // the K tail (kv is a multiple of 64)
                            const int nk = kv > 0 ? kv / 16 : 0;
                            for (int k = 0; k < nk; ++k)
                                tc_mma_ts(d_tmem, ta + 8u * k, bdesc + boff(k), IDESC, acc | (k > 0 ? 1u : 0u));
                        }
                        issued = true;
                        tc_commit(a_empty(as));
                    }
                    first = false;
                    if (!ok) break;
                    tc_commit(b_empty(qs));
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
    } else if (warp < L::EPI0) {
        // ------------------------------------------------ dequant
        const int grp = (warp - ST_DQ0) >> 2;  // takes the stages st with st % NG == grp
        const int q = warp & 3;                // TMEM lane quarter
        const int t = q * 32 + lane;           // A-tile row = TMEM lane
        const int sr = (MODE == TC_ACT) ? ((lane < 16) ? 16 * q + lane : 64 + 16 * q + (lane - 16)) : t;
        const int swz = sr & 7;                // SWIZZLE_128B: 16-byte chunk ^= row % 8
        const uint32_t tl = tmem_base + ((uint32_t)(q * 32) << 16) + ACOL;
        uint32_t st = 0, ii = 0;
        Item it;
        bool ok = true;
        for (int64_t item = blockIdx.x; ok && decode_item(wl, item, row_tiles, BN, it); item += gridDim.x, ++ii) {
            const int ns = s_end(it) - s_begin(it);
            const float* iscl = nullptr;  // item-scale mode: this row's scales
            if (iscale) {
                const int b = (int)(ii % NIB);
                if (!(ok = mbar_wait_warp(is_full(b), (ii / NIB) & 1u, G))) break;
                iscl = reinterpret_cast<const float*>(smem + L::OFF_S + b * L::ISCALE_BYTES) + sr * nb;
            }
            for (int i = (grp - (int)(st % NG) + NG) % NG; i < ns && ok; i += NG) {
                const uint32_t gs = st + (uint32_t)i;
                const int qs = (int)(gs % SQ);
                if (!(ok = mbar_wait_warp(q_full(qs), (gs / SQ) & 1u, G))) break;
                const uint8_t* qrow = smem + L::OFF_Q + qs * ST_Q + sr * 128;
                float scl[8];
                if (iscale) {  // 8-byte aligned: nb is even
                    const float2* sp2 = reinterpret_cast<const float2*>(iscl + 8 * (s_begin(it) + i));
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        const float2 f = sp2[v];
                        scl[2 * v] = f.x;
                        scl[2 * v + 1] = f.y;
                    }
                } else {
                    const float4* sp = reinterpret_cast<const float4*>(smem + L::OFF_S + qs * ST_S + sr * 32);
                    const float4 s0 = sp[0], s1 = sp[1];
                    scl[0] = s0.x; scl[1] = s0.y; scl[2] = s0.z; scl[3] = s0.w;
                    scl[4] = s1.x; scl[5] = s1.y; scl[6] = s1.z; scl[7] = s1.w;
                }
                // the row's 128 bytes of this stage into registers: the slot
                // goes back to the producer before any wait on the MMAs
                uint4 wq[8];
#pragma unroll
                for (int c = 0; c < 8; ++c) wq[c] = *reinterpret_cast<const uint4*>(qrow + ((c ^ swz) << 4));
                __syncwarp();
                if (lane == 0) mbar_arrive(q_empty(qs));
                // The two 128-K halves run as a loop, not unrolled: one copy of
                // the dequant code keeps the hot loop small for the instruction
                // cache, which three dequant warps and the issuers share per SM
                // sub-partition.  The second half's chunks move into wq[0..3].
#pragma unroll 1
                for (int h = 0; h < 2; ++h) {
                    // Four 16-column chunks through two 16-register buffers: a
                    // chunk's TMEM store runs while the next is computed (the
                    // store reads its registers when it issues; one wait before
                    // the hand-off covers all four), and the small live set lets
                    // the compiler build each store's consecutive registers in
                    // place (with two 32-register blocks it spent ~55 moves per
                    // half).  The first chunk's math comes before the wait for
                    // the A slot.
                    auto deq_chunk = [&](int c, uint32_t (&hv)[16]) {  // chunk = Q4 block 8s + 4h + c
                        const uint4 wv = wq[c];
                        const __half2 sc = __float2half2_rn(scl[c]);
                        const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            hv[4 * w + 0] = deq_pair<0>(w4[w], sc);
                            hv[4 * w + 1] = deq_pair<1>(w4[w], sc);
                            hv[4 * w + 2] = deq_pair<2>(w4[w], sc);
                            hv[4 * w + 3] = deq_pair<3>(w4[w], sc);
                        }
                    };
                    auto st16 = [&](uint32_t col, const uint32_t (&hv)[16]) {
                        asm volatile(
                            "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(tl + col),
                            "r"(hv[0]), "r"(hv[1]), "r"(hv[2]), "r"(hv[3]), "r"(hv[4]), "r"(hv[5]), "r"(hv[6]), "r"(hv[7]),
                            "r"(hv[8]), "r"(hv[9]), "r"(hv[10]), "r"(hv[11]), "r"(hv[12]), "r"(hv[13]), "r"(hv[14]), "r"(hv[15])
                            : "memory");
                    };
                    auto st_wait = [&]() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); };
                    const uint32_t la = 2u * (gs / NG) + (uint32_t)h;  // place in this group's ring
                    const int as = grp * SAG + (int)(la % SAG);
                    const uint32_t apar = ((la / SAG) & 1u) ^ 1u;
                    // the slot is nearly always free by now: a non-blocking test
                    // ahead of the math hides its latency; the bounded wait only
                    // when it was not
                    const uint32_t early = (lane == 0) ? (mbar_test(a_empty(as), apar) ? 1u : 0u) : 0u;
                    uint32_t b0[16], b1[16];
                    deq_chunk(0, b0);
                    if (__shfl_sync(0xffffffffu, early, 0) == 0u) {
                        if (!(ok = mbar_wait_warp1(a_empty(as), apar, G))) break;
                    } else {
                        __syncwarp();
                    }
                    tc_fence_after();
                    const uint32_t c0 = (uint32_t)(as * 64);
                    st16(c0, b0);
                    deq_chunk(1, b1);
                    st16(c0 + 16, b1);
                    deq_chunk(2, b0);
                    st16(c0 + 32, b0);
                    deq_chunk(3, b1);
                    // the wait covers every store: the MMAs may read the slot after it
                    st16(c0 + 48, b1);
                    st_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(a_full(as));
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        wq[c] = wq[c + 4];
                        scl[c] = scl[c + 4];
                    }
                }
                if (!ok) break;
            }
            if (!ok) break;
            if (iscale) {
                __syncwarp();
                if (lane == 0) mbar_arrive(is_empty((int)(ii % NIB)));
            }
            st += (uint32_t)ns;
        }
    } else if (warp < L::EPI0 + 4) {
        // ------------------------------------------------ epilogue
        const int q = warp & 3;       // TMEM lane quarter this warp may access
        const int i = q * 32 + lane;  // accumulator row (A-tile row)
        constexpr int CW = BN < 32 ? BN : 32;
        uint32_t est = 0;             // global stage counter at the item's first stage
        int ab = 0;
        uint32_t accp = 0;
        Item it;
        bool ok = true;
        for (int64_t item = blockIdx.x; ok && decode_item(wl, item, row_tiles, BN, it); item += gridDim.x) {
            // lane 0 waits (suspended in hardware, no issue slots), the tcgen05
            // fence after the warp's sync orders the accumulator loads.  A
            // __nanosleep back-off loop here cost ~0.9 M instructions per
            // launch: the sleep may end at once, and the four warps share
            // their SM sub-partitions with the dequant warps.
            ok = mbar_wait_warp1(acc_full(ab), accp, G);
            if (!ok) break;
            tc_fence_after();
            const int nv = min(BN, it.n - it.tt * BN);
            const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * NG * BN);
            const int ns = s_end(it) - s_begin(it);
            for (int c0 = 0; c0 < nv; c0 += CW) {
                float v[CW];
#pragma unroll
                for (int cc = 0; cc < CW; ++cc) v[cc] = 0.f;
                for (int j = 0; j < NG; ++j) {  // the issuers that had a stage of this item
                    if ((j - (int)(est % NG) + NG) % NG >= ns) continue;
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
    // Q4 rows [rows][K/2] bytes and scales [rows][K/32] fp32, one stage (256 K)
    // of 128 rows per copy: ACT as [2E][F][.] (box: 64 rows of a gate half and
    // of the matching up half), PLAIN as [rows][.] (box: 128 rows).  When the
    // scale row stride is not a multiple of 16 bytes (K % 128 == 64) no map
    // can describe the scales and the kernel copies each item's scale rows in
    // one piece instead.
    CUtensorMap qmap, bmap;
    const int iscale = (L.a.K % 128) != 0;
    CUtensorMap smap;
    const uint64_t kq = (uint64_t)L.a.K / 2, ks = (uint64_t)L.a.K / 32;
    if (MODE == TC_ACT) {
        const uint64_t halves = (uint64_t)L.total_rows / (uint64_t)L.a.F;
        const uint64_t qd[3] = {kq, (uint64_t)L.a.F, halves};
        const uint64_t qst[2] = {kq, kq * (uint64_t)L.a.F};
        const uint32_t qb[3] = {tc::ST_K / 2, 64, 2};
        if (!tc_make_map_nd(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.Wp, 3, qd, qst, qb, CU_TENSOR_MAP_SWIZZLE_128B))
            return -1;
        smap = qmap;
        const uint64_t sdm[3] = {ks, (uint64_t)L.a.F, halves};
        const uint64_t sst[2] = {ks * 4, ks * 4 * (uint64_t)L.a.F};
        const uint32_t sb[3] = {tc::ST_K / 32, 64, 2};
        if (!iscale && !tc_make_map_nd(&smap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, L.a.Ws, 3, sdm, sst, sb,
                                       CU_TENSOR_MAP_SWIZZLE_NONE))
            return -1;
    } else {
        if (!tc_make_map(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.Wp, kq, (uint64_t)L.total_rows, kq, tc::ST_K / 2,
                         128, CU_TENSOR_MAP_SWIZZLE_128B))
            return -1;
        smap = qmap;
        if (!iscale && !tc_make_map(&smap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, L.a.Ws, ks, (uint64_t)L.total_rows,
                                    ks * 4, tc::ST_K / 32, 128, CU_TENSOR_MAP_SWIZZLE_NONE))
            return -1;
    }
    // activations as [K/64 chunks][rows][64 fp16]: one box per stage lands as
    // four UMMA K-major SWIZZLE_128B tiles of BN rows x 64 K (128-byte rows,
    // so the TMA moves whole 128-byte lines)
    const uint64_t bdims[3] = {64, (uint64_t)L.b_rows, (uint64_t)L.a.K / 64};
    const uint64_t bstr[2] = {(uint64_t)L.a.K * 2, 128};
    const uint32_t bbox[3] = {64, (uint32_t)BN, tc::ST_K / 64};
    if (!tc_make_map_nd(&bmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, L.B, 3, bdims, bstr, bbox, CU_TENSOR_MAP_SWIZZLE_128B))
        return -1;
    if (iscale) {
        const int64_t nb = L.a.K / 32;
        if (128 * nb * 4 > tc::StLayout<BN>::ISCALE_BYTES) return -1;
        // every item's scale block starts on a 16-byte boundary and is whole
        // (each copy covers 64 or 128 whole rows of one expert)
        if (MODE == TC_PLAIN && L.a.R % 128 != 0) return -1;
        if (MODE == TC_ACT && L.a.F % 64 != 0) return -1;
        if ((L.a.R * nb) % 4 != 0) return -1;
    }
    const int smem = tc::StLayout<BN>::TOTAL;
    auto kern = tc::k_tc_stream<MODE, BN>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -1;
    int grid = num_sms;  // one CTA per SM: it owns all 512 TMEM columns
    if (L.max_items > 0 && L.max_items < grid) grid = (int)L.max_items;
    if (grid <= 0) return 0;
    launch_k(kern, dim3(grid), dim3(tc::StLayout<BN>::THREADS), smem, s, qmap, bmap, smap, L.a, L.total_rows, iscale);
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
    if (L.a.K < 128 || L.a.K % 64 != 0 || L.a.ksplit > nst) return -1;
    if ((reinterpret_cast<uintptr_t>(L.a.Ws) & 15u) != 0) return -1;
    return mode == TC_ACT ? launch_st_mode<TC_ACT>(L, num_sms, s) : launch_st_mode<TC_PLAIN>(L, num_sms, s);
}

}  // namespace moe
