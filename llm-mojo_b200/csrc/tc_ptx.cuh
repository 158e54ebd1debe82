// tc_ptx.cuh -- PTX wrappers shared by the tcgen05 GEMM kernels (sm_100a):
// mbarriers with bounded waits, TMA loads, tcgen05 MMA / TMEM access, UMMA
// descriptors, and the grouped work-item decoder.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "moe_tc.h"

namespace moe {
namespace tc {

// ------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t a) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t a, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}
// Non-blocking test of a phase (no suspension): issued ahead of other work
// its latency overlaps that work.
__device__ __forceinline__ bool mbar_test(uint32_t a, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    return ok != 0;
}
// A thread whose phase is not complete sleeps in the hardware until it
// completes or `kSuspendNs` pass: without the hint the time limit is short and
// the waiting loops spin, taking issue slots from the warps that work.
constexpr uint32_t kSuspendNs = 20000;
__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return ok != 0;
}

// (a & b) | c as one LOP3: with both constants in registers the mask and the
// magic exponent do not compete for the instruction's one immediate (written
// in C++ the pair compiles to two LOP3s).
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

struct Guard {
    volatile int* abort;  // shared flag
    int* err;
    uint64_t deadline;
};

// Waits for the phase of `parity`; false when the deadline passed or another
// role aborted (then the caller stops issuing work).
__device__ __forceinline__ bool mbar_wait(uint32_t a, uint32_t parity, const Guard& g) {
    for (uint32_t it = 0;; ++it) {
        if (mbar_try(a, parity)) return true;
        if ((it & 15u) == 15u) {
            if (*g.abort) return false;
            if (globaltimer() > g.deadline) {
                *g.abort = 1;
                atomicExch(g.err, 2);
                return false;
            }
        }
    }
}

// Whole-warp wait: every lane waits, and the warp leaves together (a lane
// that saw the deadline makes all of them give up), so .sync.aligned
// instructions after it always run with the full warp.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t a, uint32_t parity, const Guard& g) {
    const bool ok = mbar_wait(a, parity, g);
    return __all_sync(0xffffffffu, ok) != 0;
}
// Whole-warp wait where lane 0 alone polls: for barriers that guard no data
// the lanes read afterwards (a TMEM slot freed by MMAs; the tcgen05 fence
// after it orders the warp's stores).  32 lanes polling one barrier cost a
// few hundred cycles per wait.
__device__ __forceinline__ bool mbar_wait_warp1(uint32_t a, uint32_t parity, const Guard& g) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait(a, parity, g) ? 1 : 0;
    __syncwarp();
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t mbar,
                                            int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(mbar), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
                 : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// A from tensor memory (lanes = the 128 rows, 32-bit columns = K pairs)
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// tcgen05.st 32 lanes x 32 bit x 16 columns (this thread's lane, 16 values)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// tcgen05.st 32 lanes x 32 bit x 32 columns (this thread's lane, 32 values)
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// tcgen05.ld 32 lanes x 32 bit, N consecutive columns per thread
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float (&v)[N]);
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// UMMA shared-memory descriptor: K-major, SWIZZLE_128B, 8-row groups of
// 1024 bytes (SBO = 1024), version 1 (sm_100), LBO unused (1).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;                 // LBO (ignored for swizzled K-major)
    d |= (uint64_t)(1024u >> 4) << 32;       // SBO
    d |= (uint64_t)1u << 46;                 // version
    d |= (uint64_t)2u << 61;                 // SWIZZLE_128B
    return d;
}
// UMMA shared-memory descriptor: K-major without swizzle.  Core matrices are
// 8 rows x 16 bytes stored as 128 contiguous bytes; lbo = bytes between core
// matrices adjacent in K, sbo = bytes between core matrices adjacent in M/N.
__device__ __forceinline__ uint64_t kmajor_plain_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1u << 46;  // version
    return d;                 // layout type 0: no swizzle
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t mbar, int32_t x,
                                            int32_t y, int32_t z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(mbar), "r"(x), "r"(y), "r"(z)
        : "memory");
}
// Instruction descriptor, kind::f16: D f32, A f16, B f16, both K-major.
__host__ __device__ constexpr uint32_t f16_idesc(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// position of K element m (0..7) inside its group of 8
__device__ __forceinline__ int kpos(int m) { return m < 4 ? 2 * m : 2 * (m - 4) + 1; }

// ------------------------------------------------------------ work list
struct Item {
    int u, e, rt, tt, n, s0, ks;
};

// The grouped GEMMs' work list: the arrays the bucketing kernels wrote
// (unique experts, their token segments, the token-tile prefix), in shared
// memory once per CTA when they fit.  Every role of a kernel decodes every
// work item; from global memory each decode is a chain of about ten dependent
// L2 round trips (the binary search over the prefix), which cost the stream
// kernel's dequant warps about 14 % of their time.
constexpr int WL_CAP = 256;                       // experts staged in shared memory
constexpr int WL_SMEM = (4 * WL_CAP + 1) * 4;     // bytes
struct WorkList {
    const int* tt_prefix = nullptr;
    const int* unique_expert = nullptr;
    const int* seg_start = nullptr;
    const int* seg_count = nullptr;
    int U = 0;
    int dense_tokens = 0;
    int ksplit = 1;
};

// Every thread of the CTA calls this after griddepcontrol.wait (the lists are
// the previous kernels' output); it ends with __syncthreads.
__device__ __forceinline__ WorkList stage_worklist(const TcArgs& a, int* s_wl) {
    WorkList w;
    w.dense_tokens = a.dense_tokens;
    w.ksplit = a.ksplit;
    if (a.dense_tokens > 0) return w;
    const int U = a.meta[0];
    w.U = U;
    if (U <= WL_CAP) {
        int* sp = s_wl;
        int* se = s_wl + WL_CAP + 1;
        int* ss = se + WL_CAP;
        int* sc = ss + WL_CAP;
        for (int i = threadIdx.x; i <= U; i += blockDim.x) {
            sp[i] = a.tt_prefix[i];
            if (i < U) {
                se[i] = a.unique_expert[i];
                ss[i] = a.seg_start[i];
                sc[i] = a.seg_count[i];
            }
        }
        __syncthreads();
        w.tt_prefix = sp;
        w.unique_expert = se;
        w.seg_start = ss;
        w.seg_count = sc;
    } else {
        w.tt_prefix = a.tt_prefix;
        w.unique_expert = a.unique_expert;
        w.seg_start = a.seg_start;
        w.seg_count = a.seg_count;
    }
    return w;
}

// 32-bit arithmetic (work lists stay far below 2^31 items): 64-bit division
// by a run-time value is a long instruction sequence.
__device__ __forceinline__ bool decode_item(const WorkList& a, int64_t item64, int row_tiles, int BN,
                                            Item& it) {
    if (item64 >= 0x7FFFFFFF) return false;
    int item = (int)item64;
    if (a.ksplit > 1) {
        it.ks = item % a.ksplit;  // split-K index (PLAIN mode), fastest varying
        item /= a.ksplit;
    } else {
        it.ks = 0;
    }
    if (a.dense_tokens > 0) {
        const int ntt = (a.dense_tokens + BN - 1) / BN;
        if (item >= row_tiles * ntt) return false;
        it.u = 0;
        it.e = 0;
        it.rt = item / ntt;
        it.tt = item - it.rt * ntt;
        it.n = a.dense_tokens;
        it.s0 = 0;
        return true;
    }
    const int U = a.U;
    const int total = row_tiles * a.tt_prefix[U];
    if (item >= total) return false;
    int lo = 0, hi = U - 1;  // last u with row_tiles * tt_prefix[u] <= item
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (row_tiles * a.tt_prefix[mid] <= item) lo = mid;
        else hi = mid - 1;
    }
    const int u = lo;
    const int p0 = a.tt_prefix[u];
    const int ntt = a.tt_prefix[u + 1] - p0;
    const int rem = item - row_tiles * p0;
    it.u = u;
    it.e = a.unique_expert[u];
    it.rt = rem / ntt;
    it.tt = rem - it.rt * ntt;
    it.n = a.seg_count[u];
    it.s0 = a.seg_start[u];
    return true;
}

}  // namespace tc
}  // namespace moe
