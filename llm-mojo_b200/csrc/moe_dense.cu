// moe_dense.cu -- one-launch Q4_0 projection for up to 16 tokens
// (q4_matmul_batchN at decode batch sizes: the attention projections of a
// decode step, model_speculative_moe_batched.mojo's q/k/v/o calls).
//
// out[t][r] = sum_k W[r][k] * x[t][k] for t < M <= 16, one CTA per (128-row
// tile, K range):
//   - the CTA converts its K range of the fp32 activations to fp16 itself,
//    straight into the UMMA K-major SWIZZLE_128B layout in shared memory (no
//    separate gather kernel; the K order inside every 8-group is
//    [0,4,1,5,2,6,3,7], the order the dequantiser produces);
//   - warp 0 streams the rows' Q4 bytes and scales a stage (256 K) at a time
//    with TMA into a 3-slot ring; warps 2-5 (one per TMEM lane quarter, one
//    weight row per thread) turn each 128-K half into fp16 in TMEM with the
//    stream kernel's arithmetic (one LOP3, one HSUB2, one HMUL2 per pair);
//    warp 1 issues the tcgen05 MMAs (A in TMEM, B in shared memory, N = 16)
//    into one fp32 accumulator;
//   - with the K range split over several CTAs, those CTAs form one thread
//    block cluster: each leaves its partial sums in its shared memory and
//    split 0 adds them over distributed shared memory in split order and
//    writes the output, so one launch does the whole projection and the sum
//    order is fixed.
// Two CTAs fit per SM (102 KB shared memory, 256 TMEM columns each).  Every
// mbarrier wait is bounded; on expiry the kernel sets err_flag = 2, drains
// what it issued and returns.
#include <cuda.h>

#include "common.cuh"
#include "moe_internal.h"
#include "moe_tc.h"
#include "tc_ptx.cuh"

namespace moe {
namespace tc {

namespace dn {
constexpr int BN = 16;                       // token tile (the MMA's N)
constexpr int ST_K = 256;                    // K per stage
constexpr int ST_Q = 128 * ST_K / 2;         // packed bytes per stage (16 KB)
constexpr int ST_S = 128 * (ST_K / 32) * 4;  // scale bytes per stage (4 KB)
constexpr int SQ = 3;                        // stage ring slots
constexpr int SA = 3;                        // TMEM A slots (128 K each)
constexpr int MAXS = 4;                      // stages per CTA
constexpr int B_CHUNK = BN * 128;            // one 64-K chunk of the token tile (2 KB)
constexpr int OFF_Q = 0;
constexpr int OFF_S = OFF_Q + SQ * ST_Q;
constexpr int OFF_B = OFF_S + SQ * ST_S;
constexpr int OFF_P = OFF_B + MAXS * 4 * B_CHUNK;  // this split's partial sums [token][128 rows] fp32
constexpr int OFF_BAR = OFF_P + BN * 128 * 4;
constexpr int N_BAR = 2 * SQ + 2 * SA + 2;
constexpr int OFF_MISC = OFF_BAR + N_BAR * 8;
constexpr int TOTAL = OFF_MISC + 16 + 1024;  // + alignment slack
constexpr int THREADS = 192;                 // producer, MMA issuer, four dequant / epilogue warps
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t ACOL = 32;                // A slots after the 16-column accumulator
constexpr int MAX_SPLITS = 8;                // the K splits of a row tile form one cluster (portable size)
}  // namespace dn

template <int P>
__device__ __forceinline__ uint32_t dn_pair(uint32_t w, __half2 sc) {
    const uint32_t v = (P < 2 ? w : (w >> 8));
    const uint32_t m = (P % 2 == 0) ? and_or(v, 0x000F000Fu, 0x64006400u) : and_or(v, 0x00F000F0u, 0x54005400u);
    const __half2 off = (P % 2 == 0) ? __half2(__float2half(1032.0f), __float2half(1032.0f))
                                     : __half2(__float2half(72.0f), __float2half(72.0f));
    const __half2 x = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&m), off), sc);
    return *reinterpret_cast<const uint32_t*>(&x);
}

__global__ void __launch_bounds__(dn::THREADS, 2)
    k_dense16(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap smap, DenseArgs a) {
    using namespace dn;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t bar0 = smem_u32(smem + OFF_BAR);
    auto q_full = [&](int s) { return bar0 + 8u * s; };
    auto q_empty = [&](int s) { return bar0 + 8u * (SQ + s); };
    auto a_full = [&](int s) { return bar0 + 8u * (2 * SQ + s); };
    auto a_empty = [&](int s) { return bar0 + 8u * (2 * SQ + SA + s); };
    const uint32_t acc_full = bar0 + 8u * (2 * SQ + 2 * SA);
    const uint32_t drain_bar = bar0 + 8u * (2 * SQ + 2 * SA + 1);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);
    float* part_s = reinterpret_cast<float*>(smem + OFF_P);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nst = a.K / ST_K;
    const int rt = blockIdx.x / a.ks, ksi = blockIdx.x - rt * a.ks;
    const int s0 = ksi * nst / a.ks, ns = (ksi + 1) * nst / a.ks - s0;  // 1 <= ns <= MAXS
    const int row0 = rt * 128;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SQ; ++s) {
            mbar_init(q_full(s), 1);
            mbar_init(q_empty(s), 4);
        }
        for (int s = 0; s < SA; ++s) {
            mbar_init(a_full(s), 4);
            mbar_init(a_empty(s), 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        prefetch_tmap(&qmap);
        prefetch_tmap(&smap);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();  // barrier init and TMEM allocation overlap the previous kernel
    pdl_trigger();
    Guard G{abort_flag, a.err_flag, globaltimer() + a.timeout_ns};
    const uint64_t drain_ns = a.timeout_ns > 2000000000ull ? a.timeout_ns : 2000000000ull;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer (one thread)
        if (lane == 0) {
            uint32_t armed = 0, par = 0;
            bool ok = true;
            for (int i = 0; i < ns && ok; ++i) {
                const int qs = i % SQ;
                const uint32_t qp = (uint32_t)(i / SQ) & 1u;
                if (!(ok = mbar_wait(q_empty(qs), qp ^ 1u, G))) break;
                mbar_expect_tx(q_full(qs), ST_Q + ST_S);
                tma_load_2d(smem_u32(smem + OFF_Q + qs * ST_Q), &qmap, q_full(qs), (s0 + i) * (ST_K / 2), row0);
                tma_load_2d(smem_u32(smem + OFF_S + qs * ST_S), &smap, q_full(qs), (s0 + i) * (ST_K / 32), row0);
                armed |= 1u << qs;
                par = (par & ~(1u << qs)) | (qp << qs);
            }
            Guard Gd{abort_flag, a.err_flag, globaltimer() + drain_ns};
            volatile int no_abort = 0;
            Gd.abort = &no_abort;
            for (int s = 0; s < SQ; ++s)
                if (armed & (1u << s)) mbar_wait(q_full(s), (par >> s) & 1u, Gd);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ the token tile in fp16
        // warps 1-5: [chunk][token][128 B] with the 16-byte units of a row
        // XOR-swizzled by token % 8, tokens >= M zero; each unit holds one
        // 8-group of K as [0,4,1,5,2,6,3,7]
        const int tid = threadIdx.x - 32;
        constexpr int NT = THREADS - 32;
        const int ng = ns * (ST_K / 8);  // 8-groups per token in this CTA's K range
        const int total = BN * ng;
        const int k0 = s0 * ST_K;
        // eight 8-groups per thread per pass, all loads issued before the
        // first conversion (one L2 round trip per pass, not per group)
        for (int e0 = tid; e0 < total; e0 += 8 * NT) {
            float4 u[8], v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int e = e0 + j * NT;
                const int t = e / ng, g = e - t * ng;
                if (e < total && t < a.M) {
                    const float4* x4 = reinterpret_cast<const float4*>(a.X + (int64_t)t * a.x_stride + k0 + 8 * g);
                    u[j] = __ldg(x4);
                    v[j] = __ldg(x4 + 1);
                } else {
                    u[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                    v[j] = u[j];
                }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int e = e0 + j * NT;
                if (e < total) {
                    const int t = e / ng, g = e - t * ng;
                    const __half2 h0 = __floats2half2_rn(u[j].x, v[j].x), h1 = __floats2half2_rn(u[j].y, v[j].y);
                    const __half2 h2 = __floats2half2_rn(u[j].z, v[j].z), h3 = __floats2half2_rn(u[j].w, v[j].w);
                    const uint4 o = make_uint4(
                        *reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                        *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
                    const int c = g >> 3, u8 = g & 7;  // 64-K chunk, 16-byte unit in the row
                    *reinterpret_cast<uint4*>(smem + OFF_B + c * B_CHUNK + t * 128 + ((u8 ^ (t & 7)) << 4)) = o;
                }
            }
        }
        fence_async_smem();  // the MMAs read the tile through the async proxy
        asm volatile("bar.sync 1, %0;" ::"n"(dn::THREADS - 32) : "memory");

        if (warp == 1) {
            // -------------------------------------------- MMA issuer (one thread)
            if (lane == 0) {
                constexpr uint32_t IDESC = f16_idesc(128, BN);
                bool ok = true, issued = false;
                for (int i = 0; i < ns && ok; ++i) {
                    const uint64_t bdesc = sw128_desc(smem_u32(smem + OFF_B + 4 * i * B_CHUNK));
                    for (int h = 0; h < 2; ++h) {
                        const int j = (2 * i + h) % SA;
                        const uint32_t ap = (uint32_t)((2 * i + h) / SA) & 1u;
                        if (!(ok = mbar_wait(a_full(j), ap, G))) break;
                        tc_fence_after();
                        const uint32_t ta = tmem_base + ACOL + (uint32_t)(j * 64);
                        // 16-K step k: 64-K chunk 2h + k/4 of the stage, 32 bytes per step inside a row
#pragma unroll
                        for (int k = 0; k < 8; ++k)
                            tc_mma_ts(tmem_base, ta + 8u * k,
                                      bdesc + (uint64_t)(((2 * h + k / 4) * B_CHUNK + 32 * (k % 4)) >> 4), IDESC,
                                      (i > 0 || h > 0 || k > 0) ? 1u : 0u);
                        issued = true;
                        tc_commit(a_empty(j));
                    }
                }
                if (ok) tc_commit(acc_full);
                if (issued) {  // all MMAs complete before TMEM is released
                    tc_commit(drain_bar);
                    Guard Gd{abort_flag, a.err_flag, globaltimer() + drain_ns};
                    volatile int no_abort = 0;
                    Gd.abort = &no_abort;
                    mbar_wait(drain_bar, 0, Gd);
                }
            }
            __syncwarp();
        } else {
            // -------------------------------------------- dequant, then the epilogue
            const int q = warp & 3;          // TMEM lane quarter
            const int t = q * 32 + lane;     // weight row in the tile = TMEM lane
            const int swz = t & 7;           // SWIZZLE_128B: 16-byte chunk ^= row % 8
            const uint32_t tl = tmem_base + ((uint32_t)(q * 32) << 16);
            bool ok = true;
            for (int i = 0; i < ns && ok; ++i) {
                const int qs = i % SQ;
                if (!(ok = mbar_wait_warp(q_full(qs), (uint32_t)(i / SQ) & 1u, G))) break;
                const uint8_t* qrow = smem + OFF_Q + qs * ST_Q + t * 128;
                const float4* sp = reinterpret_cast<const float4*>(smem + OFF_S + qs * ST_S + t * 32);
                const float4 sa = sp[0], sb = sp[1];
                float scl[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
                uint4 wq[8];
#pragma unroll
                for (int c = 0; c < 8; ++c) wq[c] = *reinterpret_cast<const uint4*>(qrow + ((c ^ swz) << 4));
                __syncwarp();
                if (lane == 0) mbar_arrive(q_empty(qs));
#pragma unroll 1
                for (int h = 0; h < 2; ++h) {
                    const int j = (2 * i + h) % SA;
                    const uint32_t ap = (uint32_t)((2 * i + h) / SA) & 1u;
                    if (!(ok = mbar_wait_warp1(a_empty(j), ap ^ 1u, G))) break;
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < 4; ++c) {  // chunk = Q4 block 8 (s0 + i) + 4h + c
                        const uint4 wv = wq[c];
                        const __half2 sc = __float2half2_rn(scl[c]);
                        const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
                        uint32_t hv[16];
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            hv[4 * w + 0] = dn_pair<0>(w4[w], sc);
                            hv[4 * w + 1] = dn_pair<1>(w4[w], sc);
                            hv[4 * w + 2] = dn_pair<2>(w4[w], sc);
                            hv[4 * w + 3] = dn_pair<3>(w4[w], sc);
                        }
                        asm volatile(
                            "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
                                tl + ACOL + (uint32_t)(j * 64 + 16 * c)),
                            "r"(hv[0]), "r"(hv[1]), "r"(hv[2]), "r"(hv[3]), "r"(hv[4]), "r"(hv[5]), "r"(hv[6]),
                            "r"(hv[7]), "r"(hv[8]), "r"(hv[9]), "r"(hv[10]), "r"(hv[11]), "r"(hv[12]), "r"(hv[13]),
                            "r"(hv[14]), "r"(hv[15])
                            : "memory");
                    }
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(a_full(j));
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        wq[c] = wq[c + 4];
                        scl[c] = scl[c + 4];
                    }
                }
            }
            // epilogue: this thread's weight row, the 16 token columns
            if (ok) ok = mbar_wait_warp1(acc_full, 0, G);
            float v[16];
            if (ok) {
                tc_fence_after();
                tmem_ld<16>(tl, v);
            }
            // (loops over the 16 token columns are unrolled with a guard, so
            // that v stays in registers)
            const int64_t r = row0 + t;
            if (a.ks == 1) {
                if (ok) {
#pragma unroll
                    for (int tok = 0; tok < BN; ++tok)
                        if (tok < a.M) a.out[(int64_t)tok * a.out_stride + r] = v[tok];
                }
            } else {
#pragma unroll
                for (int tok = 0; tok < BN; ++tok) part_s[tok * 128 + t] = ok ? v[tok] : 0.f;
            }
        }
    }
    if (a.ks > 1) {
        // The K splits of this row tile are the CTAs of one cluster: split 0
        // adds the others' partial sums from their shared memory in split
        // order (the same sum on every call), then every CTA waits until it
        // is done before its shared memory goes away.
        cl_sync();
        if (ksi == 0 && warp >= 2) {
            const int t = (warp & 3) * 32 + lane;
            float acc[dn::BN];
#pragma unroll
            for (int tok = 0; tok < dn::BN; ++tok) acc[tok] = 0.f;
            for (int k = 0; k < a.ks; ++k) {
                const uint32_t base = cl_map(part_s, (uint32_t)k);
                float pv[dn::BN];
#pragma unroll
                for (int tok = 0; tok < dn::BN; ++tok) pv[tok] = cl_ldf(base + (uint32_t)(tok * 128 + t) * 4u);
#pragma unroll
                for (int tok = 0; tok < dn::BN; ++tok) acc[tok] += pv[tok];
            }
            const int64_t r = row0 + t;
#pragma unroll
            for (int tok = 0; tok < dn::BN; ++tok)
                if (tok < a.M) a.out[(int64_t)tok * a.out_stride + r] = acc[tok];
        }
        cl_sync();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(dn::TMEM_COLS)
                     : "memory");
}

}  // namespace tc

bool dense16_supported(int M, int64_t K, int64_t R) {
    // at most MAX_SPLITS splits of at most MAXS stages
    return M >= 1 && M <= tc::dn::BN && K % tc::dn::ST_K == 0 && R % 128 == 0 && K / tc::dn::ST_K >= 1 &&
           K / tc::dn::ST_K <= tc::dn::MAX_SPLITS * tc::dn::MAXS;
}

int dense16_splits(int64_t K, int requested) {
    const int nst = (int)(K / tc::dn::ST_K);
    const int lo = (nst + tc::dn::MAXS - 1) / tc::dn::MAXS;  // at most MAXS stages per split
    const int hi = nst < tc::dn::MAX_SPLITS ? nst : tc::dn::MAX_SPLITS;
    int ks = requested > 0 ? requested : (nst + 2) / 3;  // default: about three stages per split
    if (ks < lo) ks = lo;
    if (ks > hi) ks = hi;
    return ks < 1 ? 1 : ks;
}

int launch_dense16(const uint8_t* Wp, const DenseArgs& a, cudaStream_t s) {
    using namespace tc;
    if (!dense16_supported(a.M, a.K, a.R) || a.ks < 1 || a.ks > a.K / dn::ST_K || a.ks > dn::MAX_SPLITS ||
        (a.K / dn::ST_K + a.ks - 1) / a.ks > dn::MAXS)
        return -1;
    if ((reinterpret_cast<uintptr_t>(Wp) & 15u) || (reinterpret_cast<uintptr_t>(a.Ws) & 15u) ||
        (reinterpret_cast<uintptr_t>(a.X) & 15u) || (a.x_stride % 4) != 0)
        return -1;
    CUtensorMap qmap, smap;
    const uint64_t kq = (uint64_t)a.K / 2, ks = (uint64_t)a.K / 32;
    if (!tc_make_map(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, Wp, kq, (uint64_t)a.R, kq, dn::ST_K / 2, 128,
                     CU_TENSOR_MAP_SWIZZLE_128B))
        return -1;
    if (!tc_make_map(&smap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.Ws, ks, (uint64_t)a.R, ks * 4, dn::ST_K / 32, 128,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
        return -1;
    if (cudaFuncSetAttribute(k_dense16, cudaFuncAttributeMaxDynamicSharedMemorySize, dn::TOTAL) != cudaSuccess)
        return -1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((a.R / 128) * a.ks));
    cfg.blockDim = dim3(dn::THREADS);
    cfg.dynamicSmemBytes = dn::TOTAL;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)a.ks;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, k_dense16, qmap, smap, a) != cudaSuccess) return -1;
    return 1;
}

}  // namespace moe
