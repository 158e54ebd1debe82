// moe_route.cu -- the routing chain of a small decode batch in one launch.
//
// For M <= 16 tokens the routing kernels (rms norms, the Q4_0 router GEMV,
// softmax + top-k + LOD weights, bucketing by expert, token-tile prefix,
// fp16 gather of the expert input) each do microseconds of work but pay a
// launch and a dependent global round trip each.  Here one thread-block
// cluster of C CTAs does all of it (MOE_OPT_FUSED_ROUTE; off by default:
// measured on B200 at M = 1..16 it takes 40-90 us because the fp32 router
// dot products of one 8-SM cluster are slower than the separate kernels'
// whole chain):
//   1. CTA c owns the K slice [c*d/C, (c+1)*d/C) of every token: it loads
//      the slice, and sends CTA 0 (through distributed shared memory) its
//      partial sums of squares and its partial router dot products
//      sum_k W[e][k] * router_scale[k] * x[t][k] for every expert and token;
//   2. CTA 0 adds the C partials in CTA order, forms the router logits
//      (rms_norm_noscale(x) * router_scale * r_scale_factor . W), and runs
//      softmax (+1e-10), top-k (strict >, lower index first), the LOD weights,
//      the bucketing of the (token, slot) pairs of the local expert range and
//      the token-tile prefix, exactly as the separate kernels do;
//   3. every CTA writes its K slice of moe_in = rms_norm(x, pre_norm_w), the
//      XS block sums, and the fp16 rows of the pairs in bucket order (each
//      8-element group of K in [0,4,1,5,2,6,3,7] order).
// References: model_speculative_moe_batched.mojo:857-879 (norms), :2102-2118
// and :1868 (router input), :921-953 (softmax, top-k), moe_kernels.mojo:445-490
// (LOD weights), :815-835 (bucket order).
#include "common.cuh"
#include "moe_internal.h"

namespace moe {

namespace {

constexpr int RF_THREADS = 512;
constexpr int RF_MAXB = 12;  // Q4 blocks per K slice (S <= 384)
constexpr int RF_MAXM = 16;  // tokens

}  // namespace

// Shared-memory layout (floats unless noted), same size in every CTA:
//   xs   [M][S]        this CTA's K slice of x
//   part [C][M][E]     partial router dots (used in CTA 0)
//   ssq  [C][M]        partial sums of squares (CTA 0)
//   inv  [M]           1 / rms per token (CTA 0)
//   slot_e [M*K] int, slot_w [M*K], pair_tok [M*K] int (CTA 0)
//   cnt [E] int, off [E] int (CTA 0)
__global__ void __launch_bounds__(RF_THREADS, 1) k_route_fused(RouteFusedArgs a) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ float4 sm4[];
    float* smem = reinterpret_cast<float*>(sm4);
    const int M = a.M, E = a.E, K = a.K, C = a.C, d = a.d;
    const int S = d / C, P = M * K;
    float* xs = smem;
    float* part = xs + M * S;
    float* ssq = part + C * M * E;
    float* inv = ssq + C * M;
    int* slot_e = reinterpret_cast<int*>(inv + M);
    float* slot_w = reinterpret_cast<float*>(slot_e + P);
    int* pair_tok = reinterpret_cast<int*>(slot_w + P);
    int* cnt = pair_tok + P;
    int* off = cnt + E;
    float* rsl = reinterpret_cast<float*>(off + E);  // router_scale slice [S]
    const uint32_t c = cl_rank();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarp = RF_THREADS / 32;
    const int k0 = (int)c * S;

    // every CTA of the cluster must be running before any distributed
    // shared-memory access
    cl_sync();

    // ---- 1. slice of x, partial sums of squares and router dots -> CTA 0
    for (int k = tid; k < S; k += RF_THREADS) rsl[k] = __ldg(a.rscale + k0 + k);
    for (int i = tid; i < M * S / 4; i += RF_THREADS) {
        const int t = (i * 4) / S, k = (i * 4) % S;
        reinterpret_cast<float4*>(xs)[i] = __ldg(reinterpret_cast<const float4*>(a.x + (int64_t)t * d + k0 + k));
    }
    __syncthreads();
    for (int t = warp; t < M; t += nwarp) {
        float s = 0.f;
        for (int k = lane; k < S; k += 32) s += xs[t * S + k] * xs[t * S + k];
        s = warp_sum(s);
        if (lane == 0) cl_st(cl_map(ssq + c * M + t, 0), s);
    }
    // thread (e, token group): all of router row e's blocks in this slice are
    // loaded first (independent requests in flight), then each block is
    // dequantised once and dotted with every token of the group; the 32
    // threads of a warp share the token group, so their x reads broadcast
    const int nb = S / 32, TG = RF_THREADS / 128;
    for (int e0 = 0; e0 < E; e0 += 128) {
        const int e = e0 + (tid & 127), tg = tid >> 7;
        if (e < E) {
            const uint8_t* wr = a.rp + (int64_t)e * (d / 2) + k0 / 2;
            const float* sr = a.rs + (int64_t)e * (d / 32) + k0 / 32;
            uint4 q[RF_MAXB];
            float sc[RF_MAXB];
#pragma unroll
            for (int b = 0; b < RF_MAXB; ++b) {
                if (b < nb) {
                    q[b] = __ldg(reinterpret_cast<const uint4*>(wr + b * 16));
                    sc[b] = __ldg(sr + b);
                }
            }
            float acc[RF_MAXM / 4];
#pragma unroll
            for (int j = 0; j < RF_MAXM / 4; ++j) acc[j] = 0.f;
#pragma unroll
            for (int b = 0; b < RF_MAXB; ++b) {
                if (b >= nb) break;
                const uint32_t w4[4] = {q[b].x, q[b].y, q[b].z, q[b].w};
                float wv[32];
#pragma unroll
                for (int w = 0; w < 4; ++w)
#pragma unroll
                    for (int n = 0; n < 8; ++n) {
                        // byte j of the block: element 2j low nibble, 2j+1 high nibble
                        const int kk = 8 * w + n;
                        wv[kk] = (float)((int)((w4[w] >> (4 * n)) & 15u) - 8) * sc[b] * rsl[b * 32 + kk];
                    }
#pragma unroll
                for (int j = 0; j < RF_MAXM / 4; ++j) {
                    const int t = tg + TG * j;
                    if (t < M) {
                        const float4* xp = reinterpret_cast<const float4*>(xs + t * S + b * 32);
                        float s = 0.f;
#pragma unroll
                        for (int v = 0; v < 8; ++v) {
                            const float4 x4 = xp[v];
                            s = fmaf(wv[4 * v], x4.x, s);
                            s = fmaf(wv[4 * v + 1], x4.y, s);
                            s = fmaf(wv[4 * v + 2], x4.z, s);
                            s = fmaf(wv[4 * v + 3], x4.w, s);
                        }
                        acc[j] += s;
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < RF_MAXM / 4; ++j) {
                const int t = tg + TG * j;
                if (t < M) cl_st(cl_map(part + ((int)c * M + t) * E + e, 0), acc[j]);
            }
        }
    }
    cl_sync();

    // ---- 2. CTA 0: logits, softmax, top-k, LOD, buckets, prefix
    if (c == 0) {
        for (int t = warp; t < M; t += nwarp) {
            float ss = 0.f;
            for (int cc = 0; cc < C; ++cc) ss += ssq[cc * M + t];
            const float iv = 1.0f / sqrtf(ss / (float)d + 1e-6f);
            if (lane == 0) inv[t] = iv;
            // logits for experts lane, lane + 32, ...  (E <= 256)
            float lg[8];
            float m = -INFINITY;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int e = lane + 32 * j;
                lg[j] = -INFINITY;
                if (e < E) {
                    float s = 0.f;
                    for (int cc = 0; cc < C; ++cc) s += part[(cc * M + t) * E + e];
                    lg[j] = s * iv * a.rsf + (a.bias ? a.bias[e] : 0.f);
                    m = fmaxf(m, lg[j]);
                }
            }
            m = warp_max(m);
            float se = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int e = lane + 32 * j;
                if (e < E) {
                    lg[j] = expf(lg[j] - m);
                    se += lg[j];
                }
            }
            se = warp_sum(se);
            const float den = se + 1e-10f;
            // probabilities into part[t][e] of CTA 0 (row t of slice 0 is no longer needed)
            float* pr = part + t * E;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int e = lane + 32 * j;
                if (e < E) {
                    pr[e] = lg[j] / den;
                    if (a.probs_out) a.probs_out[(int64_t)t * E + e] = pr[e];
                }
            }
            __syncwarp();
            // top-k by rank: equal values keep the lower index first
            if (lane < K) {
                slot_e[t * K + lane] = -1;
                slot_w[t * K + lane] = -999999.0f;
            }
            __syncwarp();
            for (int e = lane; e < E; e += 32) {
                const float pi = pr[e];
                if (pi != pi) continue;
                int rank = 0;
                for (int j = 0; j < E; ++j) {
                    const float pj = pr[j];
                    rank += (pj > pi) || (pj == pi && j < e);
                }
                if (rank < K) {
                    // at most one expert per rank: park it in the slot table for now
                    slot_e[t * K + rank] = e;
                    slot_w[t * K + rank] = pi;
                }
            }
            __syncwarp();
            if (lane == 0) {
                int ti[32];
                float tv[32];
                for (int k = 0; k < K; ++k) {
                    ti[k] = -1;
                    tv[k] = -999999.0f;
                }
                // ranks 0..K-1 are all filled unless there are NaNs or E < K
                for (int k = 0; k < K && k < E; ++k) {
                    ti[k] = slot_e[t * K + k];
                    tv[k] = slot_w[t * K + k];
                }
                for (int k = 0; k < K; ++k) {
                    if (a.top_idx) a.top_idx[(int64_t)t * K + k] = ti[k];
                    if (a.top_val) a.top_val[(int64_t)t * K + k] = tv[k];
                }
                float sum = 0.f;
                for (int k = 0; k < K; ++k) sum += tv[k];
                const float inv_sum = 1.0f / (sum + 1e-10f);
                const float tp = (a.top_p == a.top_p) ? a.top_p : 1.0f;
                int n = 0;
                int oi[32];
                float ow[32];
                if (tp >= 1.0f) {
                    for (int k = 0; k < K; ++k) {
                        const float np_ = tv[k] * inv_sum;
                        if ((np_ >= 0.05f || k == 0) && ti[k] >= 0) {
                            oi[n] = ti[k];
                            ow[n] = np_ * a.pes[ti[k]];
                            ++n;
                        }
                    }
                } else {
                    float cum = 0.f;
                    for (int k = 0; k < K; ++k) {
                        const float np_ = tv[k] * inv_sum;
                        if (k > 0 && (np_ < 0.05f || cum >= tp)) break;
                        if (ti[k] < 0) break;
                        oi[n] = ti[k];
                        ow[n] = np_;
                        cum += np_;
                        ++n;
                    }
                    const float rn = 1.0f / (cum + 1e-10f);
                    for (int k = 0; k < n; ++k) ow[k] = (ow[k] * rn) * a.pes[oi[k]];
                }
                for (int k = 0; k < K; ++k) {
                    const bool on = k < n;
                    slot_e[t * K + k] = on ? oi[k] : -1;
                    slot_w[t * K + k] = on ? ow[k] : 0.f;
                    a.slot_expert[t * K + k] = on ? oi[k] : -1;
                    a.slot_weight[t * K + k] = on ? ow[k] : 0.f;
                    if (a.tok_idx) a.tok_idx[(int64_t)t * K + k] = on ? oi[k] : 0;
                    if (a.tok_w) a.tok_w[(int64_t)t * K + k] = on ? ow[k] : 0.f;
                }
                if (a.tok_count) a.tok_count[t] = n;
            }
        }
        __syncthreads();
        // buckets of the local expert range: ascending expert, slot order within
        for (int e = tid; e < E; e += RF_THREADS) {
            int n = 0;
            if (e >= a.e_lo && e < a.e_hi)
                for (int p = 0; p < P; ++p) n += slot_e[p] == e;
            cnt[e] = n;
        }
        __syncthreads();
        if (warp == 0) {  // scans over E (<= 256) by one warp
            int run_p = 0, run_u = 0, run_t = 0;
            for (int e0 = 0; e0 < E; e0 += 32) {
                const int e = e0 + lane;
                const int v = e < E ? cnt[e] : 0;
                const int has = v > 0 ? 1 : 0;
                const int tt = a.BN > 0 ? (v + a.BN - 1) / a.BN : 0;
                int xp = v, xu = has, xt = tt;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int yp = __shfl_up_sync(0xffffffffu, xp, o);
                    const int yu = __shfl_up_sync(0xffffffffu, xu, o);
                    const int yt = __shfl_up_sync(0xffffffffu, xt, o);
                    if (lane >= o) {
                        xp += yp;
                        xu += yu;
                        xt += yt;
                    }
                }
                const int ep = run_p + xp - v, eu = run_u + xu - has, et = run_t + xt - tt;
                if (e < E) {
                    off[e] = ep;
                    if (has) {
                        a.b.unique_expert[eu] = e;
                        a.b.seg_start[eu] = ep;
                        a.b.seg_count[eu] = v;
                        if (a.tt_prefix) a.tt_prefix[eu] = et;
                    }
                }
                run_p += __shfl_sync(0xffffffffu, xp, 31);
                run_u += __shfl_sync(0xffffffffu, xu, 31);
                run_t += __shfl_sync(0xffffffffu, xt, 31);
            }
            if (lane == 0) {
                a.b.meta[0] = run_u;
                a.b.meta[1] = run_p;
                if (a.tt_prefix) a.tt_prefix[run_u] = run_t;
            }
        }
        __syncthreads();
        for (int e = tid; e < E; e += RF_THREADS) {
            if (cnt[e] == 0) continue;
            int pos = off[e];
            for (int p = 0; p < P; ++p)
                if (slot_e[p] == e) {
                    a.b.pair_token[pos] = p / K;
                    a.b.pair_slot[pos] = p;
                    a.b.slot_pair[p] = pos;
                    pair_tok[pos] = p / K;
                    ++pos;
                }
        }
        for (int p = tid; p < P; p += RF_THREADS) {
            const int e = slot_e[p];
            if (e < a.e_lo || e >= a.e_hi) a.b.slot_pair[p] = -1;
        }
        __syncthreads();
        if (tid == 0) {  // total local pairs, read by every CTA in step 3
            int np = 0;
            for (int e = 0; e < E; ++e) np += cnt[e];
            reinterpret_cast<int*>(ssq)[0] = np;
        }
    }
    cl_sync();

    // ---- 3. moe_in, block sums and fp16 pair rows for this K slice
    __shared__ float linv[16];
    __shared__ int lptok[512];
    __shared__ int lnp;
    if (tid < M) linv[tid] = cl_ldf(cl_map(inv + tid, 0));
    if (tid == 0) lnp = cl_ldi(cl_map(ssq, 0));
    __syncthreads();
    for (int p = tid; p < lnp; p += RF_THREADS) lptok[p] = cl_ldi(cl_map(pair_tok + p, 0));
    for (int i = tid; i < M * S; i += RF_THREADS) {
        const int t = i / S, k = i % S;
        const float o = xs[i] * linv[t] * __ldg(a.pre_w + k0 + k);
        xs[i] = o;
        if (a.x32) a.x32[(int64_t)t * d + k0 + k] = o;
    }
    __syncthreads();
    if (a.xsum) {
        for (int i = warp; i < M * nb; i += nwarp) {
            const int t = i / nb, b = i % nb;
            const float s = warp_sum(xs[t * S + b * 32 + lane]);
            if (lane == 0) a.xsum[(int64_t)t * (d / 32) + k0 / 32 + b] = 1.5f * s;
        }
    }
    if (a.x16) {
        const int ng = S / 8;
        for (int i = tid; i < lnp * ng; i += RF_THREADS) {
            const int p = i / ng, g = i % ng;
            const int t = lptok[p];
            const float* src = xs + t * S + g * 8;
            const __half2 h0 = __floats2half2_rn(src[0], src[4]);
            const __half2 h1 = __floats2half2_rn(src[1], src[5]);
            const __half2 h2 = __floats2half2_rn(src[2], src[6]);
            const __half2 h3 = __floats2half2_rn(src[3], src[7]);
            reinterpret_cast<uint4*>(a.x16 + (int64_t)p * d + k0)[g] =
                make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                           *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
        }
    }
    cl_sync();  // CTA 0's shared memory stays alive until every CTA has read it
}

size_t route_fused_smem(int M, int E, int K, int C, int d) {
    const int S = d / C, P = M * K;
    return (size_t)4 * ((size_t)M * S + (size_t)C * M * E + (size_t)C * M + M + 3 * (size_t)P + 2 * (size_t)E + S);
}

bool route_fused_supported(int M, int E, int K, int d, int* C_out) {
    if (M < 1 || M > 16 || E < 1 || E > 256 || K < 1 || K > 32 || K > E || M * K > 512) return false;
    int C = 8;
    while (C > 1 && d % (32 * C) != 0) C >>= 1;
    if (d % (32 * C) != 0 || (d / C) % 4 != 0 || d / C > 32 * 12) return false;
    if (route_fused_smem(M, E, K, C, d) > 200 * 1024) return false;
    *C_out = C;
    return true;
}

int launch_route_fused(const RouteFusedArgs& a, cudaStream_t s) {
    const size_t smem = route_fused_smem(a.M, a.E, a.K, a.C, a.d);
    if (cudaFuncSetAttribute(k_route_fused, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return -1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.C);
    cfg.blockDim = dim3(RF_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, k_route_fused, a) != cudaSuccess) return -1;
    return 1;
}

}  // namespace moe
