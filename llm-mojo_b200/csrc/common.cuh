// common.cuh -- shared device helpers for libmoe_b200 (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace moe {

constexpr int kWarp = 32;

// Programmatic dependent launch.  Every kernel of this library is launched
// with programmatic stream serialization (launch_k below), so it may start
// while the previous kernel on the stream is finishing: pdl_wait() blocks
// until that kernel has completed and its writes are visible, and must come
// before the first global read of data another kernel produced and before
// the first global write.  pdl_trigger() lets the next kernel be scheduled
// once every CTA of this one has started.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Thread-block cluster helpers: distributed shared memory and barriers.
__device__ __forceinline__ uint32_t cl_map(const void* p, uint32_t cta) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                 : "=r"(r)
                 : "r"((uint32_t)__cvta_generic_to_shared(p)), "r"(cta));
    return r;
}
__device__ __forceinline__ void cl_st(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ float cl_ldf(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ int cl_ldi(uint32_t addr) {
    int v;
    asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ void cl_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cl_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Streaming loads: read once, not kept in L1.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ float ldg_stream_f(const float* p) {
    float r;
    asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide reductions (blockDim.x a multiple of 32, <= 1024). `red` is
// shared scratch of >= 33 floats.  All threads receive the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    if (wid == 0) {
        float t = lane < nw ? red[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) red[32] = t;
    }
    __syncthreads();
    return red[32];
}
__device__ __forceinline__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    if (wid == 0) {
        float t = lane < nw ? red[lane] : -INFINITY;
        t = warp_max(t);
        if (lane == 0) red[32] = t;
    }
    __syncthreads();
    return red[32];
}

// Nibble k (0..7) of a 32-bit word of packed Q4_0 bytes, returned as the
// fp32 value 1 + n/16 (n = raw nibble 0..15).  The nibble is moved into
// mantissa bits 19..22 and OR-ed with the exponent of 1.0: one shift and one
// LOP3, no int->float conversion.  Because the bytes hold element 2j in the
// low and 2j+1 in the high nibble, nibble k of word w of a block is element
// 8w + k of that block, in natural order.
template <int k>
__device__ __forceinline__ float nib_1p(uint32_t w) {
    uint32_t s = (4 * k <= 19) ? (w << (19 - 4 * k)) : (w >> (4 * k - 19));
    return __uint_as_float((s & 0x00780000u) | 0x3F800000u);
}

// fp32 activation of the gated unit (moe_kernels.mojo:438-442 for kind 0).
__device__ __forceinline__ float act_fn(float g, float u, int kind) {
    if (kind == 1) {
        float t = tanhf(0.7978845608f * (g + 0.044715f * g * g * g));
        return 0.5f * g * (1.0f + t) * u;
    }
    float sig = 1.0f / (1.0f + expf(-1.702f * g));
    return (g * sig) * u;
}

// The q layout of an activation row read by the CUDA-core expert kernels
// (moe_gemv.cu): element j is stored pre-scaled by 16^-(j % 4) at float
// position 4 * xunit(j / 4) + j % 4, where xunit XOR-swizzles the eight float4
// units of each 32-element chunk by the chunk index.
__host__ __device__ __forceinline__ int xunit(int u) {
    const int c = u >> 3;
    return (c << 3) | ((u & 7) ^ (c & 7));
}
__device__ __forceinline__ int64_t qpos(int64_t j) { return 4 * xunit((int)(j >> 2)) + (j & 3); }
__device__ __forceinline__ float qscale(int64_t j) {
    return (j & 3) == 0 ? 1.f : (j & 3) == 1 ? 0.0625f : (j & 3) == 2 ? 0.00390625f : 0.000244140625f;
}

// Position of natural element j of a K-long row inside each input layout.
__device__ __forceinline__ int64_t x_src_index(int64_t j, int64_t K, int layout) {
    if (layout == 0) return j;
    const int64_t b = j >> 5, w = j & 31, i = w >> 1;
    if (layout == 1) return (w & 1) ? (K / 2 + b * 16 + i) : (b * 16 + i);
    return b * 32 + ((w & 1) ? 16 : 0) + i;  // layout 2: block32 deinterleave
}

}  // namespace moe
