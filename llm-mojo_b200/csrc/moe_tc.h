// moe_tc.h -- launch interface of the tcgen05 grouped Q4_0 GEMM (moe_tc.cu).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace moe {

enum TcMode { TC_PLAIN = 0, TC_ACT = 1 };

struct TcArgs {
    const float* Ws = nullptr;      // expert 0's scales [E*R][K/32] (8-byte aligned)
    int K = 0;                      // multiple of 64
    int64_t R = 0;                  // rows per expert (2F in ACT mode)
    int F = 0;                      // ACT: act rows per expert (multiple of 64)
    int act = 0;                    // activation kind
    const int* meta = nullptr;      // meta[0] = U
    const int* unique_expert = nullptr;
    const int* seg_start = nullptr;
    const int* seg_count = nullptr;
    const int* tt_prefix = nullptr; // [U+1] exclusive prefix of token tiles
    int dense_tokens = 0;           // > 0: one matrix, tokens 0..n-1
    __half* act_out = nullptr;      // ACT: [P][F] fp16, K-group order [0,4,1,5,2,6,3,7]
    float* y_out = nullptr;         // PLAIN: rows of y_stride floats
    int64_t y_stride = 0;
    const int* out_row = nullptr;   // PLAIN: output row of pair p (nullptr: p)
    int ksplit = 1;                 // PLAIN: K split into this many partial sums
    int64_t split_stride = 0;       // PLAIN: floats between the partial-sum buffers
    int exact_a = 0;                // 1: dequantise in fp32 and round once to fp16 (shared-memory A
                                    // path; the router's logits); 0: fp16 arithmetic as in TMEM
    int* err_flag = nullptr;        // set to 2 when a bounded wait expires
    uint64_t timeout_ns = 4000000000ull;
};

struct TcLaunch {
    TcArgs a;
    const uint8_t* Wp = nullptr;  // expert 0's packed rows (16-byte aligned)
    int64_t total_rows = 0;       // rows covered by the Q4 tensor map (E * R)
    const __half* B = nullptr;    // activation rows [b_rows][K] fp16 (16-byte aligned)
    int64_t b_rows = 0;
    int BN = 16;                  // token tile: 16, 32, 64, 128 or 256
    int64_t max_items = 0;        // upper bound on work items (limits the grid), 0 = none
    bool a_in_smem = false;       // force the shared-memory A operand for BN <= 64
    bool stream = false;          // BN <= 64, K % 128 == 0: the streaming kernel (moe_tc_stream.cu)
};

// Returns the number of kernels launched, or -1 when the shape or the tensor
// map is not supported (the caller then uses the CUDA-core GEMV).
int launch_tc_gemm(int mode, const TcLaunch& L, int num_sms, cudaStream_t s);
int launch_tt_prefix(const int* meta, const int* seg_count, int BN, int* tt_prefix, cudaStream_t s);
int launch_gather_f16(const float* X, int64_t K, const int* pair_row, const int* meta, int64_t rows,
                      int dense_rows, __half* out, cudaStream_t s);
bool tc_supported(int64_t K, int64_t R, int act_mode, int64_t F);

// 2-D tensor map over a row-major matrix (driver entry point; false on error)
bool tc_make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t rows,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw);
// Tensor map of any rank 1..5: dims[0] innermost; strides[i] is the byte
// stride of dimension i + 1.
bool tc_make_map_nd(CUtensorMap* m, CUtensorMapDataType dt, const void* base, int rank, const uint64_t* dims,
                    const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle sw);
// Streaming variant for token tiles of 16..64 (moe_tc_stream.cu); same
// return convention as launch_tc_gemm.
int launch_tc_stream(int mode, const TcLaunch& L, int num_sms, cudaStream_t s);
int launch_reduce_splits(const float* part, int64_t stride, int splits, float* out, int64_t n,
                         cudaStream_t s);

}  // namespace moe
