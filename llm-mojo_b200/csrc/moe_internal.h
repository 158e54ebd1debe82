// moe_internal.h -- launch interface between the C ABI (moe_abi.cu) and the
// kernels (moe_kernels.cu).  Internal to libmoe_b200.so.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace moe {

// NCCL communicator of a context (moe_ep.cu).  `pending`: a collective was
// enqueued and its completion has not been observed yet.
struct EpComm {
    void* comm = nullptr;
    int rank = 0, nranks = 0;
    bool pending = false;
};
int ep_unique_id(uint8_t* out, std::string& err);
// Joins the communicator; polls its set-up until `timeout_ns` (then aborts).
int ep_init(EpComm& ep, const uint8_t* id, int rank, int nranks, uint64_t timeout_ns, std::string& err);
// In-place fp32 sum over the ranks, enqueued on `s`.
int ep_all_reduce(EpComm& ep, float* buf, size_t count, cudaStream_t s, uint64_t timeout_ns, std::string& err);
// Gathers `count` elements (fp32 or int32) of every rank into `recv`, rank order.
int ep_all_gather(EpComm& ep, const void* send, void* recv, size_t count, bool is_float, cudaStream_t s,
                  uint64_t timeout_ns, std::string& err);
// Several all-gathers in one NCCL group.
struct EpGatherBuf {
    const void* send;
    void* recv;
    size_t count;   // elements per rank
    bool is_float;  // fp32, else int32
};
int ep_all_gather_n(EpComm& ep, const EpGatherBuf* bufs, int n, cudaStream_t s, uint64_t timeout_ns,
                    std::string& err);
// Sums `send` [nranks * count] over the ranks; this rank receives its `count` slice.
int ep_reduce_scatter(EpComm& ep, const float* send, float* recv, size_t count, cudaStream_t s, uint64_t timeout_ns,
                      std::string& err);
// One point-to-point transfer of a grouped exchange.
struct EpXfer {
    bool send;
    void* buf;
    size_t count;   // elements
    bool is_float;  // fp32, else int32
    int peer;
};
// All transfers in one NCCL group (an all-to-all-v when every rank lists
// one send and one receive per peer).
int ep_exchange(EpComm& ep, const std::vector<EpXfer>& xfers, cudaStream_t s, uint64_t timeout_ns, std::string& err);
// Waits for `done` (recorded after a collective), checking the communicator's
// asynchronous error; aborts the communicator on an error, and after
// `timeout_ns` when `abort_on_timeout`.
int ep_wait(EpComm& ep, cudaEvent_t done, uint64_t timeout_ns, bool abort_on_timeout, std::string& err);
void ep_abort(EpComm& ep);
void ep_destroy(EpComm& ep);

// Pinned staging buffers of the weights-file reader; a context keeps them
// between loads and releases them when it is destroyed.
struct FileStaging {
    std::vector<char*> buf;
    std::vector<cudaEvent_t> ev;
    int64_t buf_bytes = 0;
    void release();
};

// Reads [file_offset, file_offset + bytes) of `path` (bytes < 0: to the end)
// into device memory `dst` of `dst_capacity` bytes through the staging
// buffers and copies on `stream`; returns when the copies are complete.
// MOE_E_ARG (open/read failure), MOE_E_SHAPE (range past the end of the file
// or of the destination), MOE_E_NOMEM, MOE_E_CUDA; `err` gets the message.
int load_file_range(const char* path, int64_t file_offset, int64_t bytes, char* dst,
                    int64_t dst_capacity, cudaStream_t stream, FileStaging& st, std::string& err,
                    int64_t* loaded);

// Grouped Q4_0 GEMV over a device-side work list (see k_q4_gemv).
struct GemvArgs {
    const uint8_t* Wp = nullptr;  // expert 0's packed rows
    const float* Ws = nullptr;    // expert 0's scales
    int64_t rows_per_expert = 0;  // R
    int K = 0;                    // inner dimension (multiple of 32)
    const float* X = nullptr;     // input rows [*, K], fp32 natural order, 16-byte aligned
    const float* xsum = nullptr;  // [*, K/32] 1.5 * block sums of X, or null (exact dequant)
    const int* meta = nullptr;    // meta[0] = number of unique experts U
    const int* unique_expert = nullptr;
    const int* seg_start = nullptr;
    const int* seg_count = nullptr;
    const int* pair_row = nullptr;  // input row of sorted pair p (nullptr: p)
    const int* out_row = nullptr;   // output row of sorted pair p (nullptr: p)
    int dense_tokens = 0;           // > 0: one matrix (expert 0), tokens 0..n-1
    float* out = nullptr;
    int64_t out_stride = 0;
    float* gu_out = nullptr;        // optional raw gate/up values (ACT mode)
    int64_t gu_stride = 0;
    int F = 0;                      // ACT mode: act rows; gate = rows [0,F), up = [F,2F)
    int act = 0;
    int max_tokens = 1;             // upper bound on tokens per expert (host side)
    int max_unique = 1;             // upper bound on U (host side)
    int x_qlayout = 0;              // X rows in the q layout (k_dgemv; see moe_gemv.cu)
    int out_qlayout = 0;            // ACT: write the activations in the q layout
    int* err_flag = nullptr;        // k_dgemv: set to 2 when a bounded wait expires
    uint64_t timeout_ns = 0;
};

enum GemvMode { GEMV_PLAIN = 0, GEMV_ACT = 1 };

// Per-row preparation: layout/fp16 conversion, optional norms, block sums.
struct PrepArgs {
    const void* x = nullptr;
    int x_f16 = 0;
    int x_layout = 0;
    int64_t K = 0;
    int norm = 0;                   // rms-normalise (then out = x*inv*pre_w)
    const float* pre_w = nullptr;
    const float* router_scale = nullptr;
    float rsf = 0.f;
    float* out = nullptr;           // [M][K] fp32
    float* out_sum = nullptr;       // [M][K/32] 1.5 * block sums of out (nullable)
    float* scaled = nullptr;        // [M][K] x*inv*router_scale*rsf (nullable)
    float* out_q = nullptr;         // [M][K] out in the q layout (nullable; common.cuh)
};

struct TopkArgs {
    const float* scores = nullptr;  // [M][E] router logits
    const float* part = nullptr;    // or: [part_n][M][E] partial logits (k_router_part)
    float* part_out = nullptr;      // the same buffer, written by the fused grid launch
    int part_n = 0;
    int M = 0;
    float* scores_out = nullptr;    // with part: the summed logits (nullable)
    const float* bias = nullptr;
    int E = 0, K = 0;
    const float* pes = nullptr;
    float top_p = 1.f;
    int lod = 1;
    float* probs_out = nullptr;
    int64_t* top_idx = nullptr;
    float* top_val = nullptr;
    int* ti32 = nullptr;
    float* tv = nullptr;
    int* slot_expert = nullptr;
    float* slot_weight = nullptr;
    int64_t* tok_count = nullptr;
    int64_t* tok_idx = nullptr;
    float* tok_w = nullptr;
};

struct BucketOut {
    int* meta = nullptr;  // [0] U, [1] total pairs
    int* unique_expert = nullptr;
    int* seg_start = nullptr;
    int* seg_count = nullptr;
    int* pair_token = nullptr;
    int* pair_slot = nullptr;
    int* slot_pair = nullptr;
};

struct CombineArgs {
    const float* y = nullptr;  // [pairs][d]
    int64_t d = 0;
    int K = 0;
    const int* slot_pair = nullptr;
    const float* slot_weight = nullptr;
    const float* post_w = nullptr;
    int post_norm = 0;
    int fma_mode = 0;  // 1: s = fma(y, w, s) (diffusion_kernels.mojo:396); 0: s += y*w
    int ksplit = 1;             // y holds this many partial sums ...
    int64_t split_stride = 0;   // ... this many floats apart
    void* out = nullptr;
    int out_f16 = 0;
};

// Every launcher returns the number of kernels it launched.
int launch_prep(const PrepArgs& a, int64_t M, cudaStream_t s);
int launch_topk(const TopkArgs& a, int64_t M, cudaStream_t s);
int launch_gemv_f32(const float* W, const float* X, float* out, int64_t M, int64_t E, int64_t d,
                    cudaStream_t s);
int launch_set_cover(const int* ti32, const float* tv, int64_t M, int K, int E, const float* pes,
                     float top_p, float core_top_p, float singleton_min_prob, int sub_batch,
                     int* slot_expert, float* slot_weight, int64_t* tok_count, int64_t* tok_idx,
                     float* tok_w, cudaStream_t s);
int launch_slots_from_lists(int64_t M, int K, const int64_t* count, int64_t count_scalar,
                            const int64_t* idx, const float* w, int* slot_expert,
                            float* slot_weight, int E, int* err_flag, cudaStream_t s);
int launch_slots_from_topw(int64_t M, int K, const int64_t* idx, const float* w,
                           int* slot_expert, float* slot_weight, int E, int* err_flag,
                           cudaStream_t s);
// Fused routing of a small batch (moe_route.cu): norms, Q4_0 router, softmax,
// top-k, LOD weights, buckets, token-tile prefix and fp16 gather in one
// thread-block cluster of C CTAs.
struct RouteFusedArgs {
    const float* x = nullptr;        // [M][d] fp32, 16-byte aligned
    int M = 0, d = 0, E = 0, K = 0, C = 1;
    const uint8_t* rp = nullptr;     // Q4_0 router [E][d]
    const float* rs = nullptr;
    const float* rscale = nullptr;   // router_scale [d]
    float rsf = 0.f;                 // r_scale_factor
    const float* pre_w = nullptr;    // [d]
    const float* bias = nullptr;     // optional [E]
    const float* pes = nullptr;      // per_expert_scale [E]
    float top_p = 1.f;
    int e_lo = 0, e_hi = 0;          // local expert range for the buckets
    int BN = 0;                      // token tile for the prefix (0: no prefix)
    float* x32 = nullptr;            // moe_in [M][d] (nullable)
    float* xsum = nullptr;           // [M][d/32] 1.5 * block sums (nullable)
    __half* x16 = nullptr;           // [pairs][d] fp16 in bucket order (nullable)
    float* probs_out = nullptr;
    int64_t* top_idx = nullptr;
    float* top_val = nullptr;
    int* slot_expert = nullptr;
    float* slot_weight = nullptr;
    int64_t* tok_count = nullptr;
    int64_t* tok_idx = nullptr;
    float* tok_w = nullptr;
    BucketOut b;
    int* tt_prefix = nullptr;
};
bool route_fused_supported(int M, int E, int K, int d, int* C_out);

// The routing of a small batch in one launch (moe_kernels.cu): the norms,
// the K-slice router partial sums, and, in the router CTA that finishes
// last, softmax / top-k / LOD for every token and the bucketing.  The fp16
// gather of the pair rows is left to launch_gather_f16.
struct RouteRtArgs {
    PrepArgs pa;                 // norms of the M rows: x, K, pre_w, router_scale, rsf, out, out_sum, out_q
    const uint8_t* rp = nullptr; // Q4_0 router
    const float* rs = nullptr;
    TopkArgs ta;                 // part = part_out (router partial sums), part_n = d / 128
    BucketOut b;
    int e_lo = 0, e_hi = 0;      // local expert range of the buckets
    int BN = 0;                  // token tile of the tensor-core prefix (0: none)
    int* tt_prefix = nullptr;
    unsigned* ticket = nullptr;  // zero between launches (the last CTA resets it)
};
bool route_rt_supported(int M, int E, int K, int d);
int launch_route_rt(const RouteRtArgs& a, cudaStream_t s);
int launch_route_fused(const RouteFusedArgs& a, cudaStream_t s);

// Router logits of <= 16 tokens as per-K-slice partial sums (moe_kernels.cu).
bool router_part_supported(int M, int K);
int launch_router_part(const uint8_t* W, const float* S, const float* X, int M, int K, int E, float* part,
                       cudaStream_t s);

// CUDA-core grouped GEMV for few tokens per expert (moe_gemv.cu); expert
// work lists only (dense_tokens == 0).
bool dgemv_supported(const GemvArgs& a, int mode);
int launch_dgemv(int mode, const GemvArgs& a, int num_sms, cudaStream_t s);
// One-token form (every expert has at most one token): one warp per row,
// chunks streamed straight from HBM (moe_gemv.cu); same results as k_dgemv.
// One-launch Q4 projection for 1..16 tokens (moe_dense.cu): fp32 tokens in,
// fp32 out; the K range is split over `ks` CTAs per 128-row tile (one thread
// block cluster), which add their partial sums in split order.
struct DenseArgs {
    const float* Ws = nullptr;      // scales [R][K/32] (16-byte aligned)
    const float* X = nullptr;       // tokens [M][x_stride] fp32 (16-byte aligned)
    int64_t x_stride = 0;
    int M = 0;
    int K = 0;                      // multiple of 256, at most 8192
    int64_t R = 0;                  // multiple of 128
    float* out = nullptr;           // [M][out_stride]
    int64_t out_stride = 0;
    int ks = 1;                     // 1..8, at most 4 stages of 256 K per split
    int* err_flag = nullptr;
    uint64_t timeout_ns = 4000000000ull;
};
bool dense16_supported(int M, int64_t K, int64_t R);
// The split count: about three stages per CTA, or `requested` (> 0) within
// the kernel's limits.
int dense16_splits(int64_t K, int requested);
int launch_dense16(const uint8_t* Wp, const DenseArgs& a, cudaStream_t s);

bool gemv1_supported(const GemvArgs& a);
int launch_gemv1(int mode, const GemvArgs& a, int num_sms, cudaStream_t s);
// rows x K fp32 -> the q layout k_dgemv reads (pre-scaled, swizzled per row)
int launch_to_qlayout(const float* x, float* xq, int64_t rows, int K, int num_sms, cudaStream_t s);

int launch_bucket(const int* slot_expert, int64_t P, int K, int E, int e_lo, int e_hi, const BucketOut& o,
                  cudaStream_t s, int BN = 0, int* tt_prefix = nullptr);
int launch_gemv(int mode, const GemvArgs& a, int num_sms, cudaStream_t s);
int launch_gemv_wide(const uint8_t* W, const float* S, const float* X, float* out, int64_t rows, int K,
                     int ntok, int64_t out_stride, cudaStream_t s);
int launch_combine(const CombineArgs& a, int64_t M, cudaStream_t s);
int launch_quantize(const float* src, uint8_t* packed, float* scales, int64_t nblocks,
                    cudaStream_t s);
int launch_lod(int64_t B, const int64_t* top_idx, const float* top_val, const float* pes,
               float top_p, int64_t* act_idx, float* act_w, int64_t* act_count, int K,
               int64_t E, int* err_flag, cudaStream_t s);
int launch_apply_lod(const int64_t* top_idx, const float* top_val, const float* pes, float* top_w,
                     int64_t B, int K, int64_t active_top_k, const uint8_t* eb_mask,
                     const int64_t* active_canvas_idx, int64_t unaccepted_top_k, cudaStream_t s);


// Router-subspace FFN bypass of the diffusion engine (moe_subspace.cu).
struct SubspaceFilterArgs {
    const float* r_curr = nullptr;      // [B][E] router logits of this step
    float* r_prev = nullptr;            // [canvas][E] logits at each token's last evaluation
    const int64_t* top_idx = nullptr;   // [B][K]
    int64_t* prev_top2 = nullptr;       // [canvas][2]
    const uint8_t* eb_mask = nullptr;   // [canvas] accepted tokens (nullable: all)
    const int64_t* active_idx = nullptr;  // [B] canvas position of row b (nullable: b)
    int64_t* keep_out = nullptr;        // [B] evaluated rows, ascending
    float* top_w = nullptr;             // [B][K] zeroed for bypassed rows (nullable)
    int64_t* count_out = nullptr;       // number of evaluated rows
    int64_t B = 0;
    int E = 0, K = 0;
    int64_t step = 0;
    float tau = 0.05f;
};
struct SubspaceRowsArgs {
    uint8_t* out = nullptr;              // [B] rows: moe_out (sync) or ffn_full_out (scatter)
    uint8_t* cache = nullptr;            // [canvas] rows
    const uint8_t* sub = nullptr;        // scatter: [ffn_active_len] compacted rows; sync: nullptr
    const int64_t* active_idx = nullptr;  // [B] (nullable: b)
    int* map = nullptr;                  // [B] workspace: row -> matched ffn_keep_b entry or -1
    int64_t B = 0;
    int64_t row_bytes = 0;
};
int launch_subspace_filter(const SubspaceFilterArgs& a, cudaStream_t s);
int launch_subspace_rows(const SubspaceRowsArgs& a, const int64_t* keep, int64_t len, cudaStream_t s);
// One CTA waiting on an mbarrier that nothing completes, bounded by
// `timeout_ns` (the check behind moe_device_wait_check).
int launch_wait_check(int* err_flag, uint64_t timeout_ns, cudaStream_t s);

// Expert-parallel helpers (moe_kernels.cu).
// slot_expert: global expert ids -> ids local to [e_lo, e_hi) (others -1).
int launch_ep_localize(int* slot_expert, int64_t P, int e_lo, int e_hi, cudaStream_t s);
// From the buckets of a token shard (global expert ids): the destination
// rank of every sorted pair's expert (experts_per_rank apiece), the pair's
// expert id local to that rank, and the row count per destination.
int launch_ep_pack(const BucketOut& b, int experts_per_rank, int nranks, int* send_local_e, int* send_cnt,
                   cudaStream_t s);
// dst[p] = src[map[p]] for the rows p < *n_rows (device count), fp32 rows of d.
int launch_gather_rows(const float* src, const int* map, const int* n_rows, int64_t max_rows, int64_t d, float* dst,
                       cudaStream_t s);
// A slot table for rows that each carry one pair: slot_expert[i] =
// local_e[i], slot_weight[i] = 1; ids outside [0, E) raise err_flag 1.
int launch_ep_slots(const int* local_e, int64_t P, int E, int* slot_expert, float* slot_weight, int* err_flag,
                    cudaStream_t s);

}  // namespace moe
