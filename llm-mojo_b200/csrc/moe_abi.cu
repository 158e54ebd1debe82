// moe_abi.cu -- the extern "C" boundary of libmoe_b200.so (declared in
// include/moe_b200.h): contexts, weight registration, pointer translation,
// host staging and the entry points that replace the reference's Mojo
// routines.  No CPU compute path exists here: every result is produced by
// the kernels in moe_kernels.cu / moe_tc.cu.
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <cuda.h>

#include "../../include/moe_b200.h"
#include "moe_internal.h"
#include "moe_tc.h"

namespace {

struct Reg {
    const char* host;
    size_t bytes;
    char* dev;
};

struct CopyBack {
    void* host;
    const void* dev;
    size_t bytes;
};

struct Status {
    int code = MOE_OK;
    std::string msg;
};

}  // namespace

namespace {
// Internal buffers of an expert evaluation for M tokens x K slots.
constexpr int64_t kMaxSplitY = 4;  // split-K partials of the down projection kept in y
struct ExpertBufs {
    int* slot_expert;
    float* slot_weight;
    moe::BucketOut b;
    float* x32;   // [M][d] gate/up input, fp32 natural
    float* xsum;  // [M][d/32] 1.5 * block sums of x32
    float* x32q;  // [M][d]   CUDA-core path: x32 in the q layout
    bool x32q_ready;  // x32q already written (by the router's prep)
    float* act;   // [P][F]
    float* y;     // [P][d]
    __half* x16;  // [P][d]   tensor-core path: gathered gate/up input
    __half* a16;  // [P][F]   tensor-core path: activations (down input)
    int* tt_prefix;  // [E+1]
};
}  // namespace

struct moe_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = true;
    int async_mode = 0;
    std::string err;
    std::vector<Reg> regs;
    char* ws = nullptr;
    size_t ws_cap = 0;
    size_t ws_off = 0;
    size_t ws_res = 0;
    int* err_flag = nullptr;
    unsigned* route_ticket = nullptr;    // the one-launch routing's last-CTA ticket (zero between launches)
    uint64_t launches = 0;
    int num_sms = 148;
    std::vector<CopyBack> pending;
    cudaEvent_t done = nullptr;
    int gemm_path = MOE_PATH_AUTO;       // moe_set_option(MOE_OPT_GEMM_PATH)
    int tc_min_tokens = 2;               // auto: tensor cores from this many tokens (one token: CUDA-core GEMV)
    int dense_tc_min_tokens = 2;         // auto, dense projections
    int router_tc_min_tokens = 2048;     // router on tensor cores from this many tokens
    bool tc_a_in_smem = false;           // MOE_OPT_TC_A_IN_SMEM
    int tc_stream = 1;                   // MOE_OPT_TC_STREAM
    int64_t expert_begin = 0;            // MOE_OPT_EXPERT_BEGIN
    int64_t expert_end = 0;              // MOE_OPT_EXPERT_END (0: all experts)
    int fused_route = 0;                 // MOE_OPT_FUSED_ROUTE
    bool gemv1 = true;                   // MOE_OPT_GEMV_ONE_TOKEN
    bool dense16 = true;                 // MOE_OPT_DENSE_ONE_LAUNCH
    int dense_ksplit = 0;                // MOE_OPT_DENSE_KSPLIT (0: automatic)
    uint64_t device_timeout_ns = 4000000000ull;
    // profiling (moe_profile_enable)
    int profile = 0;
    std::vector<cudaEvent_t> ev_pool;
    struct ProfRec {
        int name;
        cudaEvent_t a, b;
    };
    std::vector<ProfRec> prof_pending;
    std::vector<std::string> prof_names;
    std::vector<double> prof_ms;
    std::vector<uint64_t> prof_cnt;
    moe::FileStaging file_staging;       // moe_load_weights_file's pinned buffers
    // moe_run_moe_coalesced_stage1 -> stage2: the first half's buffers live
    // in their own device arena, so that calls in between cannot overwrite them
    char* split_ws = nullptr;
    size_t split_cap = 0;
    struct Split {
        bool active = false;
        const void* key = nullptr;  // the caller's act_deint_scratch
        int64_t sub_b = 0, top_k = 0, d = 0, F = 0, E = 0, num_unique = 0;
        int act = 0;
        const uint8_t* gu_p = nullptr;
        const float* gu_s = nullptr;
        bool tc = false, stream = false;
        ExpertBufs bb;
    } split;
    moe::EpComm ep;                      // moe_ep_init's communicator
    uint64_t ep_timeout_ns = 30000000000ull;  // MOE_OPT_EP_TIMEOUT_NS
    int ep_mode = MOE_EP_REPLICATED;     // MOE_OPT_EP_MODE
    bool ep_local_weights = false;       // MOE_OPT_EP_LOCAL_WEIGHTS
    char* ep_ws = nullptr;               // all-to-all: the rows a rank receives and evaluates
    size_t ep_cap = 0;
    int* ep_host_cnt = nullptr;          // all-to-all: pinned copy of the ranks' row counts
    int ep_host_n = 0;
};

namespace {

cudaEvent_t pool_event(moe_ctx* c) {
    if (!c->ev_pool.empty()) {
        cudaEvent_t e = c->ev_pool.back();
        c->ev_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

int prof_name_id(moe_ctx* c, const char* name) {
    for (size_t i = 0; i < c->prof_names.size(); ++i)
        if (c->prof_names[i] == name) return (int)i;
    c->prof_names.push_back(name);
    c->prof_ms.push_back(0.0);
    c->prof_cnt.push_back(0);
    return (int)c->prof_names.size() - 1;
}

// Brackets the kernels launched during its lifetime with events on the
// context's stream when profiling is on.
struct ProfScope {
    moe_ctx* c;
    int id = -1;
    cudaEvent_t a = nullptr;
    ProfScope(moe_ctx* ctx, const char* name) : c(ctx) {
        if (!c->profile) return;
        id = prof_name_id(c, name);
        a = pool_event(c);
        cudaEventRecord(a, c->stream);
    }
    ~ProfScope() {
        if (id < 0) return;
        cudaEvent_t b = pool_event(c);
        cudaEventRecord(b, c->stream);
        c->prof_pending.push_back({id, a, b});
    }
};

}  // namespace

namespace {

constexpr size_t kAlign = 256;

int fail(moe_ctx* c, int code, const std::string& m) {
    if (c) c->err = m;
    return code;
}

int cuda_fail(moe_ctx* c, cudaError_t e, const char* where) {
    std::string m = std::string(where) + ": " + cudaGetErrorString(e);
    return fail(c, MOE_E_CUDA, m);
}

#define MOE_CUDA(call)                                        \
    do {                                                      \
        cudaError_t _e = (call);                              \
        if (_e != cudaSuccess) return cuda_fail(ctx, _e, #call); \
    } while (0)

// Reserve `bytes` of workspace for one call (grows only between calls).
int ws_reserve(moe_ctx* ctx, size_t bytes) {
    bytes += 64 * kAlign;
    ctx->ws_off = 0;
    ctx->ws_res = bytes;
    if (bytes <= ctx->ws_cap) return MOE_OK;
    MOE_CUDA(cudaStreamSynchronize(ctx->stream));
    if (ctx->ws) cudaFree(ctx->ws);
    ctx->ws = nullptr;
    size_t cap = std::max(bytes, ctx->ws_cap * 2);
    cudaError_t e = cudaMalloc(&ctx->ws, cap);
    if (e != cudaSuccess) {
        ctx->ws_cap = 0;
        cudaGetLastError();
        return fail(ctx, MOE_E_NOMEM, "workspace allocation failed");
    }
    ctx->ws_cap = cap;
    return MOE_OK;
}

void* ws_take(moe_ctx* ctx, size_t bytes) {
    size_t off = (ctx->ws_off + kAlign - 1) / kAlign * kAlign;
    if (off + bytes > ctx->ws_cap) return nullptr;
    ctx->ws_off = off + bytes;
    return ctx->ws + off;
}

size_t al(size_t b) { return (b + kAlign - 1) / kAlign * kAlign; }

enum Kind { K_W, K_IN, K_OUT, K_INOUT };

// Translates p into a device pointer.  Registered host ranges map to their
// HBM mirror; device/managed memory is used as is; other host memory is
// staged through the workspace (inputs copied in now, outputs copied back
// at the end of the call).  Weights must not be staged.
int dev_ptr(moe_ctx* ctx, const void* p, size_t bytes, Kind k, void** out) {
    *out = nullptr;
    if (!p) return MOE_OK;
    const char* c = static_cast<const char*>(p);
    for (const Reg& r : ctx->regs)
        if (c >= r.host && c < r.host + r.bytes) {
            if (c + bytes > r.host + r.bytes)
                return fail(ctx, MOE_E_ARG, "buffer runs past the end of its registered range");
            *out = r.dev + (c - r.host);
            return MOE_OK;
        }
    cudaPointerAttributes at;
    cudaError_t e = cudaPointerGetAttributes(&at, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        at.type = cudaMemoryTypeUnregistered;
    }
    if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) {
        *out = at.devicePointer ? at.devicePointer : const_cast<void*>(p);
        return MOE_OK;
    }
    if (k == K_W)
        return fail(ctx, MOE_E_UNREGISTERED,
                    "weight pointer is neither device memory nor inside a registered range");
    void* d = ws_take(ctx, bytes);
    if (!d) return fail(ctx, MOE_E_NOMEM, "workspace exhausted while staging a host buffer");
    if (k == K_IN || k == K_INOUT)
        MOE_CUDA(cudaMemcpyAsync(d, p, bytes, cudaMemcpyHostToDevice, ctx->stream));
    if (k == K_OUT || k == K_INOUT) ctx->pending.push_back({const_cast<void*>(p), d, bytes});
    *out = d;
    return MOE_OK;
}

#define TRY(x)                        \
    do {                              \
        int _s = (x);                 \
        if (_s != MOE_OK) return _s;  \
    } while (0)

int begin(moe_ctx* ctx) {
    if (!ctx) return MOE_E_ARG;
    ctx->err.clear();
    ctx->pending.clear();
    MOE_CUDA(cudaSetDevice(ctx->device));
    return MOE_OK;
}

// Device error word: 1 = bad expert index in a routing array, 2 = a bounded
// device-side wait expired.
int check_flag(moe_ctx* ctx) {
    int flag = 0;
    MOE_CUDA(cudaMemcpy(&flag, ctx->err_flag, sizeof(int), cudaMemcpyDeviceToHost));
    if (!flag) return MOE_OK;
    MOE_CUDA(cudaMemset(ctx->err_flag, 0, sizeof(int)));
    if (flag == 2) return fail(ctx, MOE_E_TIMEOUT, "a device-side wait exceeded its deadline");
    return fail(ctx, MOE_E_ARG, "expert index out of range in a routing array");
}

// Launch-error check, copy-back of staged outputs, optional completion.
int finish(moe_ctx* ctx) {
    MOE_CUDA(cudaGetLastError());
    for (const CopyBack& cb : ctx->pending)
        MOE_CUDA(cudaMemcpyAsync(cb.host, cb.dev, cb.bytes, cudaMemcpyDeviceToHost, ctx->stream));
    ctx->pending.clear();
    MOE_CUDA(cudaEventRecord(ctx->done, ctx->stream));
    if (!ctx->async_mode) {
        if (ctx->ep.pending) {  // a collective: bounded wait that also watches NCCL
            std::string err;
            const int st = moe::ep_wait(ctx->ep, ctx->done, ctx->ep_timeout_ns, true, err);
            if (st != MOE_OK) return fail(ctx, st, err);
        } else {
            MOE_CUDA(cudaEventSynchronize(ctx->done));
        }
        return check_flag(ctx);
    }
    return MOE_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
bool al8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; }

int check_q4_shape(moe_ctx* ctx, int64_t K, int64_t rows) {
    if (K <= 0 || K % 32 != 0) return fail(ctx, MOE_E_SHAPE, "inner dimension must be a positive multiple of 32");
    if (rows <= 0) return fail(ctx, MOE_E_SHAPE, "row count must be positive");
    if (K > (1 << 20)) return fail(ctx, MOE_E_SHAPE, "inner dimension too large");
    return MOE_OK;
}


size_t expert_bufs_bytes(int64_t M, int64_t K, int64_t d, int64_t F, int64_t E) {
    const int64_t P = M * K;
    return al(P * 4) * 2 + al(16) + al(E * 4) * 3 + al(P * 4) * 3 + al(M * d * 4) +
           al(M * d / 32 * 4) + al(M * d * 4) + al(P * F * 4) + al(P * d * 4 * kMaxSplitY) + al(P * d * 2) +
           al(P * F * 2) + al((E + 1) * 4);
}

// Carves the buffers of one expert evaluation out of an arena; `take`
// returns nullptr once the arena is exhausted (every later take does too).
template <class Take>
bool carve_expert_bufs(Take take, int64_t M, int64_t K, int64_t d, int64_t F, int64_t E, ExpertBufs* o) {
    const int64_t P = M * K;
    o->slot_expert = (int*)take(P * 4);
    o->slot_weight = (float*)take(P * 4);
    o->b.meta = (int*)take(16);
    o->b.unique_expert = (int*)take(E * 4);
    o->b.seg_start = (int*)take(E * 4);
    o->b.seg_count = (int*)take(E * 4);
    o->b.pair_token = (int*)take(P * 4);
    o->b.pair_slot = (int*)take(P * 4);
    o->b.slot_pair = (int*)take(P * 4);
    o->x32 = (float*)take(M * d * 4);
    o->xsum = (float*)take(M * d / 32 * 4);
    o->x32q = (float*)take(M * d * 4);
    o->x32q_ready = false;
    o->act = (float*)take(P * F * 4);
    o->y = (float*)take(P * d * 4 * kMaxSplitY);
    o->x16 = (__half*)take(P * d * 2);
    o->a16 = (__half*)take(P * F * 2);
    o->tt_prefix = (int*)take((E + 1) * 4);
    return o->tt_prefix != nullptr;
}

int take_expert_bufs(moe_ctx* ctx, int64_t M, int64_t K, int64_t d, int64_t F, int64_t E,
                     ExpertBufs* o) {
    if (!carve_expert_bufs([&](size_t b) { return ws_take(ctx, b); }, M, K, d, F, E, o))
        return fail(ctx, MOE_E_NOMEM, "workspace exhausted");
    return MOE_OK;
}

struct ExpertWeights {
    const uint8_t* gu_p;
    const float* gu_s;
    const uint8_t* dn_p;
    const float* dn_s;
};

// Rows of an input (any layout, fp32 or fp16) -> fp32 natural + block sums.
int prep_rows(moe_ctx* ctx, const void* X, int x_layout, int x_f16, int64_t M, int64_t K,
              float* out, float* out_sum) {
    moe::PrepArgs pa;
    pa.x = X;
    pa.x_f16 = x_f16;
    pa.x_layout = x_layout;
    pa.K = K;
    pa.out = out;
    pa.out_sum = out_sum;
    ProfScope ps(ctx, "prep");
    ctx->launches += moe::launch_prep(pa, M, ctx->stream);
    return MOE_OK;
}

// Split-K factor for a PLAIN tensor-core GEMM with `items` work items: enough
// items to give every SM two, at least 4 k-tiles per split.
int choose_ksplit(moe_ctx* ctx, int64_t items, int64_t K) {
    const int64_t nk = K / 64, target = 2LL * ctx->num_sms;
    if (items <= 0 || items >= target) return 1;
    int64_t ks = (target + items - 1) / items;
    const int64_t cap = std::max<int64_t>(1, nk / 4);
    return (int)std::min(ks, cap);
}

// Tensor cores for the expert GEMMs: forced by the option, or (auto) from
// tc_min_tokens tokens on, when shapes and alignments allow.
bool use_tc(moe_ctx* ctx, int64_t M, int64_t d, int64_t F, const ExpertWeights& w) {
    if (ctx->gemm_path == MOE_PATH_GEMV) return false;
    if (!moe::tc_supported(d, 2 * F, 1, F) || !moe::tc_supported(F, d, 0, F)) return false;
    if (!al16(w.gu_p) || !al16(w.dn_p) || !al8(w.gu_s) || !al8(w.dn_s)) return false;
    if (ctx->gemm_path == MOE_PATH_TC) return true;
    return M >= ctx->tc_min_tokens;
}

// Local expert range [lo, hi) of the context (expert parallelism).
void expert_range(moe_ctx* ctx, int64_t E, int* lo, int* hi) {
    *lo = (int)std::min<int64_t>(ctx->expert_begin, E);
    *hi = ctx->expert_end > 0 ? (int)std::min<int64_t>(ctx->expert_end, E) : (int)E;
}

// Token tile of the expert GEMMs from the mean load of an active expert.
int expert_token_tile(int64_t P, int64_t E) {
    const int64_t max_u = std::min<int64_t>(E, P);
    const int64_t mean = (P + max_u - 1) / max_u;
    int BN = 16;
    while (BN < 256 && BN < mean) BN *= 2;
    return BN;
}

// slot table -> bucket -> gate/up (+act) -> down -> combine.  bb.x32 and
// bb.xsum must hold the gate/up input (prep_rows or the router's prep).
// `prebucketed`: the fused routing kernel already wrote the buckets, the
// token-tile prefix and (tensor-core path) the fp16 pair rows.
// Launch descriptors of one expert evaluation (gate/up + activation, then
// down), fixed before anything is launched so that the two halves can run
// as separate calls (moe_run_moe_coalesced_stage1/2) with the very kernels
// and arguments of the one-call form.
struct ExpertPlan {
    bool tc = false;
    moe::TcLaunch t1, t2;          // tensor-core path
    moe::GemvArgs g1, g2;          // CUDA-core path (q-layout forms when `stream`)
    bool stream = false;           // CUDA-core: the k_dgemv pair
    bool one = false;              // CUDA-core, one token per expert: the k_gemv1 pair
    int ksplit = 1;
    int BN = 0;
};

void plan_experts(moe_ctx* ctx, const ExpertWeights& w, int64_t M, int64_t K, int64_t d, int64_t F,
                  int64_t E, int act, const ExpertBufs& bb, ExpertPlan* p) {
    const int64_t P = M * K;
    p->tc = use_tc(ctx, M, d, F, w);
    const int max_u = (int)std::min<int64_t>(E, P);
    const int max_t = (int)std::max<int64_t>(1, M);
    if (p->tc) {
        const int BN = expert_token_tile(P, E);
        p->BN = BN;
        moe::TcLaunch& t1 = p->t1;
        t1.a.Ws = w.gu_s;
        t1.a.K = (int)d;
        t1.a.R = 2 * F;
        t1.a.F = (int)F;
        t1.a.act = act;
        t1.a.meta = bb.b.meta;
        t1.a.unique_expert = bb.b.unique_expert;
        t1.a.seg_start = bb.b.seg_start;
        t1.a.seg_count = bb.b.seg_count;
        t1.a.tt_prefix = bb.tt_prefix;
        t1.a.act_out = bb.a16;
        t1.a.err_flag = ctx->err_flag;
        t1.a.timeout_ns = ctx->device_timeout_ns;
        t1.Wp = w.gu_p;
        t1.total_rows = E * 2 * F;
        t1.B = bb.x16;
        t1.b_rows = P;
        t1.BN = BN;
        t1.max_items = (int64_t)(F / 64) * (max_u + (P + BN - 1) / BN);
        t1.a_in_smem = ctx->tc_a_in_smem;
        t1.stream = ctx->tc_stream >= 1;
        moe::TcLaunch& t2 = p->t2;
        t2 = t1;
        t2.a.Ws = w.dn_s;
        t2.a.K = (int)F;
        t2.a.R = d;
        t2.a.act_out = nullptr;
        t2.a.y_out = bb.y;
        t2.a.y_stride = d;
        t2.Wp = w.dn_p;
        t2.total_rows = E * d;
        t2.B = bb.a16;
        t2.max_items = ((d + 127) / 128) * (max_u + (P + BN - 1) / BN);
        t2.a.ksplit = (int)std::min<int64_t>(choose_ksplit(ctx, ((d + 127) / 128) * max_u, F), kMaxSplitY);
        t2.a.split_stride = P * d;
        t2.max_items *= t2.a.ksplit;
        p->ksplit = t2.a.ksplit;
        return;
    }
    moe::GemvArgs g1;
    g1.Wp = w.gu_p;
    g1.Ws = w.gu_s;
    g1.rows_per_expert = 2 * F;
    g1.K = (int)d;
    g1.X = bb.x32;
    g1.xsum = bb.xsum;
    g1.meta = bb.b.meta;
    g1.unique_expert = bb.b.unique_expert;
    g1.seg_start = bb.b.seg_start;
    g1.seg_count = bb.b.seg_count;
    g1.pair_row = bb.b.pair_token;
    g1.out = bb.act;
    g1.out_stride = F;
    g1.F = (int)F;
    g1.act = act;
    g1.max_tokens = max_t;
    g1.max_unique = max_u;
    g1.err_flag = ctx->err_flag;
    g1.timeout_ns = ctx->device_timeout_ns;

    moe::GemvArgs g2 = g1;
    g2.Wp = w.dn_p;
    g2.Ws = w.dn_s;
    g2.rows_per_expert = d;
    g2.K = (int)F;
    g2.X = bb.act;
    g2.xsum = nullptr;
    g2.pair_row = nullptr;
    g2.out = bb.y;
    g2.out_stride = d;

    // The streaming kernel pair (k_dgemv) reads its inputs in the q layout:
    // the gate/up input is converted once, the activations come out of stage
    // 1 in it.  Both stages take it or neither does.
    moe::GemvArgs q1 = g1, q2 = g2;
    q1.X = bb.x32q;
    q1.x_qlayout = 1;
    q1.out_qlayout = 1;
    q2.x_qlayout = 1;
    p->stream = moe::dgemv_supported(q1, moe::GEMV_ACT) && moe::dgemv_supported(q2, moe::GEMV_PLAIN);
    // one token per expert (a one-token batch): one warp per row, no ring
    p->one = ctx->gemv1 && p->stream && moe::gemv1_supported(q1) && moe::gemv1_supported(q2);
    p->g1 = p->stream ? q1 : g1;
    p->g2 = p->stream ? q2 : g2;
}

// Gate/up + activation: bucket the pairs (unless the caller's routing launch
// did), gather the fp16 rows, run the first GEMM.
int experts_stage1(moe_ctx* ctx, const ExpertPlan& p, ExpertBufs& bb, int64_t M, int64_t K, int64_t d,
                   int64_t E, bool prebucketed) {
    cudaStream_t s = ctx->stream;
    const int64_t P = M * K;
    if (!prebucketed) {  // the tensor-core path's token-tile prefix comes out of the same launch
        ProfScope ps(ctx, "bucket");
        int e_lo, e_hi;
        expert_range(ctx, E, &e_lo, &e_hi);
        ctx->launches += moe::launch_bucket(bb.slot_expert, P, (int)K, (int)E, e_lo, e_hi, bb.b, s,
                                            p.tc ? p.BN : 0, p.tc ? bb.tt_prefix : nullptr);
    }
    if (p.tc) {
        if (!prebucketed) {
            ProfScope ps(ctx, "gather");
            ctx->launches += moe::launch_gather_f16(bb.x32, d, bb.b.pair_token, bb.b.meta, P, 0, bb.x16, s);
        }
        int r;
        {
            ProfScope ps(ctx, "tc_gate_up");
            r = moe::launch_tc_gemm(moe::TC_ACT, p.t1, ctx->num_sms, s);
        }
        if (r < 0) return fail(ctx, MOE_E_CUDA, "tensor-core GEMM setup failed (gate/up)");
        ctx->launches += r;
        return MOE_OK;
    }
    if (p.stream && !bb.x32q_ready) {
        ProfScope ps(ctx, "qlayout");
        ctx->launches += moe::launch_to_qlayout(bb.x32, bb.x32q, M, (int)d, ctx->num_sms, s);
    }
    ProfScope ps(ctx, "gemv_gate_up");
    const int r = p.one      ? moe::launch_gemv1(moe::GEMV_ACT, p.g1, ctx->num_sms, s)
                  : p.stream ? moe::launch_dgemv(moe::GEMV_ACT, p.g1, ctx->num_sms, s)
                             : moe::launch_gemv(moe::GEMV_ACT, p.g1, ctx->num_sms, s);
    if (r < 0) return fail(ctx, MOE_E_CUDA, "expert GEMV launch failed (gate/up)");
    ctx->launches += r;
    return MOE_OK;
}

// Down GEMM, then the per-token weighted combine into `out`.
int experts_stage2(moe_ctx* ctx, const ExpertPlan& p, ExpertBufs& bb, int64_t M, int64_t K, int64_t d,
                   const moe::CombineArgs* comb_tmpl, void* out) {
    cudaStream_t s = ctx->stream;
    const int64_t P = M * K;
    if (p.tc) {
        int r;
        {
            ProfScope ps(ctx, "tc_down");
            r = moe::launch_tc_gemm(moe::TC_PLAIN, p.t2, ctx->num_sms, s);
        }
        if (r < 0) return fail(ctx, MOE_E_CUDA, "tensor-core GEMM setup failed (down)");
        ctx->launches += r;
    } else {
        ProfScope ps(ctx, "gemv_down");
        const int r = p.one      ? moe::launch_gemv1(moe::GEMV_PLAIN, p.g2, ctx->num_sms, s)
                      : p.stream ? moe::launch_dgemv(moe::GEMV_PLAIN, p.g2, ctx->num_sms, s)
                                 : moe::launch_gemv(moe::GEMV_PLAIN, p.g2, ctx->num_sms, s);
        if (r < 0) return fail(ctx, MOE_E_CUDA, "expert GEMV launch failed (down)");
        ctx->launches += r;
    }
    moe::CombineArgs c = *comb_tmpl;
    c.ksplit = p.ksplit;
    c.split_stride = P * d;
    c.y = bb.y;
    c.d = d;
    c.K = (int)K;
    c.slot_pair = bb.b.slot_pair;
    c.slot_weight = bb.slot_weight;
    c.out = out;
    {
        ProfScope ps(ctx, "combine");
        ctx->launches += moe::launch_combine(c, M, s);
    }
    return MOE_OK;
}

int run_experts(moe_ctx* ctx, const ExpertWeights& w, int64_t M, int64_t K, int64_t d, int64_t F,
                int64_t E, int act, ExpertBufs& bb, const moe::CombineArgs* comb_tmpl, void* out,
                bool prebucketed = false) {
    ExpertPlan p;
    plan_experts(ctx, w, M, K, d, F, E, act, bb, &p);
    TRY(experts_stage1(ctx, p, bb, M, K, d, E, prebucketed));
    return experts_stage2(ctx, p, bb, M, K, d, comb_tmpl, out);
}

// Workspace dense_q4 may take (fp16 copy of x and split-K partials).
size_t dense_bytes(int64_t batch, int64_t c_in, int64_t c_out) {
    return al(batch * c_in * 2) + al(batch * c_out * 4 * (c_in / 256 + 1));
}

// The one-launch projection (moe_dense.cu) for 1..16 tokens.
bool dense_one_launch_ok(moe_ctx* ctx, const void* w, const void* sc, const void* xd, int64_t c_in, int64_t c_out,
                         int64_t batch) {
    return ctx->dense16 && moe::dense16_supported((int)std::min<int64_t>(batch, 1 << 20), c_in, c_out) &&
           al16(w) && al16(sc) && al16(xd);
}
int dense_one_launch(moe_ctx* ctx, const void* w, const void* sc, const void* xd, void* od, int64_t c_in,
                     int64_t c_out, int64_t batch) {
    moe::DenseArgs da;
    da.Ws = (const float*)sc;
    da.X = (const float*)xd;
    da.x_stride = c_in;
    da.M = (int)batch;
    da.K = (int)c_in;
    da.R = c_out;
    da.out = (float*)od;
    da.out_stride = c_out;
    da.ks = moe::dense16_splits(c_in, ctx->dense_ksplit);
    da.err_flag = ctx->err_flag;
    da.timeout_ns = ctx->device_timeout_ns;
    const int r = moe::launch_dense16((const uint8_t*)w, da, ctx->stream);
    if (r < 0) return fail(ctx, MOE_E_CUDA, "tensor-core projection launch failed");
    ctx->launches += r;
    return MOE_OK;
}

// out[batch][c_out] = W[c_out][c_in] . x[batch][c_in]^T on device buffers
// (x fp32, 16-byte aligned).  Tensor cores (split-K, deterministic reduce)
// from dense_tc_min_tokens tokens on, else the token-chunked fp32 GEMV.
int dense_q4(moe_ctx* ctx, const uint8_t* w, const float* sc, const float* xd, float* od, int64_t c_in,
             int64_t c_out, int64_t batch, const char* prof_name, bool exact_a = false) {
    const bool tc = ctx->gemm_path != MOE_PATH_GEMV && moe::tc_supported(c_in, c_out, 0, 0) &&
                    al8(sc) && (ctx->gemm_path == MOE_PATH_TC || batch >= ctx->dense_tc_min_tokens);
    if (tc && !exact_a && dense_one_launch_ok(ctx, w, sc, xd, c_in, c_out, batch)) {
        // 1..16 tokens: one launch (fp16 conversion and split-K sums inside)
        ProfScope ps(ctx, prof_name);
        return dense_one_launch(ctx, w, sc, xd, od, c_in, c_out, batch);
    }
    if (tc) {
        __half* x16 = (__half*)ws_take(ctx, batch * c_in * 2);
        if (!x16) return fail(ctx, MOE_E_NOMEM, "workspace exhausted");
        moe::TcLaunch t;
        t.a.Ws = sc;
        t.a.K = (int)c_in;
        t.a.R = c_out;
        t.a.dense_tokens = (int)batch;
        t.a.y_out = od;
        t.a.y_stride = c_out;
        t.a.exact_a = exact_a ? 1 : 0;
        t.a.err_flag = ctx->err_flag;
        t.a.timeout_ns = ctx->device_timeout_ns;
        t.Wp = w;
        t.total_rows = c_out;
        t.B = x16;
        t.b_rows = batch;
        int BN = 16;
        while (BN < 256 && BN < batch) BN *= 2;
        t.BN = BN;
        t.max_items = ((c_out + 127) / 128) * ((batch + BN - 1) / BN);
        t.a_in_smem = ctx->tc_a_in_smem;
        t.stream = ctx->tc_stream >= 2;
        const int ks = ctx->dense_ksplit > 0 ? (int)std::min<int64_t>(ctx->dense_ksplit, std::max<int64_t>(1, c_in / 256))
                                             : choose_ksplit(ctx, t.max_items, c_in);
        float* part = nullptr;
        if (ks > 1) {
            part = (float*)ws_take(ctx, (size_t)ks * batch * c_out * 4);
            if (!part) return fail(ctx, MOE_E_NOMEM, "workspace exhausted");
            t.a.y_out = part;
            t.a.ksplit = ks;
            t.a.split_stride = batch * c_out;
            t.max_items *= ks;
        }
        ProfScope ps(ctx, prof_name);
        ctx->launches += moe::launch_gather_f16(xd, c_in, nullptr, nullptr, batch, (int)batch, x16, ctx->stream);
        const int r = moe::launch_tc_gemm(moe::TC_PLAIN, t, ctx->num_sms, ctx->stream);
        if (r < 0) return fail(ctx, MOE_E_CUDA, "tensor-core GEMM setup failed");
        ctx->launches += r;
        if (ks > 1)
            ctx->launches += moe::launch_reduce_splits(part, batch * c_out, ks, od, batch * c_out, ctx->stream);
        return MOE_OK;
    }
    ProfScope ps(ctx, prof_name);
    ctx->launches += moe::launch_gemv_wide(w, sc, xd, od, c_out, (int)c_in, (int)batch, c_out, ctx->stream);
    return MOE_OK;
}

// Device address of moe_q4_matmul_batchN_noalloc's static scratch on the
// context's device (defined with the entry point at the end of this file).
int noalloc_scratch(moe_ctx* ctx, void** out);

}  // namespace

// ======================================================================
extern "C" {

int moe_ctx_create(int device, moe_ctx** out) {
    if (!out) return MOE_E_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return MOE_E_CUDA;
    }
    if (device < 0 || device >= n) return MOE_E_ARG;
    moe_ctx* ctx = new moe_ctx();
    ctx->device = device;
    if (cudaSetDevice(device) != cudaSuccess ||
        cudaStreamCreateWithFlags(&ctx->stream, cudaStreamDefault) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->done, cudaEventDisableTiming) != cudaSuccess ||
        cudaMalloc(&ctx->err_flag, sizeof(int)) != cudaSuccess ||
        cudaMemset(ctx->err_flag, 0, sizeof(int)) != cudaSuccess ||
        cudaMalloc(&ctx->route_ticket, sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(ctx->route_ticket, 0, sizeof(unsigned)) != cudaSuccess) {
        cudaGetLastError();
        delete ctx;
        return MOE_E_CUDA;
    }
    cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
    // The no-alloc entry point's static scratch belongs to this file's device
    // module, which has no kernel.  Under lazy module loading (the CUDA 12
    // default) that module, and with it the 8 MiB array, is loaded the first
    // time the array's address is looked up.  Looking it up here commits the
    // memory when the first context on a device is created, so that no
    // moe_q4_matmul_batchN_noalloc call ever triggers the load.
    void* scratch = nullptr;
    if (noalloc_scratch(ctx, &scratch) != MOE_OK) {
        moe_ctx_destroy(ctx);
        return MOE_E_NOMEM;
    }
    *out = ctx;
    return MOE_OK;
}

int moe_ctx_destroy(moe_ctx* ctx) {
    if (!ctx) return MOE_E_ARG;
    cudaSetDevice(ctx->device);
    if (ctx->ep.comm) {  // complete (or abort) collectives before the stream wait below
        std::string err;
        cudaEventRecord(ctx->done, ctx->stream);
        if (moe::ep_wait(ctx->ep, ctx->done, ctx->ep_timeout_ns, true, err) == MOE_OK) moe::ep_destroy(ctx->ep);
    }
    cudaStreamSynchronize(ctx->stream);
    for (Reg& r : ctx->regs) cudaFree(r.dev);
    if (ctx->ws) cudaFree(ctx->ws);
    if (ctx->split_ws) cudaFree(ctx->split_ws);
    if (ctx->ep_ws) cudaFree(ctx->ep_ws);
    if (ctx->ep_host_cnt) cudaFreeHost(ctx->ep_host_cnt);
    if (ctx->err_flag) cudaFree(ctx->err_flag);
    if (ctx->route_ticket) cudaFree(ctx->route_ticket);
    if (ctx->done) cudaEventDestroy(ctx->done);
    for (auto& r : ctx->prof_pending) {
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    for (cudaEvent_t e : ctx->ev_pool) cudaEventDestroy(e);
    ctx->file_staging.release();
    if (ctx->own_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
    return MOE_OK;
}

const char* moe_last_error(const moe_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

uint64_t moe_kernel_launches(const moe_ctx* ctx) { return ctx ? ctx->launches : 0; }

int moe_set_stream(moe_ctx* ctx, void* stream) {
    if (!ctx) return MOE_E_ARG;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->own_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
    if (stream) {
        ctx->stream = static_cast<cudaStream_t>(stream);
        ctx->own_stream = false;
    } else {
        if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamDefault) != cudaSuccess)
            return fail(ctx, MOE_E_CUDA, "stream creation failed");
        ctx->own_stream = true;
    }
    return MOE_OK;
}

int moe_set_async(moe_ctx* ctx, int async_mode) {
    if (!ctx) return MOE_E_ARG;
    ctx->async_mode = async_mode ? 1 : 0;
    return MOE_OK;
}

int moe_wait(moe_ctx* ctx, uint64_t timeout_ns) {
    if (!ctx) return MOE_E_ARG;
    cudaSetDevice(ctx->device);
    if (ctx->ep.pending) {
        // enqueued collectives: the caller's deadline (or, without one, the
        // communicator's), watching NCCL's asynchronous error meanwhile; only
        // the communicator's own deadline aborts it
        const bool own = timeout_ns == 0 || timeout_ns >= ctx->ep_timeout_ns;
        std::string err;
        const int st = moe::ep_wait(ctx->ep, ctx->done, own ? ctx->ep_timeout_ns : timeout_ns, own, err);
        if (st != MOE_OK) return fail(ctx, st, err);
        return check_flag(ctx);
    }
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t e = cudaEventQuery(ctx->done);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) return cuda_fail(ctx, e, "moe_wait");
        if (timeout_ns) {
            const auto dt = std::chrono::duration_cast<std::chrono::nanoseconds>(
                                std::chrono::steady_clock::now() - t0)
                                .count();
            if ((uint64_t)dt > timeout_ns) return fail(ctx, MOE_E_TIMEOUT, "moe_wait: deadline expired");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    return check_flag(ctx);
}

int moe_set_option(moe_ctx* ctx, int option, int64_t value) {
    if (!ctx) return MOE_E_ARG;
    switch (option) {
        case MOE_OPT_EP_MODE:
            if (value < MOE_EP_REPLICATED || value > MOE_EP_ALL_TO_ALL) return fail(ctx, MOE_E_ARG, "bad EP mode");
            ctx->ep_mode = (int)value;
            return MOE_OK;
        case MOE_OPT_DENSE_ONE_LAUNCH:
            if (value != 0 && value != 1) return fail(ctx, MOE_E_ARG, "MOE_OPT_DENSE_ONE_LAUNCH is 0 or 1");
            ctx->dense16 = value != 0;
            return MOE_OK;
        case MOE_OPT_GEMV_ONE_TOKEN:
            ctx->gemv1 = value != 0;
            return MOE_OK;
        case MOE_OPT_EP_LOCAL_WEIGHTS:
            ctx->ep_local_weights = value != 0;
            return MOE_OK;
        case MOE_OPT_GEMM_PATH:
            if (value < MOE_PATH_AUTO || value > MOE_PATH_TC) return fail(ctx, MOE_E_ARG, "bad path");
            ctx->gemm_path = (int)value;
            return MOE_OK;
        case MOE_OPT_TC_MIN_TOKENS:
            if (value < 1) return fail(ctx, MOE_E_ARG, "bad token threshold");
            ctx->tc_min_tokens = (int)value;
            return MOE_OK;
        case MOE_OPT_DEVICE_TIMEOUT_NS:
            if (value <= 0) return fail(ctx, MOE_E_ARG, "bad timeout");
            ctx->device_timeout_ns = (uint64_t)value;
            return MOE_OK;
        case MOE_OPT_DENSE_TC_MIN_TOKENS:
            if (value < 1) return fail(ctx, MOE_E_ARG, "bad token threshold");
            ctx->dense_tc_min_tokens = (int)value;
            return MOE_OK;
        case MOE_OPT_TC_A_IN_SMEM:
            ctx->tc_a_in_smem = value != 0;
            return MOE_OK;
        case MOE_OPT_TC_STREAM:
            if (value < 0 || value > 2) return fail(ctx, MOE_E_ARG, "MOE_OPT_TC_STREAM is 0, 1 or 2");
            ctx->tc_stream = (int)value;
            return MOE_OK;
        case MOE_OPT_EXPERT_BEGIN:
            if (value < 0) return fail(ctx, MOE_E_ARG, "bad expert index");
            ctx->expert_begin = value;
            return MOE_OK;
        case MOE_OPT_EXPERT_END:
            if (value < 0) return fail(ctx, MOE_E_ARG, "bad expert index");
            ctx->expert_end = value;
            return MOE_OK;
        case MOE_OPT_EP_TIMEOUT_NS:
            if (value <= 0) return fail(ctx, MOE_E_ARG, "bad timeout");
            ctx->ep_timeout_ns = (uint64_t)value;
            return MOE_OK;
        case MOE_OPT_FUSED_ROUTE:
            if (value < 0 || value > 2) return fail(ctx, MOE_E_ARG, "bad fused-routing mode");
            ctx->fused_route = (int)value;
            return MOE_OK;
        case MOE_OPT_DENSE_KSPLIT:
            if (value < 0 || value > 64) return fail(ctx, MOE_E_ARG, "MOE_OPT_DENSE_KSPLIT is 0..64");
            ctx->dense_ksplit = (int)value;
            return MOE_OK;
        case MOE_OPT_ROUTER_TC_MIN_TOKENS:
            if (value < 1) return fail(ctx, MOE_E_ARG, "bad token threshold");
            ctx->router_tc_min_tokens = (int)value;
            return MOE_OK;
        default:
            return fail(ctx, MOE_E_ARG, "unknown option");
    }
}

int moe_profile_enable(moe_ctx* ctx, int on) {
    if (!ctx) return MOE_E_ARG;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    for (auto& r : ctx->prof_pending) {
        ctx->ev_pool.push_back(r.a);
        ctx->ev_pool.push_back(r.b);
    }
    ctx->prof_pending.clear();
    ctx->prof_names.clear();
    ctx->prof_ms.clear();
    ctx->prof_cnt.clear();
    ctx->profile = on ? 1 : 0;
    return MOE_OK;
}

int moe_profile_read(moe_ctx* ctx, int n_max, char* names, double* total_ms, uint64_t* counts,
                     int* n_out) {
    if (!ctx || !n_out) return MOE_E_ARG;
    cudaSetDevice(ctx->device);
    MOE_CUDA(cudaStreamSynchronize(ctx->stream));
    for (auto& r : ctx->prof_pending) {
        float ms = 0.f;
        MOE_CUDA(cudaEventElapsedTime(&ms, r.a, r.b));
        ctx->prof_ms[r.name] += ms;
        ctx->prof_cnt[r.name] += 1;
        ctx->ev_pool.push_back(r.a);
        ctx->ev_pool.push_back(r.b);
    }
    ctx->prof_pending.clear();
    const int n = (int)ctx->prof_names.size();
    *n_out = n;
    for (int i = 0; i < n && i < n_max; ++i) {
        if (names) {
            std::strncpy(names + 32 * i, ctx->prof_names[i].c_str(), 31);
            names[32 * i + 31] = 0;
        }
        if (total_ms) total_ms[i] = ctx->prof_ms[i];
        if (counts) counts[i] = ctx->prof_cnt[i];
    }
    return MOE_OK;
}

int moe_register_weights(moe_ctx* ctx, const void* host_base, size_t bytes) {
    TRY(begin(ctx));
    if (!host_base || !bytes) return fail(ctx, MOE_E_ARG, "null or empty range");
    const char* h = static_cast<const char*>(host_base);
    for (const Reg& r : ctx->regs)
        if (h < r.host + r.bytes && r.host < h + bytes)
            return fail(ctx, MOE_E_ARG, "range overlaps an existing registration");
    char* d = nullptr;
    if (cudaMalloc(&d, bytes) != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, MOE_E_NOMEM, "device allocation for the weight mirror failed");
    }
    cudaError_t e = cudaMemcpy(d, host_base, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(d);
        return cuda_fail(ctx, e, "weight upload");
    }
    ctx->regs.push_back({h, bytes, d});
    return MOE_OK;
}

int moe_load_weights_file(moe_ctx* ctx, const char* path, int64_t file_offset, int64_t bytes,
                          void* dst, int64_t* bytes_loaded) {
    TRY(begin(ctx));
    if (bytes_loaded) *bytes_loaded = 0;
    if (!path || !dst) return fail(ctx, MOE_E_ARG, "null pointer");
    cudaPointerAttributes at;
    cudaError_t e = cudaPointerGetAttributes(&at, dst);
    if (e != cudaSuccess || at.type != cudaMemoryTypeDevice) {
        cudaGetLastError();
        return fail(ctx, MOE_E_ARG, "dst must be device memory");
    }
    // the copies must stay inside dst's allocation (driver call looked up
    // through the runtime, so the library needs no link-time libcuda)
    using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
    static RangeFn range_fn = nullptr;
    if (!range_fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return fail(ctx, MOE_E_CUDA, "cuMemGetAddressRange not available");
        range_fn = reinterpret_cast<RangeFn>(p);
    }
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range_fn(&base, &size, (CUdeviceptr)dst) != CUDA_SUCCESS)
        return fail(ctx, MOE_E_ARG, "dst is not inside a device allocation");
    const int64_t capacity = (int64_t)(base + size - (CUdeviceptr)dst);
    // work queued earlier on the stream (e.g. a kernel still reading the old
    // contents of dst) runs before the copies, which are queued behind it
    int64_t loaded = 0;
    std::string err;
    int s = moe::load_file_range(path, file_offset, bytes, static_cast<char*>(dst), capacity,
                                 ctx->stream, ctx->file_staging, err, &loaded);
    if (s != MOE_OK) return fail(ctx, s, err);
    if (bytes_loaded) *bytes_loaded = loaded;
    return MOE_OK;
}

int moe_unregister_weights(moe_ctx* ctx, const void* host_base) {
    TRY(begin(ctx));
    for (size_t i = 0; i < ctx->regs.size(); ++i)
        if (ctx->regs[i].host == host_base) {
            MOE_CUDA(cudaStreamSynchronize(ctx->stream));
            cudaFree(ctx->regs[i].dev);
            ctx->regs.erase(ctx->regs.begin() + i);
            return MOE_OK;
        }
    return fail(ctx, MOE_E_ARG, "no registration starts at this address");
}

// ----------------------------------------------------------------- Q4_0
int moe_quantize_fp32_to_q4_0(moe_ctx* ctx, const float* src, uint8_t* dst_packed,
                              float* dst_scales, int64_t n) {
    TRY(begin(ctx));
    if (!src || !dst_packed || !dst_scales) return fail(ctx, MOE_E_ARG, "null pointer");
    if (n < 0 || n % 32) return fail(ctx, MOE_E_SHAPE, "num_elements must be a multiple of 32");
    if (n == 0) return MOE_OK;
    TRY(ws_reserve(ctx, al(n * 4) + al(n / 2) + al(n / 8)));
    void *s, *p, *sc;
    TRY(dev_ptr(ctx, src, n * 4, K_IN, &s));
    TRY(dev_ptr(ctx, dst_packed, n / 2, K_OUT, &p));
    TRY(dev_ptr(ctx, dst_scales, n / 32 * 4, K_OUT, &sc));
    if (!al16(s) || !al16(p)) return fail(ctx, MOE_E_ARG, "device buffers must be 16-byte aligned");
    ctx->launches += moe::launch_quantize((const float*)s, (uint8_t*)p, (float*)sc, n / 32, ctx->stream);
    return finish(ctx);
}

int moe_q4_matmul_batchN(moe_ctx* ctx, int64_t batch, const uint8_t* W, const float* S,
                         const float* x, float* out, int64_t c_in, int64_t c_out) {
    TRY(begin(ctx));
    if (!W || !S || !x || !out) return fail(ctx, MOE_E_ARG, "null pointer");
    TRY(check_q4_shape(ctx, c_in, c_out));
    if (batch <= 0) return fail(ctx, MOE_E_SHAPE, "batch_size must be >= 1");
    if (batch > (1 << 20)) return fail(ctx, MOE_E_SHAPE, "batch_size too large");
    TRY(ws_reserve(ctx, al(batch * c_in * 4) * 2 + al(batch * c_out * 4) + al(batch * c_in * 2) +
                            al(batch * c_out * 4 * (c_in / 256 + 1))));
    void *w, *sc, *xd, *od;
    TRY(dev_ptr(ctx, W, c_out * c_in / 2, K_W, &w));
    TRY(dev_ptr(ctx, S, c_out * c_in / 32 * 4, K_W, &sc));
    TRY(dev_ptr(ctx, x, batch * c_in * 4, K_IN, &xd));
    TRY(dev_ptr(ctx, out, batch * c_out * 4, K_OUT, &od));
    if (!al16(w)) return fail(ctx, MOE_E_ARG, "packed weights must be 16-byte aligned");
    if (!al16(xd)) {  // the GEMV reads activations as float4
        float* xc = (float*)ws_take(ctx, batch * c_in * 4);
        TRY(prep_rows(ctx, xd, MOE_X_NATURAL, 0, batch, c_in, xc, nullptr));
        xd = xc;
    }
    TRY(dense_q4(ctx, (const uint8_t*)w, (const float*)sc, (const float*)xd, (float*)od, c_in, c_out,
                 batch, "q4_matmul"));
    return finish(ctx);
}

int moe_rms_norm(moe_ctx* ctx, const float* x, const float* w, float* out, int64_t M, int64_t d) {
    TRY(begin(ctx));
    if (!x || !w || !out) return fail(ctx, MOE_E_ARG, "null pointer");
    if (M < 0 || d <= 0 || d % 32) return fail(ctx, MOE_E_SHAPE, "d must be a positive multiple of 32");
    if (M == 0) return MOE_OK;
    TRY(ws_reserve(ctx, al(M * d * 4) * 2 + al(d * 4)));
    void *xd, *wd, *od;
    TRY(dev_ptr(ctx, x, M * d * 4, K_IN, &xd));
    TRY(dev_ptr(ctx, w, d * 4, K_IN, &wd));
    TRY(dev_ptr(ctx, out, M * d * 4, K_OUT, &od));
    moe::PrepArgs pa;
    pa.x = xd;
    pa.K = d;
    pa.norm = 1;
    pa.pre_w = (const float*)wd;
    pa.out = (float*)od;
    {
        ProfScope ps(ctx, "rms_norm");
        ctx->launches += moe::launch_prep(pa, M, ctx->stream);
    }
    return finish(ctx);
}

int moe_q4_matmul_vec(moe_ctx* ctx, const uint8_t* W, const float* S, const float* x, float* out,
                      int64_t c_in, int64_t c_out) {
    return moe_q4_matmul_batchN(ctx, 1, W, S, x, out, c_in, c_out);
}

// -------------------------------------------------------------- routing
int moe_compute_moe_lod_weights(moe_ctx* ctx, int64_t batch, const int64_t* top_idx,
                                const float* top_val, const float* pes, float top_p,
                                int64_t* act_idx, float* act_w, int64_t* act_count,
                                int64_t top_k) {
    TRY(begin(ctx));
    if (!top_idx || !top_val || !pes || !act_idx || !act_w || !act_count)
        return fail(ctx, MOE_E_ARG, "null pointer");
    if (batch <= 0 || top_k <= 0) return fail(ctx, MOE_E_SHAPE, "batch and top_k must be >= 1");
    // per_expert_scale is indexed by expert id; when it has to be staged its
    // extent is taken from the largest id (host index arrays) or 128.
    int64_t E = 128;
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, top_idx) != cudaSuccess) cudaGetLastError();
    else if (at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged) {
        int64_t mx = -1;
        for (int64_t i = 0; i < batch * top_k; ++i) mx = std::max(mx, top_idx[i]);
        for (int64_t i = 0; i < batch * top_k; ++i)
            if (top_idx[i] < 0) return fail(ctx, MOE_E_ARG, "negative expert index");
        E = std::max<int64_t>(E, mx + 1);
    }
    const int64_t P = batch * top_k;
    TRY(ws_reserve(ctx, al(P * 8) * 2 + al(P * 4) * 2 + al(E * 4) + al(batch * 8)));
    void *ti, *tv, *pe, *ai, *aw, *ac;
    TRY(dev_ptr(ctx, top_idx, P * 8, K_IN, &ti));
    TRY(dev_ptr(ctx, top_val, P * 4, K_IN, &tv));
    TRY(dev_ptr(ctx, pes, E * 4, K_IN, &pe));
    TRY(dev_ptr(ctx, act_idx, P * 8, K_INOUT, &ai));
    TRY(dev_ptr(ctx, act_w, P * 4, K_INOUT, &aw));
    TRY(dev_ptr(ctx, act_count, batch * 8, K_OUT, &ac));
    ctx->launches += moe::launch_lod(batch, (const int64_t*)ti, (const float*)tv, (const float*)pe,
                                     top_p, (int64_t*)ai, (float*)aw, (int64_t*)ac, (int)top_k,
                                     E, ctx->err_flag, ctx->stream);
    return finish(ctx);
}

int moe_apply_moe_lod_and_set_cover(moe_ctx* ctx, const int64_t* top_idx, const float* top_val,
                                    const float* pes, float* top_w, int64_t B, int64_t top_k,
                                    int64_t active_top_k, float top_p, const uint8_t* eb_mask,
                                    const int64_t* active_canvas_idx, int64_t unaccepted_top_k) {
    (void)top_p;
    TRY(begin(ctx));
    if (!top_idx || !top_val || !pes || !top_w) return fail(ctx, MOE_E_ARG, "null pointer");
    if (B <= 0 || top_k <= 0) return fail(ctx, MOE_E_SHAPE, "B and top_k must be >= 1");
    const int64_t P = B * top_k;
    // eb_mask is indexed by the original canvas position
    int64_t mask_n = B;
    if (eb_mask && active_canvas_idx) {
        cudaPointerAttributes at;
        if (cudaPointerGetAttributes(&at, active_canvas_idx) != cudaSuccess) cudaGetLastError();
        else if (at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged)
            for (int64_t i = 0; i < B; ++i) mask_n = std::max(mask_n, active_canvas_idx[i] + 1);
    }
    TRY(ws_reserve(ctx, al(P * 8) + al(P * 4) * 2 + al(128 * 4) + al(mask_n) + al(B * 8)));
    void *ti, *tv, *pe, *tw, *eb = nullptr, *ac = nullptr;
    TRY(dev_ptr(ctx, top_idx, P * 8, K_IN, &ti));
    TRY(dev_ptr(ctx, top_val, P * 4, K_IN, &tv));
    TRY(dev_ptr(ctx, pes, 128 * 4, K_IN, &pe));
    TRY(dev_ptr(ctx, top_w, P * 4, K_OUT, &tw));
    if (eb_mask) TRY(dev_ptr(ctx, eb_mask, mask_n, K_IN, &eb));
    if (active_canvas_idx) TRY(dev_ptr(ctx, active_canvas_idx, B * 8, K_IN, &ac));
    ctx->launches += moe::launch_apply_lod((const int64_t*)ti, (const float*)tv, (const float*)pe,
                                           (float*)tw, B, (int)top_k, active_top_k,
                                           (const uint8_t*)eb, (const int64_t*)ac,
                                           unaccepted_top_k, ctx->stream);
    return finish(ctx);
}

int moe_compute_subbatch_set_cover_moe_weights(moe_ctx* ctx, int64_t sub_b, const int64_t* ti,
                                               const float* tv, const float* pes, float top_p,
                                               int64_t* tc, int64_t* tidx, float* tw,
                                               int64_t num_experts, int64_t top_k,
                                               float core_top_p, float smp) {
    TRY(begin(ctx));
    if (!ti || !tv || !pes || !tc || !tidx || !tw) return fail(ctx, MOE_E_ARG, "null pointer");
    if (sub_b <= 0 || sub_b > 64) return fail(ctx, MOE_E_SHAPE, "sub_b must be in [1, 64]");
    if (top_k <= 0 || top_k > 32) return fail(ctx, MOE_E_SHAPE, "top_k must be in [1, 32]");
    if (num_experts <= 0 || num_experts > 1024) return fail(ctx, MOE_E_SHAPE, "num_experts must be in [1, 1024]");
    const int64_t P = sub_b * top_k;
    TRY(ws_reserve(ctx, al(P * 8) * 3 + al(P * 4) * 4 + al(num_experts * 4) + al(sub_b * 8)));
    void *dti, *dtv, *dpe, *dtc, *dtidx, *dtw;
    TRY(dev_ptr(ctx, ti, P * 8, K_IN, &dti));
    TRY(dev_ptr(ctx, tv, P * 4, K_IN, &dtv));
    TRY(dev_ptr(ctx, pes, num_experts * 4, K_IN, &dpe));
    TRY(dev_ptr(ctx, tc, sub_b * 8, K_OUT, &dtc));
    TRY(dev_ptr(ctx, tidx, P * 8, K_INOUT, &dtidx));
    TRY(dev_ptr(ctx, tw, P * 4, K_INOUT, &dtw));
    // the kernel reads int32 ids; narrow them on device
    int* ti32 = (int*)ws_take(ctx, P * 4);
    float* dummy_w = (float*)ws_take(ctx, P * 4);
    ctx->launches += moe::launch_slots_from_lists(sub_b, (int)top_k, nullptr, top_k,
                                                  (const int64_t*)dti, nullptr, ti32, dummy_w,
                                                  (int)num_experts, ctx->err_flag, ctx->stream);
    ctx->launches += moe::launch_set_cover(ti32, (const float*)dtv, sub_b, (int)top_k,
                                           (int)num_experts, (const float*)dpe, top_p, core_top_p,
                                           smp, (int)sub_b, nullptr, nullptr, (int64_t*)dtc,
                                           (int64_t*)dtidx, (float*)dtw, ctx->stream);
    return finish(ctx);
}

// -------------------------------------------------------- expert stages
int moe_run_moe_experts_stage1(moe_ctx* ctx, const uint8_t* gu_p, const float* gu_s,
                               const float* moe_in, const int64_t* active_idx, int64_t count,
                               float* gu_out_all, float* act_all, int64_t d, int64_t F,
                               int activation) {
    TRY(begin(ctx));
    if (!gu_p || !gu_s || !moe_in || !act_all || (count > 0 && !active_idx))
        return fail(ctx, MOE_E_ARG, "null pointer");
    TRY(check_q4_shape(ctx, d, 2 * F));
    TRY(check_q4_shape(ctx, F, d));
    if (count < 0 || count > 32) return fail(ctx, MOE_E_SHAPE, "active_count must be in [0, 32]");
    if (activation < 0 || activation > 1) return fail(ctx, MOE_E_ARG, "bad activation");
    if (count == 0) return MOE_OK;
    const int64_t E = 1024;
    TRY(ws_reserve(ctx, expert_bufs_bytes(1, count, d, F, E) + al(d * 4) + al(count * 8) +
                            al(count * 2 * F * 4) + al(count * F * 4)));
    void *wp, *ws, *xi, *ai, *go = nullptr, *ao;
    TRY(dev_ptr(ctx, gu_p, 1, K_W, &wp));
    TRY(dev_ptr(ctx, gu_s, 1, K_W, &ws));
    TRY(dev_ptr(ctx, moe_in, d * 4, K_IN, &xi));
    TRY(dev_ptr(ctx, active_idx, count * 8, K_IN, &ai));
    if (gu_out_all) TRY(dev_ptr(ctx, gu_out_all, count * 2 * F * 4, K_OUT, &go));
    TRY(dev_ptr(ctx, act_all, count * F * 4, K_OUT, &ao));
    if (!al16(wp)) return fail(ctx, MOE_E_ARG, "packed weights must be 16-byte aligned");
    ExpertBufs bb;
    TRY(take_expert_bufs(ctx, 1, count, d, F, E, &bb));
    cudaStream_t s = ctx->stream;
    ctx->launches += moe::launch_slots_from_lists(1, (int)count, nullptr, count,
                                                  (const int64_t*)ai, nullptr, bb.slot_expert,
                                                  bb.slot_weight, (int)E, ctx->err_flag, s);
    ctx->launches += moe::launch_bucket(bb.slot_expert, count, (int)count, (int)E, 0, (int)E, bb.b, s);
    TRY(prep_rows(ctx, xi, MOE_X_NATURAL, 0, 1, d, bb.x32, bb.xsum));
    moe::GemvArgs g;
    g.Wp = (const uint8_t*)wp;
    g.Ws = (const float*)ws;
    g.rows_per_expert = 2 * F;
    g.K = (int)d;
    g.X = bb.x32;
    g.xsum = bb.xsum;
    g.meta = bb.b.meta;
    g.unique_expert = bb.b.unique_expert;
    g.seg_start = bb.b.seg_start;
    g.seg_count = bb.b.seg_count;
    g.pair_row = bb.b.pair_token;
    g.out_row = bb.b.pair_slot;
    g.out = (float*)ao;
    g.out_stride = F;
    g.gu_out = (float*)go;
    g.gu_stride = 2 * F;
    g.F = (int)F;
    g.act = activation;
    g.max_tokens = 1;
    g.max_unique = (int)count;
    ctx->launches += moe::launch_gemv(moe::GEMV_ACT, g, ctx->num_sms, s);
    return finish(ctx);
}

int moe_run_moe_experts_stage2(moe_ctx* ctx, const uint8_t* dn_p, const float* dn_s,
                               const float* act_all, const int64_t* active_idx,
                               const float* active_w, int64_t count, float* moe_out, int64_t d,
                               int64_t F) {
    TRY(begin(ctx));
    if (!dn_p || !dn_s || !moe_out || (count > 0 && (!act_all || !active_idx || !active_w)))
        return fail(ctx, MOE_E_ARG, "null pointer");
    TRY(check_q4_shape(ctx, F, d));
    if (count < 0 || count > 32) return fail(ctx, MOE_E_SHAPE, "active_count must be in [0, 32]");
    const int64_t E = 1024, Kc = std::max<int64_t>(count, 1);
    TRY(ws_reserve(ctx, expert_bufs_bytes(1, Kc, d, F, E) + al(Kc * F * 4) * 2 + al(Kc * 8) +
                            al(Kc * 4) + al(d * 4)));
    void *wp, *ws, *aa = nullptr, *ai = nullptr, *aw = nullptr, *mo;
    TRY(dev_ptr(ctx, dn_p, 1, K_W, &wp));
    TRY(dev_ptr(ctx, dn_s, 1, K_W, &ws));
    if (count > 0) {
        TRY(dev_ptr(ctx, act_all, count * F * 4, K_IN, &aa));
        TRY(dev_ptr(ctx, active_idx, count * 8, K_IN, &ai));
        TRY(dev_ptr(ctx, active_w, count * 4, K_IN, &aw));
    }
    TRY(dev_ptr(ctx, moe_out, d * 4, K_OUT, &mo));
    if (!al16(wp)) return fail(ctx, MOE_E_ARG, "packed weights must be 16-byte aligned");
    cudaStream_t s = ctx->stream;
    if (count == 0) {  // moe_kernels.mojo:742-743 zeroes moe_out
        MOE_CUDA(cudaMemsetAsync(mo, 0, d * 4, s));
        return finish(ctx);
    }
    ExpertBufs bb;
    TRY(take_expert_bufs(ctx, 1, count, d, F, E, &bb));
    ctx->launches += moe::launch_slots_from_lists(1, (int)count, nullptr, count,
                                                  (const int64_t*)ai, (const float*)aw,
                                                  bb.slot_expert, bb.slot_weight, (int)E,
                                                  ctx->err_flag, s);
    ctx->launches += moe::launch_bucket(bb.slot_expert, count, (int)count, (int)E, 0, (int)E, bb.b, s);
    if (!al16(aa)) {
        float* ac = (float*)ws_take(ctx, count * F * 4);
        TRY(prep_rows(ctx, aa, MOE_X_NATURAL, 0, count, F, ac, nullptr));
        aa = ac;
    }
    moe::GemvArgs g;
    g.Wp = (const uint8_t*)wp;
    g.Ws = (const float*)ws;
    g.rows_per_expert = d;
    g.K = (int)F;
    g.X = (const float*)aa;
    g.meta = bb.b.meta;
    g.unique_expert = bb.b.unique_expert;
    g.seg_start = bb.b.seg_start;
    g.seg_count = bb.b.seg_count;
    g.pair_row = bb.b.pair_slot;  // act_all rows are in slot order
    g.out = bb.y;
    g.out_stride = d;
    g.max_tokens = 1;
    g.max_unique = (int)count;
    ctx->launches += moe::launch_gemv(moe::GEMV_PLAIN, g, ctx->num_sms, s);
    moe::CombineArgs c;
    c.y = bb.y;
    c.d = d;
    c.K = (int)count;
    c.slot_pair = bb.b.slot_pair;
    c.slot_weight = bb.slot_weight;
    c.out = mo;
    ctx->launches += moe::launch_combine(c, 1, s);
    return finish(ctx);
}

int moe_run_moe_coalesced_core(moe_ctx* ctx, int64_t sub_b, const uint8_t* gu_p, const float* gu_s,
                               const uint8_t* dn_p, const float* dn_s, const float* batch_in,
                               int x_layout, const int64_t* tok_count, const int64_t* tok_idx,
                               const float* tok_w, float* batch_out, int64_t d, int64_t F,
                               int64_t E, int64_t top_k, int activation) {
    TRY(begin(ctx));
    if (!gu_p || !gu_s || !dn_p || !dn_s || !batch_in || !tok_count || !tok_idx || !tok_w || !batch_out)
        return fail(ctx, MOE_E_ARG, "null pointer");
    TRY(check_q4_shape(ctx, d, 2 * F));
    TRY(check_q4_shape(ctx, F, d));
    if (sub_b <= 0) return fail(ctx, MOE_E_SHAPE, "sub_b must be >= 1");
    if (top_k <= 0 || top_k > 32) return fail(ctx, MOE_E_SHAPE, "top_k must be in [1, 32]");
    if (E <= 0 || E > 1024) return fail(ctx, MOE_E_SHAPE, "num_experts must be in [1, 1024]");
    if (x_layout < 0 || x_layout > 2 || activation < 0 || activation > 1)
        return fail(ctx, MOE_E_ARG, "bad layout or activation");
    const int64_t P = sub_b * top_k;
    TRY(ws_reserve(ctx, expert_bufs_bytes(sub_b, top_k, d, F, E) + al(sub_b * d * 4) * 2 +
                            al(sub_b * 8) + al(P * 8) + al(P * 4)));
    void *gp, *gs, *dp, *ds, *xi, *tc, *ti, *tw, *out;
    TRY(dev_ptr(ctx, gu_p, 1, K_W, &gp));
    TRY(dev_ptr(ctx, gu_s, 1, K_W, &gs));
    TRY(dev_ptr(ctx, dn_p, 1, K_W, &dp));
    TRY(dev_ptr(ctx, dn_s, 1, K_W, &ds));
    TRY(dev_ptr(ctx, batch_in, sub_b * d * 4, K_IN, &xi));
    TRY(dev_ptr(ctx, tok_count, sub_b * 8, K_IN, &tc));
    TRY(dev_ptr(ctx, tok_idx, P * 8, K_IN, &ti));
    TRY(dev_ptr(ctx, tok_w, P * 4, K_IN, &tw));
    TRY(dev_ptr(ctx, batch_out, sub_b * d * 4, K_OUT, &out));
    if (!al16(gp) || !al16(dp)) return fail(ctx, MOE_E_ARG, "packed weights must be 16-byte aligned");
    ExpertBufs bb;
    TRY(take_expert_bufs(ctx, sub_b, top_k, d, F, E, &bb));
    ctx->launches += moe::launch_slots_from_lists(sub_b, (int)top_k, (const int64_t*)tc, 0,
                                                  (const int64_t*)ti, (const float*)tw,
                                                  bb.slot_expert, bb.slot_weight, (int)E,
                                                  ctx->err_flag, ctx->stream);
    ExpertWeights w{(const uint8_t*)gp, (const float*)gs, (const uint8_t*)dp, (const float*)ds};
    moe::CombineArgs c;
    TRY(prep_rows(ctx, xi, x_layout, 0, sub_b, d, bb.x32, bb.xsum));
    TRY(run_experts(ctx, w, sub_b, top_k, d, F, E, activation, bb, &c, out));
    return finish(ctx);
}

// ---- run_moe_coalesced_stage1 / stage2: the core in two calls
}  // extern "C"

namespace {

constexpr int64_t kBucketCap = 5;  // bucket entries per expert (moe_kernels.mojo:824)

// Reads a small caller array (host or device memory) into `dst` after the
// work queued on the context's stream.
int get_small(moe_ctx* ctx, void* dst, const void* src, size_t bytes) {
    MOE_CUDA(cudaStreamSynchronize(ctx->stream));
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, src) != cudaSuccess) {
        cudaGetLastError();
        at.type = cudaMemoryTypeUnregistered;
    }
    if (at.type == cudaMemoryTypeDevice) {
        MOE_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
        MOE_CUDA(cudaStreamSynchronize(ctx->stream));
    } else {
        std::memcpy(dst, src, bytes);
    }
    return MOE_OK;
}

// Writes a small host-computed array to a caller buffer (host or device).
int put_small(moe_ctx* ctx, void* dst, const void* src, size_t bytes) {
    if (!bytes) return MOE_OK;
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, dst) != cudaSuccess) {
        cudaGetLastError();
        at.type = cudaMemoryTypeUnregistered;
    }
    if (at.type == cudaMemoryTypeDevice) {
        MOE_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
        MOE_CUDA(cudaStreamSynchronize(ctx->stream));  // `src` is a host temporary
    } else {
        std::memcpy(dst, src, bytes);
    }
    return MOE_OK;
}

}  // namespace

extern "C" {

int moe_run_moe_coalesced_stage1(moe_ctx* ctx, int64_t sub_b, const uint8_t* gu_p, const float* gu_s,
                                 const float* batch_in, int x_layout, const int64_t* tok_count,
                                 const int64_t* tok_idx, const float* tok_w, int64_t* bucket_counts,
                                 int64_t* bucket_toks, float* bucket_weights, int64_t* unique_experts,
                                 int64_t* unique_base_slot, const float* act_deint_scratch, int64_t d,
                                 int64_t F, int64_t E, int64_t top_k, int activation, int64_t* num_unique) {
    TRY(begin(ctx));
    if (!gu_p || !gu_s || !batch_in || !tok_count || !tok_idx || !tok_w || !bucket_counts || !bucket_toks ||
        !bucket_weights || !unique_experts || !unique_base_slot || !act_deint_scratch || !num_unique)
        return fail(ctx, MOE_E_ARG, "null pointer");
    TRY(check_q4_shape(ctx, d, 2 * F));
    TRY(check_q4_shape(ctx, F, d));
    if (sub_b < 1 || sub_b > kBucketCap)
        return fail(ctx, MOE_E_SHAPE, "sub_b must be in [1, 5] (five bucket entries per expert)");
    if (top_k <= 0 || top_k > 32) return fail(ctx, MOE_E_SHAPE, "top_k must be in [1, 32]");
    if (E <= 0 || E > 1024) return fail(ctx, MOE_E_SHAPE, "num_experts must be in [1, 1024]");
    if (x_layout < 0 || x_layout > 2 || activation < 0 || activation > 1)
        return fail(ctx, MOE_E_ARG, "bad layout or activation");
    ctx->split.active = false;
    const int64_t P = sub_b * top_k;
    // the reference's buckets (moe_kernels.mojo:815-835), built on the host:
    // the call returns their unique-expert count
    std::vector<int64_t> cnt(sub_b), idx(P), bc(E, 0), bt(E * kBucketCap, 0), ue, ub;
    std::vector<float> wt(P), bw(E * kBucketCap, 0.f);
    TRY(get_small(ctx, cnt.data(), tok_count, sub_b * 8));
    TRY(get_small(ctx, idx.data(), tok_idx, P * 8));
    TRY(get_small(ctx, wt.data(), tok_w, P * 4));
    for (int64_t b = 0; b < sub_b; ++b) {
        if (cnt[b] < 0 || cnt[b] > top_k) return fail(ctx, MOE_E_ARG, "active count out of range");
        for (int64_t k = 0; k < cnt[b]; ++k) {
            const int64_t e = idx[b * top_k + k];
            if (e < 0 || e >= E) return fail(ctx, MOE_E_ARG, "expert index out of range in a routing array");
            const int64_t c = bc[e];
            if (c >= kBucketCap) return fail(ctx, MOE_E_ARG, "more than five entries for one expert");
            bt[e * kBucketCap + c] = b;
            bw[e * kBucketCap + c] = wt[b * top_k + k];
            bc[e] = c + 1;
        }
    }
    int64_t total = 0;
    for (int64_t e = 0; e < E; ++e)
        if (bc[e] > 0) {
            ue.push_back(e);
            ub.push_back(total);
            total += bc[e];
        }
    const int64_t nu = (int64_t)ue.size();
    TRY(put_small(ctx, bucket_counts, bc.data(), E * 8));
    TRY(put_small(ctx, bucket_toks, bt.data(), E * kBucketCap * 8));
    TRY(put_small(ctx, bucket_weights, bw.data(), E * kBucketCap * 4));
    TRY(put_small(ctx, unique_experts, ue.data(), nu * 8));
    TRY(put_small(ctx, unique_base_slot, ub.data(), nu * 8));
    TRY(put_small(ctx, num_unique, &nu, 8));
    // the device half: the core's kernels up to the activations, into the
    // context's split arena
    const size_t need = expert_bufs_bytes(sub_b, top_k, d, F, E) + 64 * kAlign;
    if (ctx->split_cap < need) {
        MOE_CUDA(cudaStreamSynchronize(ctx->stream));
        if (ctx->split_ws) cudaFree(ctx->split_ws);
    if (ctx->ep_ws) cudaFree(ctx->ep_ws);
    if (ctx->ep_host_cnt) cudaFreeHost(ctx->ep_host_cnt);
        ctx->split_ws = nullptr;
        ctx->split_cap = 0;
        if (cudaMalloc(&ctx->split_ws, need) != cudaSuccess) {
            cudaGetLastError();
            ctx->split_ws = nullptr;
            return fail(ctx, MOE_E_NOMEM, "device allocation for the stage-1 buffers failed");
        }
        ctx->split_cap = need;
    }
    size_t off = 0;
    auto take = [&](size_t b) -> void* {
        const size_t o = (off + kAlign - 1) / kAlign * kAlign;
        if (o + b > ctx->split_cap) return nullptr;
        off = o + b;
        return ctx->split_ws + o;
    };
    ExpertBufs bb;
    if (!carve_expert_bufs(take, sub_b, top_k, d, F, E, &bb)) return fail(ctx, MOE_E_NOMEM, "stage-1 arena exhausted");
    TRY(ws_reserve(ctx, al(sub_b * d * 4) + al(sub_b * 8) + al(P * 8) + al(P * 4)));
    void *gp, *gs, *xi, *tc, *ti, *tw;
    TRY(dev_ptr(ctx, gu_p, 1, K_W, &gp));
    TRY(dev_ptr(ctx, gu_s, 1, K_W, &gs));
    TRY(dev_ptr(ctx, batch_in, sub_b * d * 4, K_IN, &xi));
    TRY(dev_ptr(ctx, tok_count, sub_b * 8, K_IN, &tc));
    TRY(dev_ptr(ctx, tok_idx, P * 8, K_IN, &ti));
    TRY(dev_ptr(ctx, tok_w, P * 4, K_IN, &tw));
    if (!al16(gp)) return fail(ctx, MOE_E_ARG, "packed weights must be 16-byte aligned");
    ctx->launches += moe::launch_slots_from_lists(sub_b, (int)top_k, (const int64_t*)tc, 0, (const int64_t*)ti,
                                                  (const float*)tw, bb.slot_expert, bb.slot_weight, (int)E,
                                                  ctx->err_flag, ctx->stream);
    TRY(prep_rows(ctx, xi, x_layout, 0, sub_b, d, bb.x32, bb.xsum));
    ExpertWeights w{(const uint8_t*)gp, (const float*)gs, nullptr, nullptr};  // down weights: stage 2
    ExpertPlan p;
    plan_experts(ctx, w, sub_b, top_k, d, F, E, activation, bb, &p);
    TRY(experts_stage1(ctx, p, bb, sub_b, top_k, d, E, false));
    auto& sp = ctx->split;
    sp.key = act_deint_scratch;
    sp.sub_b = sub_b;
    sp.top_k = top_k;
    sp.d = d;
    sp.F = F;
    sp.E = E;
    sp.num_unique = nu;
    sp.act = activation;
    sp.gu_p = w.gu_p;
    sp.gu_s = w.gu_s;
    sp.tc = p.tc;
    sp.stream = p.stream;
    sp.bb = bb;
    TRY(finish(ctx));
    sp.active = true;
    return MOE_OK;
}

int moe_run_moe_coalesced_stage2(moe_ctx* ctx, int64_t sub_b, int64_t num_unique, const uint8_t* dn_p,
                                 const float* dn_s, const int64_t* bucket_counts, const int64_t* bucket_toks,
                                 const float* bucket_weights, const int64_t* unique_experts,
                                 const int64_t* unique_base_slot, const float* act_deint_scratch,
                                 float* batch_moe_out, int64_t d, int64_t F) {
    TRY(begin(ctx));
    (void)bucket_counts;  // the buckets stage 1 built stay on the device
    (void)bucket_toks;
    (void)bucket_weights;
    (void)unique_experts;
    (void)unique_base_slot;
    if (!dn_p || !dn_s || !act_deint_scratch || !batch_moe_out) return fail(ctx, MOE_E_ARG, "null pointer");
    auto& sp = ctx->split;
    if (!sp.active || sp.key != act_deint_scratch)
        return fail(ctx, MOE_E_STATE, "no stage-1 result for this act_deint_scratch on this context");
    if (sub_b != sp.sub_b || num_unique != sp.num_unique || d != sp.d || F != sp.F)
        return fail(ctx, MOE_E_ARG, "sub_b, num_unique or the dimensions differ from stage 1");
    TRY(ws_reserve(ctx, al(sub_b * d * 4)));
    void *dp, *ds, *out;
    TRY(dev_ptr(ctx, dn_p, 1, K_W, &dp));
    TRY(dev_ptr(ctx, dn_s, 1, K_W, &ds));
    TRY(dev_ptr(ctx, batch_moe_out, sub_b * d * 4, K_OUT, &out));
    if (!al16(dp)) return fail(ctx, MOE_E_ARG, "packed weights must be 16-byte aligned");
    ExpertWeights w{sp.gu_p, sp.gu_s, (const uint8_t*)dp, (const float*)ds};
    ExpertPlan p;
    plan_experts(ctx, w, sp.sub_b, sp.top_k, sp.d, sp.F, sp.E, sp.act, sp.bb, &p);
    if (p.tc != sp.tc || p.stream != sp.stream)
        return fail(ctx, MOE_E_STATE, "the expert path changed between the stages (options or down-weight alignment)");
    sp.active = false;  // consumed, whatever happens below
    moe::CombineArgs c;
    TRY(experts_stage2(ctx, p, sp.bb, sp.sub_b, sp.top_k, sp.d, &c, out));
    return finish(ctx);
}

int moe_run_diffusion_moe_experts_parallel(moe_ctx* ctx, const uint8_t* gu_p, const float* gu_s,
                                           const uint8_t* dn_p, const float* dn_s,
                                           const uint16_t* in_f16, const int64_t* top_idx,
                                           const float* top_w, uint16_t* out_f16, int64_t B,
                                           int64_t d, int64_t F, int64_t top_k, int activation) {
    TRY(begin(ctx));
    if (!gu_p || !gu_s || !dn_p || !dn_s || !in_f16 || !top_idx || !top_w || !out_f16)
        return fail(ctx, MOE_E_ARG, "null pointer");
    TRY(check_q4_shape(ctx, d, 2 * F));
    TRY(check_q4_shape(ctx, F, d));
    if (B <= 0) return fail(ctx, MOE_E_SHAPE, "B must be >= 1");
    if (top_k <= 0 || top_k > 32) return fail(ctx, MOE_E_SHAPE, "top_k must be in [1, 32]");
    if (activation < 0 || activation > 1) return fail(ctx, MOE_E_ARG, "bad activation");
    const int64_t E = 128;  // diffusion_kernels.mojo:255 fixes 128 expert buckets
    const int64_t P = B * top_k;
    TRY(ws_reserve(ctx, expert_bufs_bytes(B, top_k, d, F, E) + al(B * d * 2) * 2 + al(P * 8) +
                            al(P * 4)));
    void *gp, *gs, *dp, *ds, *xi, *ti, *tw, *out;
    TRY(dev_ptr(ctx, gu_p, 1, K_W, &gp));
    TRY(dev_ptr(ctx, gu_s, 1, K_W, &gs));
    TRY(dev_ptr(ctx, dn_p, 1, K_W, &dp));
    TRY(dev_ptr(ctx, dn_s, 1, K_W, &ds));
    TRY(dev_ptr(ctx, in_f16, B * d * 2, K_IN, &xi));
    TRY(dev_ptr(ctx, top_idx, P * 8, K_IN, &ti));
    TRY(dev_ptr(ctx, top_w, P * 4, K_IN, &tw));
    TRY(dev_ptr(ctx, out_f16, B * d * 2, K_OUT, &out));
    if (!al16(gp) || !al16(dp)) return fail(ctx, MOE_E_ARG, "packed weights must be 16-byte aligned");
    ExpertBufs bb;
    TRY(take_expert_bufs(ctx, B, top_k, d, F, E, &bb));
    ctx->launches += moe::launch_slots_from_topw(B, (int)top_k, (const int64_t*)ti, (const float*)tw,
                                                 bb.slot_expert, bb.slot_weight, (int)E,
                                                 ctx->err_flag, ctx->stream);
    ExpertWeights w{(const uint8_t*)gp, (const float*)gs, (const uint8_t*)dp, (const float*)ds};
    moe::CombineArgs c;
    c.fma_mode = 1;
    c.out_f16 = 1;
    TRY(prep_rows(ctx, xi, MOE_X_NATURAL, 1, B, d, bb.x32, bb.xsum));
    TRY(run_experts(ctx, w, B, top_k, d, F, E, activation, bb, &c, out));
    return finish(ctx);
}

// ------------------------------------------- diffusion router-subspace bypass
}  // extern "C"

namespace {

// Number of canvas rows the per-canvas arrays (indexed by
// active_canvas_idx[b], else by b) must hold: max(B, max index + 1).
int canvas_rows(moe_ctx* ctx, const int64_t* active_idx, int64_t B, int64_t* n) {
    *n = B;
    if (!active_idx) return MOE_OK;
    std::vector<int64_t> h((size_t)B);
    TRY(get_small(ctx, h.data(), active_idx, (size_t)B * 8));
    for (int64_t v : h) {
        if (v < 0) return fail(ctx, MOE_E_ARG, "negative entry in active_canvas_idx");
        *n = std::max(*n, v + 1);
    }
    return MOE_OK;
}

// sync_moe_subspace_cache and scatter_and_restore_ffn_subspace: `sub` is
// null for the former.
int subspace_rows(moe_ctx* ctx, const void* sub, void* cache, void* out, const int64_t* active_idx,
                  const int64_t* keep, int64_t B, int64_t len, int64_t dim, int64_t elem_bytes) {
    TRY(begin(ctx));
    if (!cache || !out || (len > 0 && !keep)) return fail(ctx, MOE_E_ARG, "null pointer");
    if (elem_bytes != 2 && elem_bytes != 4) return fail(ctx, MOE_E_ARG, "elem_bytes must be 2 (fp16) or 4 (fp32)");
    if (B <= 0 || dim <= 0) return MOE_OK;  // the reference returns at once
    if (len < 0 || len > B) return fail(ctx, MOE_E_SHAPE, "ffn_active_len must be in [0, B]");
    int64_t nc;
    TRY(canvas_rows(ctx, active_idx, B, &nc));
    const int64_t rb = dim * elem_bytes;
    TRY(ws_reserve(ctx, al(B * 4) + al(B * 8) + al(len * 8) + al(len * rb) + al(B * rb) + al(nc * rb)));
    void *m = ws_take(ctx, B * 4), *ai = nullptr, *kp = nullptr, *sp = nullptr, *cp, *op;
    TRY(dev_ptr(ctx, active_idx, B * 8, K_IN, &ai));
    if (len > 0) TRY(dev_ptr(ctx, keep, len * 8, K_IN, &kp));
    if (sub && len > 0) TRY(dev_ptr(ctx, sub, len * rb, K_IN, &sp));
    TRY(dev_ptr(ctx, cache, nc * rb, K_INOUT, &cp));
    TRY(dev_ptr(ctx, out, B * rb, sub ? K_OUT : K_INOUT, &op));
    moe::SubspaceRowsArgs a;
    a.out = (uint8_t*)op;
    a.cache = (uint8_t*)cp;
    a.sub = sub ? (const uint8_t*)(sp ? sp : op) : nullptr;  // len 0: never read, but non-null selects the form
    a.active_idx = (const int64_t*)ai;
    a.map = (int*)m;
    a.B = B;
    a.row_bytes = rb;
    ctx->launches += moe::launch_subspace_rows(a, (const int64_t*)kp, len, ctx->stream);
    return finish(ctx);
}

}  // namespace

extern "C" {

int moe_router_subspace_ffn_filter(moe_ctx* ctx, const float* r_curr, float* r_prev, const int64_t* top_idx,
                                   int64_t* prev_top2, const uint8_t* eb_mask, const int64_t* active_canvas_idx,
                                   int64_t* ffn_keep_b, int64_t B, int64_t num_experts, int64_t top_k,
                                   int64_t step, float tau_ffn, float* top_weights, int64_t* active_count) {
    TRY(begin(ctx));
    if (!active_count) return fail(ctx, MOE_E_ARG, "null pointer");
    if (B <= 0) {  // the reference returns 0 at once
        const int64_t zero = 0;
        return put_small(ctx, active_count, &zero, 8);
    }
    if (!r_curr || !r_prev || !top_idx || !prev_top2 || !ffn_keep_b) return fail(ctx, MOE_E_ARG, "null pointer");
    if (num_experts < 0 || top_k < 1 || num_experts > (1 << 20) || top_k > 1024)
        return fail(ctx, MOE_E_SHAPE, "num_experts / top_k out of range");
    int64_t nc;
    TRY(canvas_rows(ctx, active_canvas_idx, B, &nc));
    const int64_t E = num_experts, K = top_k;
    TRY(ws_reserve(ctx, al(B * E * 4) + al(nc * E * 4) + al(B * K * 8) + al(nc * 16) + al(nc) + al(B * 8) * 2 +
                            al(B * K * 4) + al(8)));
    void *rc, *rp, *ti, *pt, *eb = nullptr, *ai = nullptr, *kb, *tw = nullptr;
    TRY(dev_ptr(ctx, r_curr, B * E * 4, K_IN, &rc));
    TRY(dev_ptr(ctx, r_prev, nc * E * 4, K_INOUT, &rp));
    TRY(dev_ptr(ctx, top_idx, B * K * 8, K_IN, &ti));
    TRY(dev_ptr(ctx, prev_top2, nc * 16, K_INOUT, &pt));
    if (eb_mask) TRY(dev_ptr(ctx, eb_mask, nc, K_IN, &eb));
    TRY(dev_ptr(ctx, active_canvas_idx, B * 8, K_IN, &ai));
    TRY(dev_ptr(ctx, ffn_keep_b, B * 8, K_INOUT, &kb));
    if (top_weights) TRY(dev_ptr(ctx, top_weights, B * K * 4, K_INOUT, &tw));
    int64_t* cnt = (int64_t*)ws_take(ctx, 8);
    moe::SubspaceFilterArgs a;
    a.r_curr = (const float*)rc;
    a.r_prev = (float*)rp;
    a.top_idx = (const int64_t*)ti;
    a.prev_top2 = (int64_t*)pt;
    a.eb_mask = (const uint8_t*)eb;
    a.active_idx = (const int64_t*)ai;
    a.keep_out = (int64_t*)kb;
    a.top_w = (float*)tw;
    a.count_out = cnt;
    a.B = B;
    a.E = (int)E;
    a.K = (int)K;
    a.step = step;
    a.tau = tau_ffn;
    ctx->launches += moe::launch_subspace_filter(a, ctx->stream);
    // the count is the reference's return value: the call completes here
    const int async = ctx->async_mode;
    ctx->async_mode = 0;
    const int st = finish(ctx);
    ctx->async_mode = async;
    TRY(st);
    int64_t n = 0;
    MOE_CUDA(cudaMemcpy(&n, cnt, 8, cudaMemcpyDeviceToHost));
    return put_small(ctx, active_count, &n, 8);
}

int moe_sync_moe_subspace_cache(moe_ctx* ctx, void* moe_out, void* moe_prev_cache,
                                const int64_t* active_canvas_idx, const int64_t* ffn_keep_b, int64_t B,
                                int64_t ffn_active_len, int64_t dim, int64_t elem_bytes) {
    return subspace_rows(ctx, nullptr, moe_prev_cache, moe_out, active_canvas_idx, ffn_keep_b, B, ffn_active_len,
                         dim, elem_bytes);
}

int moe_scatter_and_restore_ffn_subspace(moe_ctx* ctx, const void* ffn_sub_out, void* ffn_prev_cache,
                                         void* ffn_full_out, const int64_t* active_canvas_idx,
                                         const int64_t* ffn_keep_b, int64_t B, int64_t ffn_active_len, int64_t dim,
                                         int64_t elem_bytes) {
    if (ctx && !ffn_sub_out && ffn_active_len > 0) return fail(ctx, MOE_E_ARG, "null pointer");
    static const char kNone = 0;  // a non-null marker when no sub-batch row exists
    return subspace_rows(ctx, ffn_sub_out ? ffn_sub_out : &kNone, ffn_prev_cache, ffn_full_out, active_canvas_idx,
                         ffn_keep_b, B, ffn_active_len, dim, elem_bytes);
}

int moe_device_wait_check(moe_ctx* ctx) {
    TRY(begin(ctx));
    ctx->launches += moe::launch_wait_check(ctx->err_flag, ctx->device_timeout_ns, ctx->stream);
    const int async = ctx->async_mode;
    ctx->async_mode = 0;
    const int st = finish(ctx);
    ctx->async_mode = async;
    return st;
}

// ------------------------------------------------------------ layer level
namespace {

struct LayerDev {
    const uint8_t* rp = nullptr;
    const float* rs = nullptr;
    const float* rf32 = nullptr;
    const float* bias = nullptr;
    const float* router_scale = nullptr;
    const float* pes = nullptr;
    const float* pre_w = nullptr;
    const float* post_w = nullptr;
    ExpertWeights w{};
};

int check_desc(moe_ctx* ctx, const moe_layer_desc* L) {
    if (!L) return fail(ctx, MOE_E_ARG, "null layer descriptor");
    TRY(check_q4_shape(ctx, L->embed_dim, 2 * L->expert_mlp_dim));
    TRY(check_q4_shape(ctx, L->expert_mlp_dim, L->embed_dim));
    if (L->embed_dim > 12288) return fail(ctx, MOE_E_SHAPE, "embed_dim must be <= 12288");
    if (L->num_experts <= 0 || L->num_experts > 1024) return fail(ctx, MOE_E_SHAPE, "num_experts must be in [1, 1024]");
    if (L->top_k <= 0 || L->top_k > 32 || L->top_k > L->num_experts)
        return fail(ctx, MOE_E_SHAPE, "top_k must be in [1, min(32, num_experts)]");
    if (L->activation < 0 || L->activation > 1) return fail(ctx, MOE_E_ARG, "bad activation");
    if (!(L->router_packed && L->router_scales) && !L->router_f32)
        return fail(ctx, MOE_E_ARG, "no router weights");
    if (!L->router_scale || !L->per_expert_scale || !L->pre_norm_w || !L->gate_up_packed ||
        !L->gate_up_scales || !L->down_packed || !L->down_scales)
        return fail(ctx, MOE_E_ARG, "null weight pointer in layer descriptor");
    return MOE_OK;
}

size_t layer_small_bytes(const moe_layer_desc* L) {
    const int64_t d = L->embed_dim, E = L->num_experts;
    return al(d * 4) * 3 + al(E * 4) * 2 + (L->router_f32 ? al(E * d * 4) : 0);
}

// `E_w`: experts the descriptor's expert arrays hold (-1: num_experts; an
// expert-parallel rank with MOE_OPT_EP_LOCAL_WEIGHTS holds only its own).
int layer_dev(moe_ctx* ctx, const moe_layer_desc* L, int flags, LayerDev* o, int64_t E_w = -1) {
    const int64_t d = L->embed_dim, E = L->num_experts, F = L->expert_mlp_dim;
    const int64_t Ew = E_w < 0 ? E : E_w;
    void* p;
    if (L->router_packed) {
        TRY(dev_ptr(ctx, L->router_packed, E * d / 2, K_W, &p));
        o->rp = (const uint8_t*)p;
        TRY(dev_ptr(ctx, L->router_scales, E * d / 32 * 4, K_W, &p));
        o->rs = (const float*)p;
        if (!al16(o->rp)) return fail(ctx, MOE_E_ARG, "router weights must be 16-byte aligned");
    } else {
        TRY(dev_ptr(ctx, L->router_f32, E * d * 4, K_IN, &p));
        o->rf32 = (const float*)p;
    }
    if (L->router_logit_bias) {
        TRY(dev_ptr(ctx, L->router_logit_bias, E * 4, K_IN, &p));
        o->bias = (const float*)p;
    }
    TRY(dev_ptr(ctx, L->router_scale, d * 4, K_IN, &p));
    o->router_scale = (const float*)p;
    TRY(dev_ptr(ctx, L->per_expert_scale, E * 4, K_IN, &p));
    o->pes = (const float*)p;
    TRY(dev_ptr(ctx, L->pre_norm_w, d * 4, K_IN, &p));
    o->pre_w = (const float*)p;
    if (flags & MOE_F_POST_NORM) {
        if (!L->post_norm_w) return fail(ctx, MOE_E_ARG, "MOE_F_POST_NORM needs post_norm_w");
        TRY(dev_ptr(ctx, L->post_norm_w, d * 4, K_IN, &p));
        o->post_w = (const float*)p;
    }
    TRY(dev_ptr(ctx, L->gate_up_packed, Ew * 2 * F * d / 2, K_W, &p));
    o->w.gu_p = (const uint8_t*)p;
    TRY(dev_ptr(ctx, L->gate_up_scales, Ew * 2 * F * d / 32 * 4, K_W, &p));
    o->w.gu_s = (const float*)p;
    TRY(dev_ptr(ctx, L->down_packed, Ew * d * F / 2, K_W, &p));
    o->w.dn_p = (const uint8_t*)p;
    TRY(dev_ptr(ctx, L->down_scales, Ew * d * F / 32 * 4, K_W, &p));
    o->w.dn_s = (const float*)p;
    if (!al16(o->w.gu_p) || !al16(o->w.dn_p)) return fail(ctx, MOE_E_ARG, "packed weights must be 16-byte aligned");
    return MOE_OK;
}

// Bytes route_dev takes from the workspace.
size_t route_bytes(int64_t M, int64_t d, int64_t E, int64_t K) {
    return al(M * K * 4) * 2 + al(M * d * 4) * 2 + al(M * d / 32 * 4) + al(M * E * 4) + dense_bytes(M, d, E) +
           al(M * E * 4 * (d / 128 + 1));  // router partial sums (few tokens)
}

// Router: prep (norms, router input, block sums) -> router GEMV -> softmax /
// top-k / LOD (or set-cover).  moe_in / moe_in_sum receive the expert input.
int route_dev(moe_ctx* ctx, const moe_layer_desc* L, const LayerDev& ld, int64_t M,
              const float* xd, int flags, float* moe_in, float* moe_in_sum, int* slot_expert,
              float* slot_weight, float* probs, int64_t* top_idx, float* top_val, int64_t* tc,
              int64_t* ti, float* tw, float* moe_in_q = nullptr) {
    const int64_t K = L->top_k, d = L->embed_dim, E = L->num_experts;
    int* ti32 = (int*)ws_take(ctx, M * K * 4);
    float* tv = (float*)ws_take(ctx, M * K * 4);
    float* scaled = (float*)ws_take(ctx, M * d * 4);
    float* scores = (float*)ws_take(ctx, M * E * 4);
    if (!moe_in) moe_in = (float*)ws_take(ctx, M * d * 4);
    if (!moe_in_sum) moe_in_sum = (float*)ws_take(ctx, M * d / 32 * 4);
    if (!tv || !scaled || !scores || !moe_in || !moe_in_sum)
        return fail(ctx, MOE_E_NOMEM, "workspace exhausted");
    cudaStream_t s = ctx->stream;
    moe::PrepArgs pa;
    pa.x = xd;
    pa.K = d;
    pa.norm = 1;
    pa.pre_w = ld.pre_w;
    pa.router_scale = ld.router_scale;
    pa.rsf = L->r_scale_factor;
    pa.out = moe_in;
    pa.out_sum = moe_in_sum;
    pa.out_q = moe_in_q;
    pa.scaled = scaled;
    {
        ProfScope ps(ctx, "prep");
        ctx->launches += moe::launch_prep(pa, M, s);
    }
    float* part = nullptr;
    int part_n = 0;
    if (ld.rp && M >= ctx->router_tc_min_tokens && ctx->gemm_path != MOE_PATH_GEMV) {
        TRY(dense_q4(ctx, ld.rp, ld.rs, scaled, scores, d, E, M, "router", true));
    } else if (ld.rp && moe::router_part_supported((int)M, (int)d)) {
        // few tokens: fp32 partial sums over 128-wide K slices, added by k_topk
        part_n = (int)(d / 128);
        part = (float*)ws_take(ctx, (size_t)part_n * M * E * 4);
        if (!part) return fail(ctx, MOE_E_NOMEM, "workspace exhausted");
        ProfScope ps(ctx, "router");
        ctx->launches += moe::launch_router_part(ld.rp, ld.rs, scaled, (int)M, (int)d, (int)E, part, s);
    } else if (ld.rp) {  // fp32 router: routing follows the reference's arithmetic
        ProfScope ps(ctx, "router");
        ctx->launches += moe::launch_gemv_wide(ld.rp, ld.rs, scaled, scores, E, (int)d, (int)M, E, s);
    } else {
        ProfScope ps(ctx, "router");
        ctx->launches += moe::launch_gemv_f32(ld.rf32, scaled, scores, M, E, d, s);
    }
    moe::TopkArgs a;
    a.scores = scores;
    a.part = part;
    a.part_n = part_n;
    a.M = (int)M;
    a.bias = ld.bias;
    a.E = (int)E;
    a.K = (int)K;
    a.pes = ld.pes;
    a.top_p = L->moe_top_p;
    a.lod = (flags & MOE_F_SET_COVER) ? 0 : 1;
    a.probs_out = probs;
    a.top_idx = top_idx;
    a.top_val = top_val;
    a.ti32 = ti32;
    a.tv = tv;
    a.slot_expert = slot_expert;
    a.slot_weight = slot_weight;
    a.tok_count = tc;
    a.tok_idx = ti;
    a.tok_w = tw;
    {
        ProfScope ps(ctx, "topk");
        ctx->launches += moe::launch_topk(a, M, s);
    }
    if (flags & MOE_F_SET_COVER)
        ctx->launches += moe::launch_set_cover(ti32, tv, M, (int)K, (int)E, ld.pes, L->moe_top_p,
                                               0.85f, 0.068f, 5, slot_expert, slot_weight, tc, ti,
                                               tw, s);
    return MOE_OK;
}

// ---------------------------------------------------------------- expert
// parallelism: the gather and all-to-all forms of moe_layer_forward.

// The local expert slice [e_lo, e_lo + El) of the descriptor's weights.
ExpertWeights local_weights(moe_ctx* ctx, const ExpertWeights& w, int64_t e_lo, int64_t d, int64_t F) {
    if (ctx->ep_local_weights) return w;
    ExpertWeights o = w;
    o.gu_p += e_lo * 2 * F * d / 2;
    o.gu_s += e_lo * 2 * F * d / 32;
    o.dn_p += e_lo * d * F / 2;
    o.dn_s += e_lo * d * F / 32;
    return o;
}

// The context's expert-range options are cleared for the call (the expert
// kernels see the local slice as experts 0 .. El-1) and come back on exit.
struct ClearRange {
    moe_ctx* c;
    int64_t b, e;
    explicit ClearRange(moe_ctx* ctx_) : c(ctx_), b(ctx_->expert_begin), e(ctx_->expert_end) {
        c->expert_begin = 0;
        c->expert_end = 0;
    }
    ~ClearRange() {
        c->expert_begin = b;
        c->expert_end = e;
    }
};

int post_norm_rows(moe_ctx* ctx, float* od, const float* post_w, int64_t M, int64_t d) {
    moe::PrepArgs pa;
    pa.x = od;
    pa.K = d;
    pa.norm = 1;
    pa.pre_w = post_w;
    pa.out = od;
    ProfScope ps(ctx, "rms_norm");
    ctx->launches += moe::launch_prep(pa, M, ctx->stream);
    return MOE_OK;
}

// Gather form (decode): every rank passes its own M tokens (the same M on
// every rank).  The tokens of all ranks are gathered, routed, and this
// rank's experts evaluated for all of them; the partial outputs are summed
// by a reduce-scatter that leaves each rank its own M rows, then the
// post-norm.  No host synchronisation inside.
int ep_gather_forward(moe_ctx* ctx, const moe_layer_desc* L, int64_t M, const float* x, void* out, int flags,
                      int64_t* tc, int64_t* ti, float* tw) {
    const int N = ctx->ep.nranks, r = ctx->ep.rank;
    const int64_t d = L->embed_dim, E = L->num_experts, K = L->top_k, F = L->expert_mlp_dim;
    const int64_t El = E / N, e_lo = r * El, Mt = M * N, Pt = Mt * K;
    cudaStream_t s = ctx->stream;
    TRY(ws_reserve(ctx, layer_small_bytes(L) + expert_bufs_bytes(Mt, K, d, F, El) + route_bytes(Mt, d, E, K) +
                            al(M * d * 4) * 2 + al(Mt * d * 4) * 2 + al(Mt * 8) + al(Pt * 8) + al(Pt * 4) +
                            al(M * 8) + al(M * K * 8) + al(M * K * 4) + al(M * d * 4) + al(M * d / 32 * 4) +
                            al(M * K * 4) * 2));
    LayerDev ld;
    TRY(layer_dev(ctx, L, flags, &ld, ctx->ep_local_weights ? El : E));
    void *xd, *od, *dtc = nullptr, *dti = nullptr, *dtw = nullptr;
    TRY(dev_ptr(ctx, x, M * d * 4, K_IN, &xd));
    TRY(dev_ptr(ctx, out, M * d * 4, K_OUT, &od));
    if (tc) TRY(dev_ptr(ctx, tc, M * 8, K_OUT, &dtc));
    if (ti) TRY(dev_ptr(ctx, ti, M * K * 8, K_OUT, &dti));
    if (tw) TRY(dev_ptr(ctx, tw, M * K * 4, K_OUT, &dtw));
    float* x_all = (float*)ws_take(ctx, Mt * d * 4);
    float* part = (float*)ws_take(ctx, Mt * d * 4);
    int64_t* tc_all = (int64_t*)ws_take(ctx, Mt * 8);
    int64_t* ti_all = (int64_t*)ws_take(ctx, Pt * 8);
    float* tw_all = (float*)ws_take(ctx, Pt * 4);
    ExpertBufs bb;
    TRY(take_expert_bufs(ctx, Mt, K, d, F, El, &bb));
    if (!tw_all) return fail(ctx, MOE_E_NOMEM, "workspace exhausted");
    const ExpertWeights wl = local_weights(ctx, ld.w, e_lo, d, F);
    std::string err;
    int st;
    const bool cc = !use_tc(ctx, Mt, d, F, wl);
    if (!cc) {
        // Each rank routes its own M tokens, then the routed expert inputs and
        // slot tables are gathered (one NCCL group): routing all N * M tokens
        // on every rank took 66 us per step at 8 ranks (the wide router).
        float* x32_own = (float*)ws_take(ctx, M * d * 4);
        float* xsum_own = (float*)ws_take(ctx, M * d / 32 * 4);
        int* se_own = (int*)ws_take(ctx, M * K * 4);
        float* sw_own = (float*)ws_take(ctx, M * K * 4);
        if (!sw_own) return fail(ctx, MOE_E_NOMEM, "workspace exhausted");
        TRY(route_dev(ctx, L, ld, M, (const float*)xd, flags, x32_own, xsum_own, se_own, sw_own, nullptr, nullptr,
                      nullptr, (int64_t*)dtc, (int64_t*)dti, (float*)dtw));
        const moe::EpGatherBuf g[3] = {{x32_own, bb.x32, (size_t)(M * d), true},
                                       {se_own, bb.slot_expert, (size_t)(M * K), false},
                                       {sw_own, bb.slot_weight, (size_t)(M * K), true}};
        st = moe::ep_all_gather_n(ctx->ep, g, 3, s, ctx->ep_timeout_ns, err);
        if (st != MOE_OK) return fail(ctx, st, err);
        bb.x32q_ready = false;
    } else {
        // the CUDA-core expert path (a few tokens in all) needs the q-layout
        // input the router's prep writes: gather the tokens and route them all
        st = moe::ep_all_gather(ctx->ep, xd, x_all, (size_t)(M * d), true, s, ctx->ep_timeout_ns, err);
        if (st != MOE_OK) return fail(ctx, st, err);
        TRY(route_dev(ctx, L, ld, Mt, x_all, flags, bb.x32, bb.xsum, bb.slot_expert, bb.slot_weight, nullptr,
                      nullptr, nullptr, tc_all, ti_all, tw_all, bb.x32q));
        bb.x32q_ready = true;
        // this rank's rows of the routing outputs
        if (dtc) MOE_CUDA(cudaMemcpyAsync(dtc, tc_all + r * M, M * 8, cudaMemcpyDeviceToDevice, s));
        if (dti) MOE_CUDA(cudaMemcpyAsync(dti, ti_all + r * M * K, M * K * 8, cudaMemcpyDeviceToDevice, s));
        if (dtw) MOE_CUDA(cudaMemcpyAsync(dtw, tw_all + r * M * K, M * K * 4, cudaMemcpyDeviceToDevice, s));
    }
    ctx->launches += moe::launch_ep_localize(bb.slot_expert, Pt, (int)e_lo, (int)(e_lo + El), s);
    moe::CombineArgs c;
    {
        ClearRange cr(ctx);
        TRY(run_experts(ctx, wl, Mt, K, d, F, El, L->activation, bb, &c, part));
    }
    st = moe::ep_reduce_scatter(ctx->ep, part, (float*)od, (size_t)(M * d), s, ctx->ep_timeout_ns, err);
    if (st != MOE_OK) return fail(ctx, st, err);
    if (flags & MOE_F_POST_NORM) TRY(post_norm_rows(ctx, (float*)od, ld.post_w, M, d));
    return finish(ctx);
}

// All-to-all form (prefill): every rank passes its own M tokens (M may
// differ between ranks, 0 included).  Each rank routes its tokens; the
// routed (token, expert) pairs, sorted by expert and so grouped by the rank
// that owns the expert, travel as fp32 rows to that rank, which evaluates
// them on its experts; the results travel back in the same order and the
// home rank adds each token's slots in slot order and applies the post-norm.
// The row counts are exchanged first and read on the host (one wait per
// call) to size the exchange.
int ep_a2a_forward(moe_ctx* ctx, const moe_layer_desc* L, int64_t M, const float* x, void* out, int flags,
                   int64_t* tc, int64_t* ti, float* tw) {
    const int N = ctx->ep.nranks, r = ctx->ep.rank;
    const int64_t d = L->embed_dim, E = L->num_experts, K = L->top_k, F = L->expert_mlp_dim;
    const int64_t El = E / N, e_lo = r * El, Mh = std::max<int64_t>(M, 1), P = Mh * K;
    cudaStream_t s = ctx->stream;
    TRY(ws_reserve(ctx, layer_small_bytes(L) + expert_bufs_bytes(Mh, K, d, F, E) + route_bytes(Mh, d, E, K) +
                            al(M * d * 4) * 2 + al(M * 8) + al(M * K * 8) + al(M * K * 4) + al(P * d * 4) * 2 +
                            al(P * 4) + al(N * 4) + al((size_t)N * N * 4)));
    LayerDev ld;
    TRY(layer_dev(ctx, L, flags, &ld, ctx->ep_local_weights ? El : E));
    void *xd = nullptr, *od = nullptr, *dtc = nullptr, *dti = nullptr, *dtw = nullptr;
    if (M > 0) {
        TRY(dev_ptr(ctx, x, M * d * 4, K_IN, &xd));
        TRY(dev_ptr(ctx, out, M * d * 4, K_OUT, &od));
        if (tc) TRY(dev_ptr(ctx, tc, M * 8, K_OUT, &dtc));
        if (ti) TRY(dev_ptr(ctx, ti, M * K * 8, K_OUT, &dti));
        if (tw) TRY(dev_ptr(ctx, tw, M * K * 4, K_OUT, &dtw));
    }
    ExpertBufs bb;
    TRY(take_expert_bufs(ctx, Mh, K, d, F, E, &bb));
    float* send_x = (float*)ws_take(ctx, P * d * 4);
    float* y_back = (float*)ws_take(ctx, P * d * 4);
    int* send_e = (int*)ws_take(ctx, P * 4);
    int* send_cnt = (int*)ws_take(ctx, N * 4);
    int* all_cnt = (int*)ws_take(ctx, (size_t)N * N * 4);
    if (!all_cnt) return fail(ctx, MOE_E_NOMEM, "workspace exhausted");
    if (M > 0) {
        TRY(route_dev(ctx, L, ld, M, (const float*)xd, flags, bb.x32, bb.xsum, bb.slot_expert, bb.slot_weight,
                      nullptr, nullptr, nullptr, (int64_t*)dtc, (int64_t*)dti, (float*)dtw));
        ProfScope ps(ctx, "ep_dispatch");
        ctx->launches += moe::launch_bucket(bb.slot_expert, M * K, (int)K, (int)E, 0, (int)E, bb.b, s);
        ctx->launches += moe::launch_ep_pack(bb.b, (int)El, N, send_e, send_cnt, s);
        ctx->launches += moe::launch_gather_rows(bb.x32, bb.b.pair_token, bb.b.meta + 1, M * K, d, send_x, s);
    } else {
        MOE_CUDA(cudaMemsetAsync(send_cnt, 0, N * 4, s));
    }
    std::string err;
    int st = moe::ep_all_gather(ctx->ep, send_cnt, all_cnt, (size_t)N, false, s, ctx->ep_timeout_ns, err);
    if (st != MOE_OK) return fail(ctx, st, err);
    if (ctx->ep_host_n < N * N) {
        if (ctx->ep_host_cnt) cudaFreeHost(ctx->ep_host_cnt);
        ctx->ep_host_cnt = nullptr;
        ctx->ep_host_n = 0;
        if (cudaMallocHost(&ctx->ep_host_cnt, (size_t)N * N * 4) != cudaSuccess) {
            cudaGetLastError();
            return fail(ctx, MOE_E_NOMEM, "pinned count buffer");
        }
        ctx->ep_host_n = N * N;
    }
    MOE_CUDA(cudaMemcpyAsync(ctx->ep_host_cnt, all_cnt, (size_t)N * N * 4, cudaMemcpyDeviceToHost, s));
    MOE_CUDA(cudaEventRecord(ctx->done, s));
    st = moe::ep_wait(ctx->ep, ctx->done, ctx->ep_timeout_ns, true, err);
    if (st != MOE_OK) return fail(ctx, st, err);
    // row counts: this rank sends cnt[r][j] rows to j and receives cnt[j][r] from j
    std::vector<int64_t> sc(N), rc(N), so(N + 1, 0), ro(N + 1, 0);
    for (int j = 0; j < N; ++j) {
        sc[j] = ctx->ep_host_cnt[r * N + j];
        rc[j] = ctx->ep_host_cnt[j * N + r];
        if (sc[j] < 0 || rc[j] < 0) return fail(ctx, MOE_E_STATE, "bad row count in the exchange");
        so[j + 1] = so[j] + sc[j];
        ro[j + 1] = ro[j] + rc[j];
    }
    const int64_t Pr = ro[N];
    if (so[N] > (M > 0 ? M * K : 0)) return fail(ctx, MOE_E_STATE, "row counts disagree with the routing");
    // receive side: its own arena, sized now that the counts are known (the
    // stream is idle here)
    const int64_t Prh = std::max<int64_t>(Pr, 1);
    const size_t need = al(Prh * d * 4) * 2 + al(Prh * 4) + expert_bufs_bytes(Prh, 1, d, F, El) + 64 * kAlign;
    if (need > ctx->ep_cap) {
        if (ctx->ep_ws) cudaFree(ctx->ep_ws);
        ctx->ep_ws = nullptr;
        ctx->ep_cap = 0;
        const size_t cap = std::max(need, need + need / 2);
        if (cudaMalloc(&ctx->ep_ws, cap) != cudaSuccess) {
            cudaGetLastError();
            return fail(ctx, MOE_E_NOMEM, "expert-parallel receive arena");
        }
        ctx->ep_cap = cap;
    }
    size_t off = 0;
    auto take = [&](size_t b) -> void* {
        size_t o = (off + kAlign - 1) / kAlign * kAlign;
        if (o + b > ctx->ep_cap) return nullptr;
        off = o + b;
        return ctx->ep_ws + o;
    };
    float* recv_x = (float*)take(Prh * d * 4);
    float* y2 = (float*)take(Prh * d * 4);
    int* recv_e = (int*)take(Prh * 4);
    ExpertBufs b2;
    if (!carve_expert_bufs(take, Prh, 1, d, F, El, &b2) || !recv_e)
        return fail(ctx, MOE_E_NOMEM, "expert-parallel receive arena exhausted");
    std::vector<moe::EpXfer> xf;
    for (int j = 0; j < N; ++j) {
        xf.push_back({true, send_x + so[j] * d, (size_t)(sc[j] * d), true, j});
        xf.push_back({true, send_e + so[j], (size_t)sc[j], false, j});
        xf.push_back({false, recv_x + ro[j] * d, (size_t)(rc[j] * d), true, j});
        xf.push_back({false, recv_e + ro[j], (size_t)rc[j], false, j});
    }
    st = moe::ep_exchange(ctx->ep, xf, s, ctx->ep_timeout_ns, err);
    if (st != MOE_OK) return fail(ctx, st, err);
    if (Pr > 0) {
        const ExpertWeights wl = local_weights(ctx, ld.w, e_lo, d, F);
        ctx->launches += moe::launch_ep_slots(recv_e, Pr, (int)El, b2.slot_expert, b2.slot_weight, ctx->err_flag, s);
        TRY(prep_rows(ctx, recv_x, MOE_X_NATURAL, 0, Pr, d, b2.x32, b2.xsum));
        moe::CombineArgs c0;  // one slot of weight 1 per row: the expert output itself
        ClearRange cr(ctx);
        TRY(run_experts(ctx, wl, Pr, 1, d, F, El, L->activation, b2, &c0, y2));
    }
    xf.clear();
    for (int j = 0; j < N; ++j) {
        xf.push_back({true, y2 + ro[j] * d, (size_t)(rc[j] * d), true, j});
        xf.push_back({false, y_back + so[j] * d, (size_t)(sc[j] * d), true, j});
    }
    st = moe::ep_exchange(ctx->ep, xf, s, ctx->ep_timeout_ns, err);
    if (st != MOE_OK) return fail(ctx, st, err);
    if (M > 0) {
        moe::CombineArgs c;
        c.post_norm = (flags & MOE_F_POST_NORM) ? 1 : 0;
        c.post_w = ld.post_w;
        c.y = y_back;
        c.d = d;
        c.K = (int)K;
        c.slot_pair = bb.b.slot_pair;
        c.slot_weight = bb.slot_weight;
        c.out = od;
        ProfScope ps(ctx, "combine");
        ctx->launches += moe::launch_combine(c, M, s);
    }
    return finish(ctx);
}

}  // namespace

int moe_route(moe_ctx* ctx, const moe_layer_desc* L, int64_t M, const float* x, int flags,
              float* scores, int64_t* top_idx, float* top_val, int64_t* tc, int64_t* ti,
              float* tw, float* moe_in) {
    TRY(begin(ctx));
    TRY(check_desc(ctx, L));
    if (!x || !tc || !ti || !tw) return fail(ctx, MOE_E_ARG, "null pointer");
    if (M <= 0) return fail(ctx, MOE_E_SHAPE, "M must be >= 1");
    const int64_t d = L->embed_dim, E = L->num_experts, K = L->top_k, P = M * K;
    TRY(ws_reserve(ctx, layer_small_bytes(L) + route_bytes(M, d, E, K) + al(M * d * 4) * 2 +
                            al(M * E * 4) + al(P * 8) * 2 + al(P * 4) * 6 + al(M * 8)));
    LayerDev ld;
    TRY(layer_dev(ctx, L, flags & ~MOE_F_POST_NORM, &ld));
    void *xd, *sc = nullptr, *dti = nullptr, *dtv = nullptr, *dtc, *dtidx, *dtw, *mi = nullptr;
    TRY(dev_ptr(ctx, x, M * d * 4, K_IN, &xd));
    if (scores) TRY(dev_ptr(ctx, scores, M * E * 4, K_OUT, &sc));
    if (top_idx) TRY(dev_ptr(ctx, top_idx, P * 8, K_OUT, &dti));
    if (top_val) TRY(dev_ptr(ctx, top_val, P * 4, K_OUT, &dtv));
    TRY(dev_ptr(ctx, tc, M * 8, K_OUT, &dtc));
    TRY(dev_ptr(ctx, ti, P * 8, K_OUT, &dtidx));
    TRY(dev_ptr(ctx, tw, P * 4, K_OUT, &dtw));
    if (moe_in) TRY(dev_ptr(ctx, moe_in, M * d * 4, K_OUT, &mi));
    int* se = (int*)ws_take(ctx, P * 4);
    float* sw = (float*)ws_take(ctx, P * 4);
    TRY(route_dev(ctx, L, ld, M, (const float*)xd, flags, (float*)mi, nullptr, se, sw,
                  (float*)sc, (int64_t*)dti, (float*)dtv, (int64_t*)dtc, (int64_t*)dtidx,
                  (float*)dtw));
    return finish(ctx);
}

int moe_layer_forward(moe_ctx* ctx, const moe_layer_desc* L, int64_t M, const float* x, void* out,
                      int flags, int64_t* tc, int64_t* ti, float* tw) {
    TRY(begin(ctx));
    TRY(check_desc(ctx, L));
    const int64_t d = L->embed_dim, E = L->num_experts, K = L->top_k, F = L->expert_mlp_dim;
    // expert parallelism (moe_ep_init): this rank's experts for the call
    const bool ep = ctx->ep.comm != nullptr;
    const bool a2a = ep && ctx->ep_mode == MOE_EP_ALL_TO_ALL;
    if (M < 0 || (M == 0 && !a2a)) return fail(ctx, MOE_E_SHAPE, "M must be >= 1");
    if (M > 0 && (!x || !out)) return fail(ctx, MOE_E_ARG, "null pointer");
    if (ep) {
        if (flags & MOE_F_FP16_OUT)
            return fail(ctx, MOE_E_ARG, "expert parallelism sums fp32 partial outputs: MOE_F_FP16_OUT not supported");
        if (E < ctx->ep.nranks) return fail(ctx, MOE_E_SHAPE, "num_experts must be >= the number of ranks");
        if (ctx->ep_mode != MOE_EP_REPLICATED && E % ctx->ep.nranks != 0)
            return fail(ctx, MOE_E_SHAPE, "the gather and all-to-all forms need num_experts divisible by the ranks");
        if (ctx->ep_mode == MOE_EP_GATHER) return ep_gather_forward(ctx, L, M, x, out, flags, tc, ti, tw);
        if (a2a) return ep_a2a_forward(ctx, L, M, x, out, flags, tc, ti, tw);
    }
    struct RangeScope {  // the option values come back on every exit
        moe_ctx* c;
        int64_t b, e;
        RangeScope(moe_ctx* ctx_, bool on, int64_t E_) : c(ctx_), b(ctx_->expert_begin), e(ctx_->expert_end) {
            if (!on) return;
            c->expert_begin = (int64_t)c->ep.rank * E_ / c->ep.nranks;
            c->expert_end = (int64_t)(c->ep.rank + 1) * E_ / c->ep.nranks;
        }
        ~RangeScope() {
            c->expert_begin = b;
            c->expert_end = e;
        }
    } range_scope(ctx, ep, E);
    const int64_t P = M * K;
    const size_t out_bytes = M * d * ((flags & MOE_F_FP16_OUT) ? 2 : 4);
    TRY(ws_reserve(ctx, layer_small_bytes(L) + expert_bufs_bytes(M, K, d, F, E) +
                            route_bytes(M, d, E, K) + al(M * d * 4) + al(out_bytes) +
                            al(P * 4) * 2 + al(M * 8) + al(P * 8) + al(P * 4)));
    LayerDev ld;
    TRY(layer_dev(ctx, L, flags, &ld));
    void *xd, *od, *dtc = nullptr, *dti = nullptr, *dtw = nullptr;
    TRY(dev_ptr(ctx, x, M * d * 4, K_IN, &xd));
    TRY(dev_ptr(ctx, out, out_bytes, K_OUT, &od));
    if (tc) TRY(dev_ptr(ctx, tc, M * 8, K_OUT, &dtc));
    if (ti) TRY(dev_ptr(ctx, ti, P * 8, K_OUT, &dti));
    if (tw) TRY(dev_ptr(ctx, tw, P * 4, K_OUT, &dtw));
    ExpertBufs bb;
    TRY(take_expert_bufs(ctx, M, K, d, F, E, &bb));
    int C = 0;
    const bool rt = ctx->fused_route == 2 && ld.rp && !(flags & MOE_F_SET_COVER) &&
                    M < ctx->router_tc_min_tokens && al16(xd) && moe::route_rt_supported((int)M, (int)E, (int)K, (int)d);
    const bool fused = rt || (ctx->fused_route == 1 && ld.rp && !(flags & MOE_F_SET_COVER) &&
                              M < ctx->router_tc_min_tokens && al16(xd) &&
                              moe::route_fused_supported((int)M, (int)E, (int)K, (int)d, &C));
    if (rt) {
        // norms, router, top-k / LOD and buckets in one launch, then the gather
        const bool tc_path = use_tc(ctx, M, d, F, ld.w);
        const int nsl = (int)(d / 128);
        int* ti32 = (int*)ws_take(ctx, P * 4);
        float* tv = (float*)ws_take(ctx, P * 4);
        float* part = (float*)ws_take(ctx, (size_t)nsl * M * E * 4);
        if (!part) return fail(ctx, MOE_E_NOMEM, "workspace exhausted");
        moe::RouteRtArgs ra;
        ra.pa.x = xd;
        ra.pa.K = d;
        ra.pa.norm = 1;
        ra.pa.pre_w = ld.pre_w;
        ra.pa.router_scale = ld.router_scale;
        ra.pa.rsf = L->r_scale_factor;
        ra.pa.out = bb.x32;
        ra.pa.out_sum = bb.xsum;
        ra.pa.out_q = tc_path ? nullptr : bb.x32q;
        ra.rp = ld.rp;
        ra.rs = ld.rs;
        ra.ta.part = part;
        ra.ta.part_out = part;
        ra.ta.part_n = nsl;
        ra.ta.M = (int)M;
        ra.ta.bias = ld.bias;
        ra.ta.E = (int)E;
        ra.ta.K = (int)K;
        ra.ta.pes = ld.pes;
        ra.ta.top_p = L->moe_top_p;
        ra.ta.lod = 1;
        ra.ta.ti32 = ti32;
        ra.ta.tv = tv;
        ra.ta.slot_expert = bb.slot_expert;
        ra.ta.slot_weight = bb.slot_weight;
        ra.ta.tok_count = (int64_t*)dtc;
        ra.ta.tok_idx = (int64_t*)dti;
        ra.ta.tok_w = (float*)dtw;
        ra.b = bb.b;
        expert_range(ctx, E, &ra.e_lo, &ra.e_hi);
        ra.BN = tc_path ? expert_token_tile(P, E) : 0;
        ra.tt_prefix = tc_path ? bb.tt_prefix : nullptr;
        ra.ticket = ctx->route_ticket;
        int r;
        {
            ProfScope ps(ctx, "route");
            r = moe::launch_route_rt(ra, ctx->stream);
        }
        if (r < 0) return fail(ctx, MOE_E_CUDA, "routing launch failed");
        ctx->launches += r;
        if (tc_path) {
            ProfScope ps(ctx, "gather");
            ctx->launches += moe::launch_gather_f16(bb.x32, d, bb.b.pair_token, bb.b.meta, P, 0, bb.x16, ctx->stream);
        }
        bb.x32q_ready = !tc_path;
    } else if (fused) {
        const bool tc_path = use_tc(ctx, M, d, F, ld.w);
        moe::RouteFusedArgs ra;
        ra.x = (const float*)xd;
        ra.M = (int)M;
        ra.d = (int)d;
        ra.E = (int)E;
        ra.K = (int)K;
        ra.C = C;
        ra.rp = ld.rp;
        ra.rs = ld.rs;
        ra.rscale = ld.router_scale;
        ra.rsf = L->r_scale_factor;
        ra.pre_w = ld.pre_w;
        ra.bias = ld.bias;
        ra.pes = ld.pes;
        ra.top_p = L->moe_top_p;
        expert_range(ctx, E, &ra.e_lo, &ra.e_hi);
        ra.BN = tc_path ? expert_token_tile(P, E) : 0;
        ra.x32 = bb.x32;
        ra.xsum = bb.xsum;
        ra.x16 = tc_path ? bb.x16 : nullptr;
        ra.slot_expert = bb.slot_expert;
        ra.slot_weight = bb.slot_weight;
        ra.tok_count = (int64_t*)dtc;
        ra.tok_idx = (int64_t*)dti;
        ra.tok_w = (float*)dtw;
        ra.b = bb.b;
        ra.tt_prefix = tc_path ? bb.tt_prefix : nullptr;
        int r;
        {
            ProfScope ps(ctx, "route_fused");
            r = moe::launch_route_fused(ra, ctx->stream);
        }
        if (r < 0) return fail(ctx, MOE_E_CUDA, "fused routing launch failed");
        ctx->launches += r;
    } else {
        // the CUDA-core expert kernels read the gate/up input in the q layout:
        // the router's prep writes it alongside
        const bool cc = !use_tc(ctx, M, d, F, ld.w);
        TRY(route_dev(ctx, L, ld, M, (const float*)xd, flags, bb.x32, bb.xsum, bb.slot_expert,
                      bb.slot_weight, nullptr, nullptr, nullptr, (int64_t*)dtc, (int64_t*)dti,
                      (float*)dtw, cc ? bb.x32q : nullptr));
        bb.x32q_ready = cc;
    }
    moe::CombineArgs c;
    c.post_norm = (!ep && (flags & MOE_F_POST_NORM)) ? 1 : 0;
    c.post_w = ld.post_w;
    c.out_f16 = (flags & MOE_F_FP16_OUT) ? 1 : 0;
    TRY(run_experts(ctx, ld.w, M, K, d, F, E, L->activation, bb, &c, od, fused));
    if (ep) {
        // sum of the ranks' partial outputs, then the post-norm of the sum
        std::string err;
        const int st = moe::ep_all_reduce(ctx->ep, (float*)od, (size_t)(M * d), ctx->stream, ctx->ep_timeout_ns, err);
        if (st != MOE_OK) return fail(ctx, st, err);
        if (flags & MOE_F_POST_NORM) {
            moe::PrepArgs pa;
            pa.x = od;
            pa.K = d;
            pa.norm = 1;
            pa.pre_w = ld.post_w;
            pa.out = (float*)od;
            ProfScope ps(ctx, "rms_norm");
            ctx->launches += moe::launch_prep(pa, M, ctx->stream);
        }
    }
    return finish(ctx);
}

int moe_ep_get_unique_id(uint8_t* id) {
    if (!id) return MOE_E_ARG;
    std::string err;
    const int st = moe::ep_unique_id(id, err);
    if (st != MOE_OK) std::fprintf(stderr, "moe_ep_get_unique_id: %s\n", err.c_str());
    return st;
}

int moe_ep_init(moe_ctx* ctx, const uint8_t* id, int rank, int nranks) {
    TRY(begin(ctx));
    if (!id) return fail(ctx, MOE_E_ARG, "null communicator id");
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail(ctx, MOE_E_ARG, "bad rank or rank count");
    if (ctx->ep.comm) return fail(ctx, MOE_E_STATE, "the context already has a communicator");
    std::string err;
    const int st = moe::ep_init(ctx->ep, id, rank, nranks, ctx->ep_timeout_ns, err);
    if (st != MOE_OK) return fail(ctx, st, err);
    return MOE_OK;
}

int moe_ep_finalize(moe_ctx* ctx) {
    TRY(begin(ctx));
    if (!ctx->ep.comm) return MOE_OK;
    std::string err;
    MOE_CUDA(cudaEventRecord(ctx->done, ctx->stream));
    const int st = moe::ep_wait(ctx->ep, ctx->done, ctx->ep_timeout_ns, true, err);
    if (st != MOE_OK) return fail(ctx, st, err);
    moe::ep_destroy(ctx->ep);
    return MOE_OK;
}

}  // extern "C"

// ======================================================================
// Dense Q4_0 matmul without allocation.
//
// moe_q4_matmul_batchN takes its fp16 activation copy and split-K partial
// sums from the context workspace, which grows with cudaMalloc when a call
// needs more than it holds, and it stages host buffers through the same
// workspace.  Some callers must not allocate during a call: a serving loop
// that hands out all of HBM to its own arenas when it starts (any later
// cudaMalloc fails or evicts), and a latency-bound decode loop, where
// cudaMalloc / cudaFree synchronise the device.  For them the variant below
// keeps its scratch in one static device array per device, of fixed size,
// created with the module; it makes no cudaMalloc, cudaFree or other
// allocating call.
namespace {

// Fixed scratch: the fp16 copy of the activations (batch * c_in * 2 bytes)
// and, when space is left, split-K partial sums.  No byte of it needs an
// initial value: every byte a call reads is written earlier in that call.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch on the current device; looked up once per
// device (with that device current) and cached.
int noalloc_scratch(moe_ctx* ctx, void** out) {
    *out = nullptr;
    if (ctx->device < 0 || ctx->device >= kMaxDevices) return fail(ctx, MOE_E_ARG, "device ordinal too large");
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    if (!g_noalloc_ptr[ctx->device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return fail(ctx, MOE_E_CUDA, std::string("cudaGetSymbolAddress of the static scratch failed: ") +
                                             cudaGetErrorString(e));
        }
        g_noalloc_ptr[ctx->device] = p;
    }
    *out = g_noalloc_ptr[ctx->device];
    return MOE_OK;
}

// Device address of p without staging: a device (or managed) pointer, or a
// host pointer inside a registered range.
int dev_only(moe_ctx* ctx, const void* p, size_t bytes, const char* what, void** out) {
    *out = nullptr;
    const char* c = static_cast<const char*>(p);
    for (const Reg& r : ctx->regs)
        if (c >= r.host && c < r.host + r.bytes) {
            if (c + bytes > r.host + r.bytes)
                return fail(ctx, MOE_E_ARG, std::string(what) + " runs past the end of its registered range");
            *out = r.dev + (c - r.host);
            return MOE_OK;
        }
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        at.type = cudaMemoryTypeUnregistered;
    }
    if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) {
        *out = at.devicePointer ? at.devicePointer : const_cast<void*>(p);
        return MOE_OK;
    }
    return fail(ctx, MOE_E_ARG,
                std::string(what) + " must be device memory or inside a registered range (this entry point "
                                    "does not stage host buffers)");
}

}  // namespace

extern "C" {

int moe_q4_matmul_batchN_noalloc(moe_ctx* ctx, int64_t batch, const uint8_t* W, const float* S,
                                 const float* x, float* out, int64_t c_in, int64_t c_out) {
    TRY(begin(ctx));
    if (!W || !S || !x || !out) return fail(ctx, MOE_E_ARG, "null pointer");
    TRY(check_q4_shape(ctx, c_in, c_out));
    if (batch <= 0) return fail(ctx, MOE_E_SHAPE, "batch_size must be >= 1");
    if (batch > (int64_t)(kNoAllocScratchBytes / 2) || batch * c_in * 2 > (int64_t)kNoAllocScratchBytes)
        return fail(ctx, MOE_E_SHAPE,
                    "batch_size * c_in * 2 bytes exceeds the no-alloc entry point's fixed scratch of 8 MiB "
                    "(use moe_q4_matmul_batchN)");
    void *w, *sc, *xd, *od, *scratch;
    TRY(dev_only(ctx, W, c_out * c_in / 2, "W_packed", &w));
    TRY(dev_only(ctx, S, c_out * c_in / 32 * 4, "scales", &sc));
    TRY(dev_only(ctx, x, batch * c_in * 4, "x_batch", &xd));
    TRY(dev_only(ctx, out, batch * c_out * 4, "out_batch", &od));
    if (!al16(w)) return fail(ctx, MOE_E_ARG, "packed weights must be 16-byte aligned");
    if (!al16(xd)) return fail(ctx, MOE_E_ARG, "x_batch must be 16-byte aligned");
    TRY(noalloc_scratch(ctx, &scratch));
    const bool tc = ctx->gemm_path != MOE_PATH_GEMV && moe::tc_supported(c_in, c_out, 0, 0) && al8(sc) &&
                    (ctx->gemm_path == MOE_PATH_TC || batch >= ctx->dense_tc_min_tokens);
    if (!tc) {
        ctx->launches += moe::launch_gemv_wide((const uint8_t*)w, (const float*)sc, (const float*)xd, (float*)od,
                                               c_out, (int)c_in, (int)batch, c_out, ctx->stream);
        return finish(ctx);
    }
    if (dense_one_launch_ok(ctx, w, sc, xd, c_in, c_out, batch)) {
        // the same kernel and split as moe_q4_matmul_batchN (the same bits);
        // it needs no scratch
        TRY(dense_one_launch(ctx, w, sc, xd, od, c_in, c_out, batch));
        return finish(ctx);
    }
    __half* x16 = static_cast<__half*>(scratch);
    const size_t x16_bytes = al(batch * c_in * 2);
    moe::TcLaunch t;
    t.a.Ws = (const float*)sc;
    t.a.K = (int)c_in;
    t.a.R = c_out;
    t.a.dense_tokens = (int)batch;
    t.a.y_out = (float*)od;
    t.a.y_stride = c_out;
    t.a.err_flag = ctx->err_flag;
    t.a.timeout_ns = ctx->device_timeout_ns;
    t.Wp = (const uint8_t*)w;
    t.total_rows = c_out;
    t.B = x16;
    t.b_rows = batch;
    int BN = 16;
    while (BN < 256 && BN < batch) BN *= 2;
    t.BN = BN;
    t.max_items = ((c_out + 127) / 128) * ((batch + BN - 1) / BN);
    t.a_in_smem = ctx->tc_a_in_smem;
    t.stream = ctx->tc_stream >= 2;
    // split-K partials go after the activation copy: the split count
    // moe_q4_matmul_batchN would choose (so both give the same bits), lowered
    // only when that many partial sums do not fit
    int ks = ctx->dense_ksplit > 0 ? (int)std::min<int64_t>(ctx->dense_ksplit, std::max<int64_t>(1, c_in / 256))
                                   : choose_ksplit(ctx, t.max_items, c_in);
    const size_t part_room = kNoAllocScratchBytes - x16_bytes;
    while (ks > 1 && (size_t)ks * batch * c_out * 4 > part_room) --ks;
    float* part = nullptr;
    if (ks > 1) {
        part = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) + x16_bytes);
        t.a.y_out = part;
        t.a.ksplit = ks;
        t.a.split_stride = batch * c_out;
        t.max_items *= ks;
    }
    ctx->launches += moe::launch_gather_f16((const float*)xd, c_in, nullptr, nullptr, batch, (int)batch, x16,
                                            ctx->stream);
    const int r = moe::launch_tc_gemm(moe::TC_PLAIN, t, ctx->num_sms, ctx->stream);
    if (r < 0) return fail(ctx, MOE_E_CUDA, "tensor-core GEMM setup failed");
    ctx->launches += r;
    if (ks > 1)
        ctx->launches += moe::launch_reduce_splits(part, batch * c_out, ks, (float*)od, batch * c_out, ctx->stream);
    return finish(ctx);
}

}  // extern "C"
