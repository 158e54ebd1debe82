/*
 * moe_b200.h -- C ABI of libmoe_b200.so, a B200 (sm_100a) implementation of
 * phildrip/llm-mojo's Q4_0 Mixture-of-Experts FFN hot path.
 *
 * Every compute entry point replaces one Mojo routine of the reference; the
 * comment above it cites that routine (file:line within the reference
 * project) and states where the arguments differ.  Conventions shared by all
 * entry points:
 *
 *  - Pointers are plain addresses.  A pointer may be (a) a device pointer,
 *    (b) a host pointer inside a range registered with moe_register_weights
 *    (it is translated to the HBM mirror of that range), or (c) for
 *    activations, routing arrays and outputs only, any other host pointer:
 *    the call copies it to the device and the results back.  Weight
 *    pointers of kind (c) are rejected with MOE_E_UNREGISTERED so that a
 *    forgotten registration never streams gigabytes over PCIe per call.
 *  - Index arrays are int64 (Mojo ``Int``).  Weights are the reference's
 *    packed Q4_0 layout: per row, K/2 bytes (byte j of block b holds element
 *    32b+2j in its low nibble and 32b+2j+1 in its high nibble) plus K/32
 *    fp32 scales; value = (nibble - 8) * scale.  K must be a multiple of 32.
 *  - Calls are synchronous unless moe_set_async(ctx, 1) was called; then
 *    they are enqueued on the context's stream and moe_wait() completes them.
 *    The context's own stream is a blocking stream, so its kernels run after
 *    earlier work on the legacy default stream; device buffers produced on
 *    any other stream need moe_set_stream() (or a caller-side sync) first.
 *  - Every call returns MOE_OK (0) or an MOE_E_* code; moe_last_error()
 *    gives the message.  There is no CPU fallback: a context can only be
 *    created on a CUDA device.
 *  - One context per host thread.
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct moe_ctx moe_ctx;

enum moe_status {
    MOE_OK = 0,
    MOE_E_ARG = 1,          /* null pointer or bad enum */
    MOE_E_SHAPE = 2,        /* dimension not supported (e.g. K % 32 != 0) */
    MOE_E_UNREGISTERED = 3, /* weight pointer is neither device memory nor registered */
    MOE_E_CUDA = 4,         /* CUDA runtime error */
    MOE_E_NCCL = 5,         /* collective error (expert parallel) */
    MOE_E_TIMEOUT = 6,      /* bounded wait expired (moe_wait, EP init, device wait) */
    MOE_E_NOMEM = 7,        /* device or pinned allocation failed */
    MOE_E_STATE = 8         /* call not valid in the context's current state */
};

enum moe_activation {
    MOE_ACT_SIGMOID1702 = 0, /* g * sigmoid(1.702 g) * u  (moe_kernels.mojo:438-442, the reference's form) */
    MOE_ACT_GELU_TANH = 1    /* 0.5 g (1 + tanh(0.79788456 (g + 0.044715 g^3))) * u */
};

/* layout of an activation input row of length K */
enum moe_x_layout {
    MOE_X_NATURAL = 0,      /* x[k] */
    MOE_X_DEINT_HALVES = 1, /* [x[0],x[2],...,x[K-2] | x[1],x[3],...]  per 32-block pairs, as
                               moe_kernels.mojo:96-101 (even half then odd half) */
    MOE_X_DEINT_BLOCK32 = 2 /* per 32-block: 16 even then 16 odd (diffusion_kernels.mojo:52-75) */
};

/* ----------------------------------------------------------- context */
int moe_ctx_create(int device, moe_ctx** out);
int moe_ctx_destroy(moe_ctx* ctx);
const char* moe_last_error(const moe_ctx* ctx);
/* Number of kernels this context has launched so far (evidence counter). */
uint64_t moe_kernel_launches(const moe_ctx* ctx);
/* Use the caller's CUDA stream (cudaStream_t) instead of the context's own. */
int moe_set_stream(moe_ctx* ctx, void* cuda_stream);
/* 1: calls return after enqueueing; 0 (default): calls complete before returning. */
int moe_set_async(moe_ctx* ctx, int async_mode);
/* Completes enqueued work.  Gives up with MOE_E_TIMEOUT after timeout_ns
 * (0 = wait without limit).  Modelled on enqueue_matmul/wait_matmul
 * (kfd_gpu.mojo:1216-1260), which raise after a bounded poll. */
int moe_wait(moe_ctx* ctx, uint64_t timeout_ns);

/* Context options (moe_set_option). */
enum moe_option {
    MOE_OPT_GEMM_PATH = 1,        /* value: moe_gemm_path */
    MOE_OPT_TC_MIN_TOKENS = 2,    /* auto path, expert GEMMs: tensor cores from this many tokens in
                                     the batch (default 2: a single token uses the CUDA-core GEMV) */
    MOE_OPT_DEVICE_TIMEOUT_NS = 3, /* deadline of every device-side wait (default 4 s) */
    MOE_OPT_DENSE_TC_MIN_TOKENS = 4, /* auto path, dense projections and router: tensor cores from this
                                        many tokens (default 2) */
    MOE_OPT_TC_A_IN_SMEM = 5,      /* 1: stage the dequantised weights in shared memory even for token
                                      tiles <= 64 (default 0: tensor memory) */
    MOE_OPT_ROUTER_TC_MIN_TOKENS = 6, /* router on tensor cores from this many tokens (default 2048;
                                        below it the router runs in fp32 like the reference) */
    MOE_OPT_TC_STREAM = 7,         /* streaming tensor-core kernel for token tiles <= 64 and
                                      K % 64 == 0: 0 never, 1 (default) expert GEMMs, 2 expert
                                      and dense GEMMs; else the general kernel */
    /* Expert parallelism: moe_layer_forward, moe_run_moe_coalesced_core and
       moe_run_diffusion_moe_experts_parallel evaluate only experts in
       [BEGIN, END) (END 0: all, the default).  Routing still covers all
       experts; a token's output is the sum over its local slots (sum the
       partial outputs across ranks, then moe_rms_norm for the post-norm).
       No counterpart in the reference (a single process). */
    MOE_OPT_EXPERT_BEGIN = 8,
    MOE_OPT_EXPERT_END = 9,
    MOE_OPT_FUSED_ROUTE = 10,      /* moe_layer_forward's routing of small batches (Q4_0 router, LOD
                                      routing): 0 the separate norm / router / top-k / bucket /
                                      gather kernels; 1 one thread-block cluster (<= 16 tokens);
                                      2 one launch for the norms, the router, top-k / LOD and the
                                      buckets (its last CTA routes every token), then the fp16
                                      gather; routing bit-identical to 0 (<= 64 tokens, <= 512
                                      experts) */
    MOE_OPT_DENSE_KSPLIT = 11,     /* dense tensor-core GEMMs: split K into this many partial sums
                                      (0, the default: enough work items for two per SM) */
    MOE_OPT_EP_TIMEOUT_NS = 12,    /* deadline of every host wait on the expert-parallel
                                      communicator (set-up, collectives; default 30 s) */
    MOE_OPT_EP_MODE = 13,          /* moe_ep_mode: how moe_layer_forward splits the layer over the
                                      ranks of the context's communicator (default REPLICATED) */
    MOE_OPT_EP_LOCAL_WEIGHTS = 14, /* 1: in the GATHER and ALL_TO_ALL modes the descriptor's expert
                                      arrays hold only this rank's experts (expert rank*E/N + i at
                                      index i); 0 (default): all E experts */
    MOE_OPT_GEMV_ONE_TOKEN = 15,   /* CUDA-core expert path when every expert has at most one token
                                      (one-token batches): 1 (default) one warp per weight row,
                                      rows streamed from HBM; 0 the ring-buffered GEMV.  Same
                                      results either way */
    MOE_OPT_DENSE_ONE_LAUNCH = 16  /* moe_q4_matmul_batchN on tensor cores for 1..16 tokens
                                      (c_in % 256 == 0, c_in <= 8192, c_out % 128 == 0): 1 (default)
                                      one kernel that converts the tokens to fp16 itself and adds
                                      its split-K partial sums in split order (the splits of a row
                                      tile are one thread block cluster); 0 the fp16 gather, the
                                      general GEMM and a reduction kernel */
};
/* Expert-parallel forms of moe_layer_forward (no counterpart in the
 * single-process reference; see moe_ep_init).  Rank r of N owns the experts
 * [r*E/N, (r+1)*E/N); GATHER and ALL_TO_ALL need E % N == 0. */
enum moe_ep_mode {
    MOE_EP_REPLICATED = 0, /* every rank passes the same M tokens and receives the whole output:
                              partial outputs are all-reduced (decode, M <= 64) */
    MOE_EP_GATHER = 1,     /* every rank passes its own M tokens (M equal on all ranks): tokens are
                              all-gathered, each rank evaluates its experts for all of them, and a
                              reduce-scatter returns each rank its own rows (decode batches; no host
                              synchronisation in the call) */
    MOE_EP_ALL_TO_ALL = 2  /* every rank passes its own M >= 0 tokens: routed (token, expert) rows
                              are sent, sorted by expert, to the expert's owner, evaluated there and
                              sent back; the home rank adds each token's slots in slot order
                              (prefill; the per-peer row counts are read on the host once per call) */
};
enum moe_gemm_path {
    MOE_PATH_AUTO = 0, /* CUDA-core GEMV for few tokens, tensor cores above the threshold */
    MOE_PATH_GEMV = 1, /* always the CUDA-core grouped GEMV (fp32 arithmetic) */
    MOE_PATH_TC = 2    /* always the tcgen05 grouped GEMM (fp16 operands, fp32 accumulate) */
};
int moe_set_option(moe_ctx* ctx, int option, int64_t value);

/* Per-kernel timing with CUDA events recorded on the launching stream
 * around each kernel of the path (off by default; the reference's
 * perf_counter phase accumulators, model_speculative_moe.mojo:732-734, are
 * its CPU counterpart).  Enabling clears the accumulators. */
int moe_profile_enable(moe_ctx* ctx, int on);
/* Completes outstanding work, then reports per kernel name (32-byte
 * NUL-terminated slots in `names`) the total device milliseconds and launch
 * count since moe_profile_enable.  *n_out receives the number of names. */
int moe_profile_read(moe_ctx* ctx, int n_max, char* names, double* total_ms, uint64_t* counts,
                     int* n_out);

/* Mirror a host weight blob (e.g. the whole gemma4_moe_weights_q4.bin
 * allocation, model_speculative_moe_batched.mojo:1347-1356) to HBM once.
 * Later calls may pass any host pointer inside [host_base, host_base+bytes). */
int moe_register_weights(moe_ctx* ctx, const void* host_base, size_t bytes);
int moe_unregister_weights(moe_ctx* ctx, const void* host_base);

/* ------------------------------------------------ Q4_0 kernels, one matrix */
/* quantize_fp32_to_q4_0 (moe_kernels.mojo:7-56; convert_gemma4_moe.py:9-35).
 * Bit-exact with the reference on every input without an exact .5 tie. */
int moe_quantize_fp32_to_q4_0(moe_ctx* ctx, const float* src, uint8_t* dst_packed,
                              float* dst_scales, int64_t num_elements);

/* rms_norm (model_speculative_moe_batched.mojo:857-879): out[m] = x[m] *
 * (1 / sqrt(mean(x[m]^2) + 1e-6)) * w, for M rows of d (d % 32 == 0).  Used
 * for the post-norm after partial expert outputs were summed across ranks. */
int moe_rms_norm(moe_ctx* ctx, const float* x, const float* w, float* out, int64_t M, int64_t d);

/* q4_matmul_vec (moe_kernels.mojo:59-67): out[c_out] = W[c_out x c_in] x[c_in]. */
int moe_q4_matmul_vec(moe_ctx* ctx, const uint8_t* W_packed, const float* scales,
                      const float* x, float* out, int64_t c_in, int64_t c_out);

/* q4_matmul_batchN (moe_kernels.mojo:254-264) and q4_matmul_batch5 (:165-174):
 * out[b*c_out + r] for b < batch_size.  Any batch_size >= 1 (the reference
 * limits it to 5). */
int moe_q4_matmul_batchN(moe_ctx* ctx, int64_t batch_size, const uint8_t* W_packed,
                         const float* scales, const float* x_batch, float* out_batch,
                         int64_t c_in, int64_t c_out);

/* moe_q4_matmul_batchN without any allocation during the call.  No
 * counterpart in the reference (its Mojo routines allocate nothing on a
 * device); this is for callers that must not allocate while they run: a
 * server that hands all of HBM to its own arenas at start-up, where a later
 * cudaMalloc fails, and latency-bound loops, where cudaMalloc/cudaFree would
 * synchronise the device.  Same arguments and results as
 * moe_q4_matmul_batchN, except:
 *  - scratch (the fp16 copy of x_batch and split-K partial sums) lives in
 *    one static device array of 8 MiB per device.  moe_ctx_create commits
 *    it when the first context on a device is created (it stays until the
 *    process exits), so no call of this entry point loads or allocates it;
 *    batch_size * c_in * 2 must be <= 8 MiB (8388608 bytes), else the call
 *    returns MOE_E_SHAPE and does nothing.  The scratch needs no initial
 *    value: every byte a call reads was written earlier in that call;
 *  - the split-K count is the one moe_q4_matmul_batchN picks (including
 *    MOE_OPT_DENSE_KSPLIT), so the results are the same bits; only when
 *    that many partial sums do not fit beside the fp16 copy is it lowered,
 *    and the results then differ by fp32 reassociation;
 *  - every pointer must be device memory or inside a registered range
 *    (MOE_E_ARG otherwise: host buffers are not staged), and x_batch and
 *    W_packed 16-byte aligned;
 *  - the scratch is shared by every context and stream on the device: two
 *    calls in flight at the same time on one device (different streams,
 *    contexts or threads) race on it.  Calls ordered on one stream do not. */
int moe_q4_matmul_batchN_noalloc(moe_ctx* ctx, int64_t batch_size, const uint8_t* W_packed,
                                 const float* scales, const float* x_batch, float* out_batch,
                                 int64_t c_in, int64_t c_out);

/* ------------------------------------------------------------- routing */
/* compute_moe_lod_weights (moe_kernels.mojo:445-490) for `batch` tokens laid
 * out back to back (top_k entries each).  active_count[b] receives the count
 * the reference returns. */
int moe_compute_moe_lod_weights(moe_ctx* ctx, int64_t batch, const int64_t* top_idx,
                                const float* top_val, const float* per_expert_scale,
                                float moe_top_p, int64_t* active_idx, float* active_weights,
                                int64_t* active_count, int64_t top_k);

/* apply_moe_lod_and_set_cover (diffusion_kernels.mojo:3607-3664).
 * eb_mask (uint8, 0/1) and active_canvas_idx may be NULL. */
int moe_apply_moe_lod_and_set_cover(moe_ctx* ctx, const int64_t* canvas_top_idx,
                                    const float* canvas_top_val,
                                    const float* router_per_expert_scale,
                                    float* canvas_top_weights, int64_t B, int64_t top_k_experts,
                                    int64_t active_top_k, float moe_top_p,
                                    const uint8_t* eb_mask, const int64_t* active_canvas_idx,
                                    int64_t unaccepted_top_k);

/* compute_subbatch_set_cover_moe_weights (moe_kernels.mojo:493-611). */
int moe_compute_subbatch_set_cover_moe_weights(
    moe_ctx* ctx, int64_t sub_b, const int64_t* all_top_idx, const float* all_top_val,
    const float* per_expert_scale, float moe_top_p, int64_t* tok_active_count,
    int64_t* tok_active_idx, float* tok_active_weights, int64_t num_experts, int64_t top_k,
    float core_top_p, float singleton_min_prob);

/* ------------------------------------------------------- expert stages */
/* run_moe_experts_stage1_8core (moe_kernels.mojo:614-627): for each active
 * slot s, gate_up_out_all[s*2F + r] = W_gu[e_s][r] . moe_in and
 * act_all[s*F + j] = act(g_j) * u_j.  gate_up_out_all may be NULL (it is
 * scratch for the reference's callers).  The reference's moe_in_deint
 * scratch argument is not needed. */
int moe_run_moe_experts_stage1(moe_ctx* ctx, const uint8_t* experts_gate_up_packed,
                               const float* experts_gate_up_scales, const float* moe_in,
                               const int64_t* active_idx, int64_t active_count,
                               float* gate_up_out_all, float* act_all, int64_t embed_dim,
                               int64_t expert_mlp_dim, int activation);

/* run_moe_experts_stage2_8core (moe_kernels.mojo:699-712): moe_out[r] =
 * sum_s active_weights[s] * (W_dn[e_s][r] . act_all[s]), slots in order. */
int moe_run_moe_experts_stage2(moe_ctx* ctx, const uint8_t* experts_down_packed,
                               const float* experts_down_scales, const float* act_all,
                               const int64_t* active_idx, const float* active_weights,
                               int64_t active_count, float* moe_out, int64_t embed_dim,
                               int64_t expert_mlp_dim);

/* run_moe_coalesced_core (moe_kernels.mojo:1321-1345): bucket-sorted expert
 * evaluation of sub_b tokens (any sub_b >= 1; the reference allows <= 5).
 * batch_in is in `x_layout` (the reference passes MOE_X_DEINT_HALVES).
 * tok_active_idx / weights have stride top_k (8 in the reference). */
int moe_run_moe_coalesced_core(moe_ctx* ctx, int64_t sub_b,
                               const uint8_t* experts_gate_up_packed,
                               const float* experts_gate_up_scales,
                               const uint8_t* experts_down_packed,
                               const float* experts_down_scales, const float* batch_in,
                               int x_layout, const int64_t* tok_active_count,
                               const int64_t* tok_active_idx, const float* tok_active_weights,
                               float* batch_moe_out, int64_t embed_dim, int64_t expert_mlp_dim,
                               int64_t num_experts, int64_t top_k, int activation);

/* run_moe_coalesced_stage1 (moe_kernels.mojo:784-1069) and
 * run_moe_coalesced_stage2 (:1072-1318): the core in two calls, so that a
 * caller can put other work between the gate/up half and the down half
 * (model_speculative_moe_batched.mojo:3165-3234).  Together they give the
 * same bits as moe_run_moe_coalesced_core on the same inputs.
 * Stage 1 fills the reference's buckets: bucket_counts[E], bucket_toks[E*5]
 * and bucket_weights[E*5] (token b and its weight at e*5 + c, in token then
 * slot order), unique_experts / unique_base_slot (ascending expert ids and
 * the prefix of their counts; *num_unique entries), and returns the count in
 * *num_unique.  These arrays are read on the host, so the call completes
 * before returning (also in asynchronous mode) as far as the routing
 * arrays go.  1 <= sub_b <= 5, as in the reference (five bucket entries per
 * expert).  The activations stay in device memory of the context, which
 * keeps one stage-1 result at a time, identified by `act_deint_scratch`
 * (its contents are not used); calls of other entry points in between do not
 * disturb it.  Stage 2 takes the down weights, evaluates the down half of
 * that result and writes the per-token weighted sums to batch_moe_out [sub_b
 * x d]; the bucket arguments are accepted for signature parity and not read.
 * MOE_E_STATE: no stage-1 result for that scratch pointer, or the options or
 * the down weights' alignment changed the expert path between the calls.
 * Summation order: stage 2 adds each token's expert outputs in the token's
 * slot order (as run_moe_experts_stage2_8core does, moe_kernels.mojo:775-779);
 * the reference's coalesced stage 2 zeroes the output and adds in ascending
 * expert order (:1095-1318).  The two orders differ only by fp32
 * reassociation of at most top_k terms per output element. */
int moe_run_moe_coalesced_stage1(moe_ctx* ctx, int64_t sub_b, const uint8_t* experts_gate_up_packed,
                                 const float* experts_gate_up_scales, const float* batch_in,
                                 int x_layout, const int64_t* tok_active_count,
                                 const int64_t* tok_active_idx, const float* tok_active_weights,
                                 int64_t* bucket_counts, int64_t* bucket_toks, float* bucket_weights,
                                 int64_t* unique_experts, int64_t* unique_base_slot,
                                 const float* act_deint_scratch, int64_t embed_dim,
                                 int64_t expert_mlp_dim, int64_t num_experts, int64_t top_k,
                                 int activation, int64_t* num_unique);
int moe_run_moe_coalesced_stage2(moe_ctx* ctx, int64_t sub_b, int64_t num_unique,
                                 const uint8_t* experts_down_packed, const float* experts_down_scales,
                                 const int64_t* bucket_counts, const int64_t* bucket_toks,
                                 const float* bucket_weights, const int64_t* unique_experts,
                                 const int64_t* unique_base_slot, const float* act_deint_scratch,
                                 float* batch_moe_out, int64_t embed_dim, int64_t expert_mlp_dim);

/* run_diffusion_moe_experts_parallel (diffusion_kernels.mojo:236-253): fp16
 * canvas in/out (IEEE binary16 bits), a slot is active iff its weight > 0,
 * per-token fp32 combine then one rounding to fp16.  The reference's three
 * preallocated scratch buffers are not needed. */
int moe_run_diffusion_moe_experts_parallel(moe_ctx* ctx, const uint8_t* experts_gate_up_packed,
                                           const float* experts_gate_up_scales,
                                           const uint8_t* experts_down_packed,
                                           const float* experts_down_scales,
                                           const uint16_t* canvas_moe_in,
                                           const int64_t* canvas_top_idx,
                                           const float* canvas_top_weights,
                                           uint16_t* canvas_moe_out, int64_t B,
                                           int64_t embed_dim, int64_t expert_mlp_dim,
                                           int64_t top_k_experts, int activation);

/* ------------------------------------- diffusion router-subspace FFN bypass */
/* router_subspace_ffn_filter (diffusion_kernels.mojo:2253-2337).  For each
 * canvas row b (canvas position o = active_canvas_idx[b], or b when it is
 * NULL): when step >= 1, the token is accepted (eb_mask[o] != 0, or eb_mask
 * NULL), top_k >= 2, its top-2 experts equal prev_top2[o] and the drift of
 * its router logits r_curr[b] from r_prev[o] is small (sum (c-p)^2 <=
 * tau_ffn^2 * sum p^2, or <= 1e-12 when sum p^2 <= 1e-12), the row is
 * bypassed: its top_weights row (if given) is zeroed.  Otherwise b is
 * appended to ffn_keep_b (ascending) and r_prev[o], prev_top2[o] take the
 * current values.  *active_count receives the reference's return value (the
 * number of kept rows); the call completes before returning, also in
 * asynchronous mode.  The drift sums are formed in the reference's 8-lane
 * order, so every decision is the reference's bit for bit.  r_curr [B x
 * num_experts], r_prev [canvas x num_experts] fp32; top_idx [B x top_k],
 * prev_top2 [canvas x 2] int64; eb_mask [canvas] uint8; ffn_keep_b [B].
 * The canvas positions of the B rows must be distinct. */
int moe_router_subspace_ffn_filter(moe_ctx* ctx, const float* r_curr, float* r_prev,
                                   const int64_t* top_idx, int64_t* prev_top2,
                                   const uint8_t* eb_mask, const int64_t* active_canvas_idx,
                                   int64_t* ffn_keep_b, int64_t B, int64_t num_experts,
                                   int64_t top_k, int64_t step, float tau_ffn,
                                   float* top_weights, int64_t* active_count);

/* sync_moe_subspace_cache (diffusion_kernels.mojo:2345-2381): rows of dim
 * elements of elem_bytes bytes (2: the reference's default fp16; 4: fp32).
 * Walking b in order with a cursor into ffn_keep_b[0, ffn_active_len), row b
 * of moe_out is saved to moe_prev_cache[o] when it is the cursor's entry
 * (evaluated), else restored from it (bypassed). */
int moe_sync_moe_subspace_cache(moe_ctx* ctx, void* moe_out, void* moe_prev_cache,
                                const int64_t* active_canvas_idx, const int64_t* ffn_keep_b,
                                int64_t B, int64_t ffn_active_len, int64_t dim,
                                int64_t elem_bytes);

/* scatter_and_restore_ffn_subspace (diffusion_kernels.mojo:2386-2426): as
 * the sync above, but an evaluated row comes from the compacted sub-batch
 * output ffn_sub_out[cursor] and goes to both ffn_full_out[b] and
 * ffn_prev_cache[o]; a bypassed row of ffn_full_out comes from the cache. */
int moe_scatter_and_restore_ffn_subspace(moe_ctx* ctx, const void* ffn_sub_out,
                                         void* ffn_prev_cache, void* ffn_full_out,
                                         const int64_t* active_canvas_idx,
                                         const int64_t* ffn_keep_b, int64_t B,
                                         int64_t ffn_active_len, int64_t dim,
                                         int64_t elem_bytes);

/* Check of the bounded device-side waits (no counterpart in the reference).
 * Every pipelined kernel of the library waits on shared-memory barriers
 * with a deadline of MOE_OPT_DEVICE_TIMEOUT_NS; when one passes, the kernel
 * stops, drains what it issued, raises the context's error word and the
 * call returns MOE_E_TIMEOUT.  This call launches one block that waits on a
 * barrier nothing completes, with the same wait code and the context's
 * deadline, so it returns MOE_E_TIMEOUT after about that deadline when the
 * mechanism works (never MOE_OK).  The context stays usable afterwards. */
int moe_device_wait_check(moe_ctx* ctx);

/* --------------------------------------------------------- whole layer */
enum moe_layer_flags {
    MOE_F_POST_NORM = 1, /* apply rms_norm(moe_out, post_norm_w) (model_speculative_moe_batched.mojo:1144-1150) */
    MOE_F_SET_COVER = 4, /* set-cover routing per sub-batch of 5 (:1060-1072) instead of LOD */
    MOE_F_FP16_OUT = 8   /* write the output as fp16 bits instead of fp32 */
};

typedef struct moe_layer_desc {
    int64_t embed_dim;      /* d, 2816 */
    int64_t expert_mlp_dim; /* F, 704 */
    int64_t num_experts;    /* E, 128 (<= 1024) */
    int64_t top_k;          /* 8 (<= 32) */
    int32_t activation;     /* moe_activation */
    float r_scale_factor;   /* 1/sqrt(d) (model_speculative_moe_batched.mojo:1868) */
    float moe_top_p;        /* 1.0 = lossless LOD (:1269) */
    const uint8_t* router_packed; /* Q4_0 router [E x d] (:155, :179) */
    const float* router_scales;
    const float* router_f32;      /* optional fp32 router [E x d], used when router_packed == NULL */
    const float* router_logit_bias; /* optional [E] added to router scores; NULL in the reference.
                                       Synthetic skewed-routing workloads only. */
    const float* router_scale;     /* [d] */
    const float* per_expert_scale; /* [E] */
    const float* pre_norm_w;       /* [d] pre_feedforward_layernorm_2 */
    const float* post_norm_w;      /* [d] post_feedforward_layernorm_2 (MOE_F_POST_NORM) */
    const uint8_t* gate_up_packed; /* [E][2F x d] */
    const float* gate_up_scales;
    const uint8_t* down_packed;    /* [E][d x F] */
    const float* down_scales;
} moe_layer_desc;

/* Router half of run_moe_coalesced_subbatch_stage1
 * (model_speculative_moe_batched.mojo:957-1083; decode block :2102-2118) for
 * M tokens: rms_norm_noscale(x) * router_scale * r_scale_factor -> Q4 router
 * -> softmax -> top-k -> LOD (or set-cover), and moe_in = rms_norm(x,
 * pre_norm_w).  Output pointers other than the three tok_active_* may be NULL. */
int moe_route(moe_ctx* ctx, const moe_layer_desc* L, int64_t M, const float* x, int flags,
              float* scores, int64_t* top_idx, float* top_val, int64_t* tok_active_count,
              int64_t* tok_active_idx, float* tok_active_weights, float* moe_in);

/* run_moe_coalesced_subbatch (model_speculative_moe_batched.mojo:1155-1204)
 * for any M: route, expert evaluation and (flag) the post-norm.  `out` is
 * fp32 [M x d] (fp16 bits with MOE_F_FP16_OUT).  The routing outputs may be
 * NULL. */
int moe_layer_forward(moe_ctx* ctx, const moe_layer_desc* L, int64_t M, const float* x,
                      void* out, int flags, int64_t* tok_active_count, int64_t* tok_active_idx,
                      float* tok_active_weights);

/* ------------------------------------------ weights file, straight to HBM */
/* The layer-blob file that convert_gemma4_moe.py:164-262 writes
 * (gemma4_moe_weights_q4.bin): per layer, Q4_0 packed bytes of ten matrices
 * in a fixed order, then their fp32 block scales in the same order, then
 * twelve fp32 vectors, zero-padded to a multiple of 4096 bytes; layers follow
 * each other with no header.  The reader's offsets are MoEConfig's
 * get_layer_aligned_size / get_layer_offset / get_layer_weights
 * (model_speculative_moe_batched.mojo:57-231).  The reference hard-codes the
 * attention shapes (16 heads; head_dim 256 and 8 kv heads on sliding layers,
 * 512 and 2 kv heads without v_proj on every sixth, global, layer); here they
 * are fields of the configuration, with the reference's values as defaults. */
typedef struct moe_model_config {
    int64_t embed_dim;        /* 2816 */
    int64_t standard_mlp_dim; /* 2112: the dense (shared) MLP */
    int64_t expert_mlp_dim;   /* 704 */
    int64_t num_experts;      /* 128 */
    int64_t top_k;            /* 8 (copied into layer descriptors) */
    int64_t num_layers;       /* 30 */
    int64_t num_heads;        /* 16 */
    int64_t head_dim_sliding, kv_heads_sliding; /* 256, 8 */
    int64_t head_dim_global, kv_heads_global;   /* 512, 2 */
    int64_t global_every;     /* 6: layer i is global when i % 6 == 5 (no v_proj) */
} moe_model_config;

/* The ten Q4_0 matrices of a layer, in file order. */
enum moe_weight_matrix {
    MOE_W_Q = 0, MOE_W_K, MOE_W_V, MOE_W_O, MOE_W_GATE, MOE_W_UP, MOE_W_DOWN, MOE_W_ROUTER,
    MOE_W_EXPERTS_GATE_UP, MOE_W_EXPERTS_DOWN, MOE_W_COUNT
};
/* The twelve fp32 vectors of a layer, in file order. */
enum moe_weight_vector {
    MOE_V_INPUT_LAYERNORM = 0, MOE_V_POST_ATTENTION_LAYERNORM, MOE_V_PRE_FEEDFORWARD_LAYERNORM,
    MOE_V_PRE_FEEDFORWARD_LAYERNORM_2, MOE_V_POST_FEEDFORWARD_LAYERNORM,
    MOE_V_POST_FEEDFORWARD_LAYERNORM_1, MOE_V_POST_FEEDFORWARD_LAYERNORM_2, MOE_V_Q_NORM,
    MOE_V_K_NORM, MOE_V_ROUTER_SCALE, MOE_V_ROUTER_PER_EXPERT_SCALE, MOE_V_LAYER_SCALAR,
    MOE_V_COUNT
};

typedef struct moe_layer_layout {
    int64_t layer_offset;  /* byte offset of the layer's blob in the file */
    int64_t layer_bytes;   /* blob size, a multiple of 4096 */
    int64_t payload_bytes; /* bytes before the zero padding */
    int64_t is_global;
    int64_t head_dim, kv_heads;
    /* matrix m is rows[m] x cols[m] (cols = the inner dimension K; the expert
       matrices stack all experts' rows: E*2F x d and E*d x F); rows 0 = absent */
    int64_t rows[MOE_W_COUNT], cols[MOE_W_COUNT];
    int64_t packed_offset[MOE_W_COUNT]; /* byte offsets within the blob */
    int64_t scales_offset[MOE_W_COUNT];
    int64_t vec_offset[MOE_V_COUNT];
    int64_t vec_len[MOE_V_COUNT];       /* fp32 elements */
} moe_layer_layout;

/* Fills *cfg with the reference's MoEConfig defaults (Gemma-4 26B-A4B). */
int moe_default_model_config(moe_model_config* cfg);
/* Layout of layer `layer` (0 <= layer < num_layers).  MOE_E_SHAPE when a
 * matrix's inner dimension is not a positive multiple of 32.  The
 * router_per_expert_scale vector has num_experts elements, as the converter
 * writes it (the reference reader reserves 128, the same for its model). */
int moe_weights_layout(const moe_model_config* cfg, int64_t layer, moe_layer_layout* out);
/* Size in bytes of the whole file (15311790080 for the defaults, the size
 * model_speculative_moe_batched.mojo:1347 hard-codes). */
int moe_weights_file_size(const moe_model_config* cfg, int64_t* bytes);
/* The MoE layer descriptor of layer `layer` of a file image that starts at
 * `weights_base` (device memory, or a registered host range), as
 * get_layer_weights (model_speculative_moe_batched.mojo:121-231) hands the
 * layer to run_moe_coalesced_subbatch: Q4_0 router, router_scale,
 * router_per_expert_scale, pre_feedforward_layernorm_2 as pre-norm,
 * post_feedforward_layernorm_2 as post-norm, the expert matrices;
 * activation MOE_ACT_SIGMOID1702, r_scale_factor 1/sqrt(d), moe_top_p 1.
 * Address arithmetic only: nothing is read. */
int moe_layer_desc_from_weights(const moe_model_config* cfg, const void* weights_base,
                                int64_t layer, moe_layer_desc* out);
/* Reads bytes [file_offset, file_offset + bytes) of the file at `path` into
 * device memory at `dst` (bytes < 0: to the end of the file), replacing the
 * reference's read of the whole file into host RAM
 * (model_speculative_moe_batched.mojo:1333-1380).  The file is read by
 * several host threads into pinned staging buffers while earlier chunks
 * copy to HBM on the context's stream.  Returns when the data is in place
 * (also in asynchronous mode); *bytes_loaded (may be NULL) receives the
 * count.  MOE_E_ARG: the file cannot be opened or read, or `dst` is not
 * device memory; MOE_E_SHAPE: the range runs past the end of the file. */
int moe_load_weights_file(moe_ctx* ctx, const char* path, int64_t file_offset, int64_t bytes,
                          void* dst, int64_t* bytes_loaded);

/* ------------------------------------------------ expert parallelism (NCCL) */
/* No counterpart in the reference (a single process on one machine); the
 * multi-GPU form of run_moe_coalesced_subbatch for a host that drives the
 * library through this ABI alone.  One process (and context) per GPU. */
#define MOE_EP_UNIQUE_ID_BYTES 128
/* Creates the communicator id on one rank; the host passes the 128 bytes to
 * every rank by its own means (a file, a socket, its launcher). */
int moe_ep_get_unique_id(uint8_t* id);
/* Joins the communicator of `nranks` ranks as `rank`.  Returns when all
 * ranks joined, MOE_E_TIMEOUT (communicator aborted) when they have not
 * within MOE_OPT_EP_TIMEOUT_NS, MOE_E_NCCL when NCCL cannot be loaded or
 * fails, MOE_E_STATE when the context already has a communicator.  From then
 * on moe_layer_forward evaluates the experts [rank*E/N, (rank+1)*E/N) only
 * and combines the ranks' work as MOE_OPT_EP_MODE says: REPLICATED (default)
 * sums the partial outputs of all ranks in place (NCCL all-reduce on the
 * context's stream) and applies MOE_F_POST_NORM to the sum, every rank
 * passing the same M tokens and receiving the whole layer's output; GATHER
 * and ALL_TO_ALL take each rank's own tokens and return their rows (see
 * moe_ep_mode).  The routing outputs (tok_active_*) describe the rank's own
 * tokens in GATHER and ALL_TO_ALL.  Every rank must make the same
 * moe_layer_forward calls in the same order, with the same mode.  Output
 * must be fp32 (MOE_F_FP16_OUT is refused), num_experts >= nranks, and the
 * MOE_OPT_EXPERT_BEGIN/END options are ignored meanwhile.  Host waits on a
 * call with a collective (completion of a synchronous call, moe_wait) give
 * up after MOE_OPT_EP_TIMEOUT_NS or on an NCCL error: the communicator is
 * then aborted and the call returns MOE_E_TIMEOUT / MOE_E_NCCL; the context
 * stays usable without it. */
int moe_ep_init(moe_ctx* ctx, const uint8_t* id, int rank, int nranks);
/* Leaves the communicator (after completing enqueued work); the context
 * evaluates all experts again.  MOE_OK also when there was none. */
int moe_ep_finalize(moe_ctx* ctx);

#ifdef __cplusplus
}
#endif
#endif /* MOE_B200_H */
