/*
 * moe_oracle.h -- CPU restatement of phildrip/llm-mojo's Q4_0 MoE-FFN path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * path in libmoe_b200.so and the timed CPU baseline in bench.py.  Nothing in
 * the product links, loads or calls it.
 *
 * Two precisions are offered for every compute routine:
 *   ORC_F64  scalar, fp64 accumulation (the checker used for tolerances;
 *            modelled on the scalar oracle of test_q4_4row_tiling.mojo:14-35)
 *   ORC_F32  fp32 restatement of the reference's SIMD kernels: activations
 *            deinterleaved into even/odd halves, 16-lane fp32 FMA
 *            accumulators, lane reduction, rows split over threads
 *            (moe_kernels.mojo:59-162, :614-781).  This is the CPU baseline.
 *
 * Pinning: the quantizer is checked bit-exactly against the reference's own
 * numpy quantizer (convert_gemma4_moe.py:9-35) through committed fixtures in
 * tests/golden/; routing helpers are checked against the known answers of
 * test_moe_lod_top_p.mojo:28-49 and test_kernels.mojo:3021-3053.
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_F32 = 0, ORC_F64 = 1 };
enum { ORC_ACT_SIGMOID1702 = 0, ORC_ACT_GELU_TANH = 1 };

/* moe_kernels.mojo:7-56 and convert_gemma4_moe.py:9-35.  Returns the number
 * of exact .5 rounding ties met (numpy rounds them to even). */
int64_t orc_quantize_q4_0(const float* src, int64_t n, uint8_t* packed, float* scales);

/* out[b*c_out + r] = sum_k deq(W)[r,k] * x[b*c_in + k]
 * (q4_matmul_vec moe_kernels.mojo:59, q4_matmul_batchN :254) */
void orc_q4_matmul(const uint8_t* W, const float* S, const float* x, float* out,
                   int64_t c_in, int64_t c_out, int64_t batch, int prec, int nthreads);

/* model_speculative_moe_batched.mojo:857-879; w == NULL is rms_norm_noscale */
void orc_rms_norm(const float* x, const float* w, float* out, int64_t n);
/* model_speculative_moe_batched.mojo:921-933 */
void orc_softmax(float* s, int64_t n);
/* model_speculative_moe_batched.mojo:936-953 (strict '>' insertion) */
void orc_get_top_k(const float* p, int64_t n, int64_t k, int64_t* idx, float* val);
/* moe_kernels.mojo:445-490 */
int64_t orc_compute_moe_lod_weights(const int64_t* top_idx, const float* top_val,
                                    const float* per_expert_scale, float top_p,
                                    int64_t* act_idx, float* act_w, int64_t top_k);
/* moe_kernels.mojo:493-611 */
void orc_compute_subbatch_set_cover_moe_weights(
    int64_t sub_b, const int64_t* all_top_idx, const float* all_top_val,
    const float* per_expert_scale, float top_p, int64_t* tok_active_count,
    int64_t* tok_active_idx, float* tok_active_weights, int64_t num_experts,
    int64_t top_k, float core_top_p, float singleton_min_prob);
/* diffusion_kernels.mojo:3607-3664 */
void orc_apply_moe_lod_and_set_cover(const int64_t* top_idx, const float* top_val,
                                     const float* per_expert_scale, float* top_w,
                                     int64_t B, int64_t top_k, int64_t active_top_k,
                                     float top_p, const uint8_t* eb_mask,
                                     const int64_t* active_canvas_idx,
                                     int64_t unaccepted_top_k);

/* run_moe_experts_stage1_8core moe_kernels.mojo:614-696 (+ gelu_and_mul_moe :429) */
void orc_experts_stage1(const uint8_t* gu_p, const float* gu_s, const float* moe_in,
                        const int64_t* act_idx, int64_t count, float* gu_out_all,
                        float* act_all, int64_t d, int64_t F, int act, int prec,
                        int nthreads);
/* run_moe_experts_stage2_8core moe_kernels.mojo:699-781 */
void orc_experts_stage2(const uint8_t* dn_p, const float* dn_s, const float* act_all,
                        const int64_t* act_idx, const float* act_w, int64_t count,
                        float* moe_out, int64_t d, int64_t F, int prec, int nthreads);

/* Router for M tokens, model_speculative_moe_batched.mojo:2102-2118 and
 * :1001-1083: rms_norm_noscale * router_scale * r_scale_factor -> Q4 router
 * -> softmax -> top-k -> LOD (or set-cover), plus the expert input
 * moe_in = rms_norm(x, pre_norm_w).  Any output pointer may be NULL. */
typedef struct {
    int64_t d, F, E, top_k;
    int act;                      /* ORC_ACT_* */
    float r_scale_factor, top_p;
    const uint8_t* router_p; const float* router_s;   /* Q4_0 router [E x d] */
    const float* router_f32;      /* optional fp32 router [E x d]; used when router_p == NULL */
    const float* router_scale;    /* [d] */
    const float* per_expert_scale;/* [E] */
    const float* pre_norm_w;      /* [d] pre_feedforward_layernorm_2 */
    const float* post_norm_w;     /* [d] post_feedforward_layernorm_2 */
    const uint8_t* gu_p; const float* gu_s;           /* [E][2F x d] */
    const uint8_t* dn_p; const float* dn_s;           /* [E][d x F]  */
    /* optional [E], added to the router logits before the softmax.  No
     * counterpart in the reference (its router has no bias): the synthetic
     * skew of the M=8192 prefill workload, a Zipf(1.1) bias, goes through
     * the same place in the library (moe_layer_desc.router_logit_bias). */
    const float* router_logit_bias;
} orc_layer;

void orc_route(const orc_layer* L, int64_t M, const float* x, int use_set_cover,
               float* scores_out, int64_t* top_idx, float* top_val,
               int64_t* tok_count, int64_t* tok_idx, float* tok_w, float* moe_in,
               int prec);

/* Expert half of the layer for M tokens given routing (run_moe_coalesced_core
 * semantics, moe_kernels.mojo:1321-1383, any number of tokens). */
void orc_experts_forward(const orc_layer* L, int64_t M, const float* moe_in,
                         const int64_t* tok_count, const int64_t* tok_idx,
                         const float* tok_w, float* moe_out, int prec, int nthreads);

/* Whole layer: route, experts, optional post-norm (flags & 1). */
void orc_layer_forward(const orc_layer* L, int64_t M, const float* x, float* out,
                       int flags, int prec, int nthreads, int64_t* tok_count,
                       int64_t* tok_idx, float* tok_w);

/* run_diffusion_moe_experts_parallel diffusion_kernels.mojo:236-404:
 * fp16 canvas in/out, slot active iff weight > 0, fp32 combine then fp16. */
void orc_diffusion_experts(const uint8_t* gu_p, const float* gu_s, const uint8_t* dn_p,
                           const float* dn_s, const uint16_t* in_f16,
                           const int64_t* top_idx, const float* top_w, uint16_t* out_f16,
                           int64_t B, int64_t d, int64_t F, int64_t top_k, int act,
                           int prec, int nthreads);

/* Diffusion router-subspace bypass: router_subspace_ffn_filter
 * (diffusion_kernels.mojo:2253-2337; returns the number of evaluated
 * tokens), sync_moe_subspace_cache (:2345-2381) and
 * scatter_and_restore_ffn_subspace (:2386-2426) over rows of row_bytes. */
int64_t orc_router_subspace_ffn_filter(const float* r_curr, float* r_prev, const int64_t* top_idx,
                                       int64_t* prev_top2, const uint8_t* eb_mask,
                                       const int64_t* active_canvas_idx, int64_t* ffn_keep_b,
                                       int64_t B, int64_t num_experts, int64_t top_k, int64_t step,
                                       float tau_ffn, float* top_weights);
void orc_sync_moe_subspace_cache(uint8_t* moe_out, uint8_t* cache, const int64_t* active_canvas_idx,
                                 const int64_t* ffn_keep_b, int64_t B, int64_t ffn_active_len,
                                 int64_t row_bytes);
void orc_scatter_and_restore_ffn_subspace(const uint8_t* sub_out, uint8_t* cache, uint8_t* full_out,
                                          const int64_t* active_canvas_idx, const int64_t* ffn_keep_b,
                                          int64_t B, int64_t ffn_active_len, int64_t row_bytes);

/* fp16 helpers (round to nearest even) */
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);

#ifdef __cplusplus
}
#endif
#endif
