/*
 * moe_oracle.c -- CPU restatement of phildrip/llm-mojo's Q4_0 MoE-FFN path.
 *
 * TEST INFRASTRUCTURE ONLY: parity checker for libmoe_b200.so and the timed
 * CPU baseline of bench.py.  The product never links or calls this file.
 * Every routine names the reference file:line it restates (paths are within
 * the reference project).  Build: oracle/Makefile (gcc, OpenMP).
 */
#include "moe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define LANES 16

/* ------------------------------------------------------------------ fp16 */
uint16_t orc_f32_to_f16(float f) {
    _Float16 h = (_Float16)f; /* IEEE round-to-nearest-even */
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}
float orc_f16_to_f32(uint16_t u) {
    _Float16 h;
    memcpy(&h, &u, 2);
    return (float)h;
}

/* --------------------------------------------------------------- quantizer
 * moe_kernels.mojo:7-56 == convert_gemma4_moe.py:9-35: per 32-weight block
 * scale = max(max|w| / 7, 1e-5) (fp32), q = round(w * (1/scale)) clamped to
 * [-8, 7], stored +8; element 2j -> low nibble of byte j, 2j+1 -> high. */
int64_t orc_quantize_q4_0(const float* src, int64_t n, uint8_t* packed, float* scales) {
    int64_t ties = 0;
    for (int64_t b = 0; b < n / 32; ++b) {
        const float* v = src + b * 32;
        float max_abs = 0.0f;
        for (int j = 0; j < 32; ++j) {
            float a = fabsf(v[j]);
            if (a > max_abs) max_abs = a;
        }
        float scale = max_abs / 7.0f;
        if (scale < 1e-5f) scale = 1e-5f;
        scales[b] = scale;
        float inv = 1.0f / scale;
        uint8_t q[32];
        for (int j = 0; j < 32; ++j) {
            float t = v[j] * inv;
            if (fabsf(t - truncf(t)) == 0.5f) ++ties;
            float r = nearbyintf(t); /* ties to even, as numpy */
            if (r < -8.0f) r = -8.0f;
            if (r > 7.0f) r = 7.0f;
            q[j] = (uint8_t)((int)r + 8);
        }
        for (int j = 0; j < 16; ++j) packed[b * 16 + j] = (uint8_t)(q[2 * j] | (q[2 * j + 1] << 4));
    }
    return ties;
}

/* ------------------------------------------------------- lane reductions */
static inline float reduce16(const float* a) {
    float t8[8], t4[4], t2[2];
    for (int i = 0; i < 8; ++i) t8[i] = a[i] + a[i + 8];
    for (int i = 0; i < 4; ++i) t4[i] = t8[i] + t8[i + 4];
    for (int i = 0; i < 2; ++i) t2[i] = t4[i] + t4[i + 2];
    return t2[0] + t2[1];
}
static inline float reduce8(const float* a) {
    float t4[4], t2[2];
    for (int i = 0; i < 4; ++i) t4[i] = a[i] + a[i + 4];
    for (int i = 0; i < 2; ++i) t2[i] = t4[i] + t4[i + 2];
    return t2[0] + t2[1];
}

/* even/odd halves: moe_kernels.mojo:96-101 (x_even = x[2j], x_odd = x[2j+1]) */
static void deint_halves(const float* x, float* xd, int64_t c_in) {
    int64_t half = c_in / 2;
    for (int64_t b = 0; b < c_in / 32; ++b)
        for (int j = 0; j < 16; ++j) {
            xd[b * 16 + j] = x[b * 32 + 2 * j];
            xd[half + b * 16 + j] = x[b * 32 + 2 * j + 1];
        }
}

/* One row of q4_matmul_vec's inner loop, moe_kernels.mojo:141-149:
 * acc = we.fma(xe, wo.fma(xo, acc)); result = acc.reduce_add(). */
static inline float row_dot_f32(const uint8_t* wr, const float* sr, const float* xe,
                                const float* xo, int64_t nb) {
    float acc[LANES] = {0};
    for (int64_t b = 0; b < nb; ++b) {
        float sc = sr[b];
        const uint8_t* by = wr + b * 16;
        for (int j = 0; j < LANES; ++j) {
            float we = (float)((int)(by[j] & 15) - 8) * sc;
            float wo = (float)((int)(by[j] >> 4) - 8) * sc;
            acc[j] = fmaf(we, xe[b * 16 + j], fmaf(wo, xo[b * 16 + j], acc[j]));
        }
    }
    return reduce16(acc);
}

/* fp64 scalar row, modelled on test_q4_4row_tiling.mojo:14-35 */
static inline double row_dot_f64(const uint8_t* wr, const float* sr, const float* x, int64_t nb) {
    double row = 0.0;
    for (int64_t b = 0; b < nb; ++b) {
        double blk = 0.0;
        for (int j = 0; j < 16; ++j) {
            int by = wr[b * 16 + j];
            blk += (double)((by & 15) - 8) * x[b * 32 + 2 * j] +
                   (double)((by >> 4) - 8) * x[b * 32 + 2 * j + 1];
        }
        row += blk * (double)sr[b];
    }
    return row;
}

static int clamp_threads(int nthreads) { return nthreads < 1 ? 1 : nthreads; }

/* q4_matmul_vec moe_kernels.mojo:59-162 / q4_matmul_batchN :254-414 (the
 * batched forms compute the same per-token lane sums). */
void orc_q4_matmul(const uint8_t* W, const float* S, const float* x, float* out,
                   int64_t c_in, int64_t c_out, int64_t batch, int prec, int nthreads) {
    int64_t nb = c_in / 32, cp = c_in / 2;
    nthreads = clamp_threads(nthreads);
    if (prec == ORC_F64) {
#pragma omp parallel for num_threads(nthreads) schedule(static) collapse(2)
        for (int64_t t = 0; t < batch; ++t)
            for (int64_t r = 0; r < c_out; ++r)
                out[t * c_out + r] = (float)row_dot_f64(W + r * cp, S + r * nb, x + t * c_in, nb);
        return;
    }
    float* xd = (float*)malloc(sizeof(float) * (size_t)(c_in * batch));
    for (int64_t t = 0; t < batch; ++t) deint_halves(x + t * c_in, xd + t * c_in, c_in);
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t r = 0; r < c_out; ++r)
        for (int64_t t = 0; t < batch; ++t)
            out[t * c_out + r] =
                row_dot_f32(W + r * cp, S + r * nb, xd + t * c_in, xd + t * c_in + cp, nb);
    free(xd);
}

/* ------------------------------------------------------------ norms etc. */
/* rms_norm / rms_norm_noscale, model_speculative_moe_batched.mojo:857-879 */
void orc_rms_norm(const float* x, const float* w, float* out, int64_t n) {
    float acc[8] = {0};
    for (int64_t i = 0; i < n; i += 8)
        for (int l = 0; l < 8; ++l) {
            float v = x[i + l];
            acc[l] = acc[l] + v * v;
        }
    float sum_sq = reduce8(acc);
    float inv_rms = 1.0f / sqrtf(sum_sq / (float)n + 1e-6f);
    for (int64_t i = 0; i < n; ++i) out[i] = w ? x[i] * inv_rms * w[i] : x[i] * inv_rms;
}

/* softmax, model_speculative_moe_batched.mojo:921-933 */
void orc_softmax(float* s, int64_t n) {
    float mx = s[0];
    for (int64_t i = 1; i < n; ++i)
        if (s[i] > mx) mx = s[i];
    float sum = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        s[i] = expf(s[i] - mx);
        sum += s[i];
    }
    for (int64_t i = 0; i < n; ++i) s[i] /= (sum + 1e-10f);
}

/* get_top_k, model_speculative_moe_batched.mojo:936-953 */
void orc_get_top_k(const float* p, int64_t n, int64_t k, int64_t* idx, float* val) {
    for (int64_t i = 0; i < k; ++i) {
        idx[i] = -1;
        val[i] = -999999.0f;
    }
    for (int64_t i = 0; i < n; ++i) {
        float cv = p[i];
        int64_t ci = i;
        for (int64_t j = 0; j < k; ++j)
            if (cv > val[j]) {
                float tv = val[j];
                int64_t ti = idx[j];
                val[j] = cv;
                idx[j] = ci;
                cv = tv;
                ci = ti;
            }
    }
}

/* compute_moe_lod_weights, moe_kernels.mojo:445-490 */
int64_t orc_compute_moe_lod_weights(const int64_t* top_idx, const float* top_val,
                                    const float* pes, float top_p, int64_t* act_idx,
                                    float* act_w, int64_t top_k) {
    float sum = 0.0f;
    for (int64_t i = 0; i < top_k; ++i) sum += top_val[i];
    float inv_sum = 1.0f / (sum + 1e-10f);
    float safe = (top_p == top_p) ? top_p : 1.0f;
    int64_t count = 0;
    if (safe >= 1.0f) {
        for (int64_t i = 0; i < top_k; ++i) {
            float np_ = top_val[i] * inv_sum;
            if (np_ >= 0.05f || i == 0) {
                int64_t e = top_idx[i];
                act_idx[count] = e;
                act_w[count] = np_ * pes[e];
                ++count;
            }
        }
        return count;
    }
    float cum = 0.0f;
    for (int64_t i = 0; i < top_k; ++i) {
        float np_ = top_val[i] * inv_sum;
        if (i > 0 && (np_ < 0.05f || cum >= safe)) break;
        act_idx[count] = top_idx[i];
        act_w[count] = np_;
        cum += np_;
        ++count;
    }
    float renorm = 1.0f / (cum + 1e-10f);
    for (int64_t i = 0; i < count; ++i) act_w[i] = (act_w[i] * renorm) * pes[act_idx[i]];
    return count;
}

/* compute_subbatch_set_cover_moe_weights, moe_kernels.mojo:493-611 */
void orc_compute_subbatch_set_cover_moe_weights(
    int64_t sub_b, const int64_t* all_top_idx, const float* all_top_val, const float* pes,
    float top_p, int64_t* tok_count, int64_t* tok_idx, float* tok_w, int64_t num_experts,
    int64_t top_k, float core_top_p, float singleton_min_prob) {
    (void)num_experts;
    if (sub_b <= 0) return;
    tok_count[0] = orc_compute_moe_lod_weights(all_top_idx, all_top_val, pes, top_p, tok_idx,
                                               tok_w, top_k);
    if (sub_b == 1) return;
    uint8_t in_pool[256] = {0}, freq[256] = {0};
    for (int64_t k = 0; k < tok_count[0]; ++k) {
        int64_t e0 = tok_idx[k];
        if (e0 >= 0 && e0 < 256) {
            in_pool[e0] = 1;
            freq[e0] = 1;
        }
    }
    float safe = (top_p == top_p) ? top_p : 1.0f;
    float inv_sums[64];
    float elig_sums[64];
    for (int64_t b = 1; b < sub_b && b < 64; ++b) {
        const int64_t* ti = all_top_idx + b * top_k;
        const float* tv = all_top_val + b * top_k;
        float s = 0.0f;
        for (int64_t i = 0; i < top_k; ++i) s += tv[i];
        float inv_s = 1.0f / (s + 1e-10f);
        inv_sums[b] = inv_s;
        float cum = 0.0f;
        for (int64_t i = 0; i < top_k; ++i) {
            float np_ = tv[i] * inv_s;
            if (safe >= 1.0f) {
                if (np_ < 0.05f && i > 0) continue;
            } else if (i > 0 && (np_ < 0.05f || cum >= safe)) {
                break;
            }
            int64_t e = ti[i];
            if (e >= 0 && e < 256) {
                freq[e] = (uint8_t)(freq[e] + 1);
                if (i < 2 || np_ >= singleton_min_prob || cum < core_top_p) in_pool[e] = 1;
            }
            cum += np_;
        }
        elig_sums[b] = cum;
    }
    for (int64_t b = 1; b < sub_b && b < 64; ++b) {
        const int64_t* ti = all_top_idx + b * top_k;
        const float* tv = all_top_val + b * top_k;
        int64_t* oi = tok_idx + b * top_k;
        float* ow = tok_w + b * top_k;
        float inv_s = inv_sums[b];
        float cum = 0.0f, kept = 0.0f;
        int64_t count = 0;
        int pruned = 0;
        for (int64_t i = 0; i < top_k; ++i) {
            float np_ = tv[i] * inv_s;
            if (safe >= 1.0f) {
                if (np_ < 0.05f && i > 0) continue;
            } else if (i > 0 && (np_ < 0.05f || cum >= safe)) {
                break;
            }
            int64_t e = ti[i];
            int is_core = (i < 2) || (np_ >= singleton_min_prob) || (cum < core_top_p);
            int is_shared = (e >= 0 && e < 256) && (in_pool[e] != 0 || freq[e] >= 2);
            cum += np_;
            if (is_core || is_shared) {
                oi[count] = e;
                ow[count] = np_;
                kept += np_;
                ++count;
            } else {
                pruned = 1;
            }
        }
        float target = (safe < 1.0f) ? 1.0f : elig_sums[b];
        float renorm = (pruned || safe < 1.0f) ? (target / (kept + 1e-10f)) : 1.0f;
        for (int64_t k = 0; k < count; ++k) ow[k] = (ow[k] * renorm) * pes[oi[k]];
        tok_count[b] = count;
    }
}

/* apply_moe_lod_and_set_cover, diffusion_kernels.mojo:3607-3664 */
void orc_apply_moe_lod_and_set_cover(const int64_t* top_idx, const float* top_val,
                                     const float* pes, float* top_w, int64_t B,
                                     int64_t top_k, int64_t active_top_k, float top_p,
                                     const uint8_t* eb_mask, const int64_t* active_canvas_idx,
                                     int64_t unaccepted_top_k) {
    (void)top_p;
    int64_t eff_k = active_top_k <= top_k ? active_top_k : top_k;
    if (eff_k < 1) eff_k = 1;
    int64_t unacc_k = unaccepted_top_k <= eff_k ? unaccepted_top_k : eff_k;
    if (unacc_k < 1) unacc_k = 1;
    for (int64_t b = 0; b < B; ++b) {
        int64_t orig = active_canvas_idx ? active_canvas_idx[b] : b;
        int accepted = eb_mask ? (eb_mask[orig] != 0) : 1;
        int64_t tok_k = accepted ? eff_k : unacc_k;
        const int64_t* ti = top_idx + b * top_k;
        const float* tv = top_val + b * top_k;
        float* tw = top_w + b * top_k;
        float sd = 0.0f;
        for (int64_t s = 0; s < tok_k; ++s)
            if (ti[s] >= 0) sd += tv[s];
        float inv = 1.0f / (sd + 1e-10f);
        for (int64_t s = 0; s < top_k; ++s) {
            int64_t e = ti[s];
            float np_ = tv[s] * inv;
            tw[s] = (s < tok_k && e >= 0 && e < 128 && np_ >= 0.05f) ? np_ * pes[e] : 0.0f;
        }
    }
}

/* --------------------------------------------------------- activations */
/* gelu_and_mul_moe moe_kernels.mojo:429-442: g * (1/(1+exp(-1.702 g))) * u */
static inline float act_f32(float g, float u, int act) {
    if (act == ORC_ACT_GELU_TANH) {
        float t = tanhf(0.7978845608f * (g + 0.044715f * g * g * g));
        return 0.5f * g * (1.0f + t) * u;
    }
    float sig = 1.0f / (1.0f + expf(-1.702f * g));
    return (g * sig) * u;
}
static inline double act_f64(double g, double u, int act) {
    if (act == ORC_ACT_GELU_TANH) {
        double t = tanh(0.7978845608028654 * (g + 0.044715 * g * g * g));
        return 0.5 * g * (1.0 + t) * u;
    }
    return g / (1.0 + exp(-1.702 * g)) * u;
}

/* ------------------------------------------------------------ stages */
/* run_moe_experts_stage1_8core moe_kernels.mojo:614-696 */
void orc_experts_stage1(const uint8_t* gu_p, const float* gu_s, const float* moe_in,
                        const int64_t* act_idx, int64_t count, float* gu_out_all,
                        float* act_all, int64_t d, int64_t F, int act, int prec,
                        int nthreads) {
    int64_t rows = 2 * F, half = d / 2, nb = d / 32;
    nthreads = clamp_threads(nthreads);
    float* xd = (float*)malloc(sizeof(float) * (size_t)d);
    deint_halves(moe_in, xd, d);
    float* gu = gu_out_all ? gu_out_all : (float*)malloc(sizeof(float) * (size_t)(rows * (count > 0 ? count : 1)));
    for (int64_t s = 0; s < count; ++s) {
        int64_t e = act_idx[s];
        const uint8_t* wp = gu_p + e * rows * half;
        const float* ws = gu_s + e * rows * nb;
        float* g = gu + s * rows;
        if (prec == ORC_F64) {
            double* tmp = (double*)malloc(sizeof(double) * (size_t)rows);
#pragma omp parallel for num_threads(nthreads) schedule(static)
            for (int64_t r = 0; r < rows; ++r) tmp[r] = row_dot_f64(wp + r * half, ws + r * nb, moe_in, nb);
            for (int64_t r = 0; r < rows; ++r) g[r] = (float)tmp[r];
            for (int64_t j = 0; j < F; ++j) act_all[s * F + j] = (float)act_f64(tmp[j], tmp[F + j], act);
            free(tmp);
        } else {
#pragma omp parallel for num_threads(nthreads) schedule(static)
            for (int64_t r = 0; r < rows; ++r) g[r] = row_dot_f32(wp + r * half, ws + r * nb, xd, xd + half, nb);
            for (int64_t j = 0; j < F; ++j) act_all[s * F + j] = act_f32(g[j], g[F + j], act);
        }
    }
    if (!gu_out_all) free(gu);
    free(xd);
}

/* run_moe_experts_stage2_8core moe_kernels.mojo:699-781 */
void orc_experts_stage2(const uint8_t* dn_p, const float* dn_s, const float* act_all,
                        const int64_t* act_idx, const float* act_w, int64_t count,
                        float* moe_out, int64_t d, int64_t F, int prec, int nthreads) {
    int64_t half = F / 2, nb = F / 32;
    nthreads = clamp_threads(nthreads);
    if (prec == ORC_F64) {
#pragma omp parallel for num_threads(nthreads) schedule(static)
        for (int64_t r = 0; r < d; ++r) {
            double acc = 0.0;
            for (int64_t s = 0; s < count; ++s) {
                int64_t e = act_idx[s];
                acc += (double)act_w[s] * row_dot_f64(dn_p + e * d * half + r * half,
                                                      dn_s + e * d * nb + r * nb, act_all + s * F, nb);
            }
            moe_out[r] = (float)acc;
        }
        return;
    }
    float* ad = (float*)malloc(sizeof(float) * (size_t)(F * (count > 0 ? count : 1)));
    for (int64_t s = 0; s < count; ++s) deint_halves(act_all + s * F, ad + s * F, F);
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t r = 0; r < d; ++r) {
        moe_out[r] = 0.0f;
        for (int64_t s = 0; s < count; ++s) {
            int64_t e = act_idx[s];
            float v = row_dot_f32(dn_p + e * d * half + r * half, dn_s + e * d * nb + r * nb,
                                  ad + s * F, ad + s * F + half, nb);
            moe_out[r] += v * act_w[s];
        }
    }
    free(ad);
}

/* --------------------------------------------------------------- router */
void orc_route(const orc_layer* L, int64_t M, const float* x, int use_set_cover,
               float* scores_out, int64_t* top_idx, float* top_val, int64_t* tok_count,
               int64_t* tok_idx, float* tok_w, float* moe_in, int prec) {
    int64_t d = L->d, E = L->E, K = L->top_k;
    float* nx = (float*)malloc(sizeof(float) * (size_t)d);
    float* sx = (float*)malloc(sizeof(float) * (size_t)d);
    float* sc = (float*)malloc(sizeof(float) * (size_t)E);
    int64_t* ti = (int64_t*)malloc(sizeof(int64_t) * (size_t)(M * K));
    float* tv = (float*)malloc(sizeof(float) * (size_t)(M * K));
    for (int64_t t = 0; t < M; ++t) {
        const float* xt = x + t * d;
        /* model_speculative_moe_batched.mojo:2102-2104 */
        orc_rms_norm(xt, NULL, nx, d);
        for (int64_t j = 0; j < d; ++j) sx[j] = nx[j] * L->router_scale[j] * L->r_scale_factor;
        if (L->router_p) {
            orc_q4_matmul(L->router_p, L->router_s, sx, sc, d, E, 1, prec, 1);
        } else {
            for (int64_t e = 0; e < E; ++e) {
                double a = 0.0;
                for (int64_t j = 0; j < d; ++j) a += (double)L->router_f32[e * d + j] * sx[j];
                sc[e] = (float)a;
            }
        }
        if (scores_out) memcpy(scores_out + t * E, sc, sizeof(float) * (size_t)E);
        if (L->router_logit_bias)  /* synthetic skew only; the reference has no bias */
            for (int64_t e = 0; e < E; ++e) sc[e] += L->router_logit_bias[e];
        orc_softmax(sc, E);
        orc_get_top_k(sc, E, K, ti + t * K, tv + t * K);
        if (moe_in) orc_rms_norm(xt, L->pre_norm_w, moe_in + t * d, d);
    }
    if (top_idx) memcpy(top_idx, ti, sizeof(int64_t) * (size_t)(M * K));
    if (top_val) memcpy(top_val, tv, sizeof(float) * (size_t)(M * K));
    if (tok_count && tok_idx && tok_w) {
        if (use_set_cover) {
            /* engine processes sub-batches of <= 5 (model_speculative_moe_batched.mojo:2690-2727) */
            for (int64_t t0 = 0; t0 < M; t0 += 5) {
                int64_t sb = M - t0 < 5 ? M - t0 : 5;
                orc_compute_subbatch_set_cover_moe_weights(sb, ti + t0 * K, tv + t0 * K,
                                                           L->per_expert_scale, L->top_p,
                                                           tok_count + t0, tok_idx + t0 * K,
                                                           tok_w + t0 * K, E, K, 0.85f, 0.068f);
            }
        } else {
            for (int64_t t = 0; t < M; ++t)
                tok_count[t] = orc_compute_moe_lod_weights(ti + t * K, tv + t * K,
                                                           L->per_expert_scale, L->top_p,
                                                           tok_idx + t * K, tok_w + t * K, K);
        }
    }
    free(nx); free(sx); free(sc); free(ti); free(tv);
}

/* --------------------------------------------------- expert half, M tokens
 * F32: run_moe_coalesced_core moe_kernels.mojo:1321-1383 over sub-batches of
 * <= 5 tokens (the engine's chunking, model_speculative_moe_batched.mojo:
 * 2690-2727): bucket by expert in ascending order, each unique expert's rows
 * read once for its tokens, stage-2 accumulation in ascending expert order.
 * F64: per token, per slot, fp64. */
static void coalesced_chunk_f32(const orc_layer* L, int64_t sb, const float* xin,
                                const int64_t* cnt, const int64_t* idx, const float* w,
                                float* out, int nthreads) {
    int64_t d = L->d, F = L->F, E = L->E, K = L->top_k;
    int64_t rows = 2 * F, half = d / 2, nb = d / 32, dh = F / 2, dnb = F / 32;
    int64_t* bc = (int64_t*)calloc((size_t)E, sizeof(int64_t));
    int64_t* bt = (int64_t*)malloc(sizeof(int64_t) * (size_t)(E * sb));
    float* bw = (float*)malloc(sizeof(float) * (size_t)(E * sb));
    /* moe_kernels.mojo:815-835 */
    for (int64_t b = 0; b < sb; ++b)
        for (int64_t k = 0; k < cnt[b]; ++k) {
            int64_t e = idx[b * K + k];
            bt[e * sb + bc[e]] = b;
            bw[e * sb + bc[e]] = w[b * K + k];
            bc[e]++;
        }
    int64_t* ue = (int64_t*)malloc(sizeof(int64_t) * (size_t)E);
    int64_t* ub = (int64_t*)malloc(sizeof(int64_t) * (size_t)E);
    int64_t nu = 0, pairs = 0;
    for (int64_t e = 0; e < E; ++e)
        if (bc[e] > 0) {
            ue[nu] = e;
            ub[nu] = pairs;
            pairs += bc[e];
            ++nu;
        }
    float* xd = (float*)malloc(sizeof(float) * (size_t)(sb * d));
    for (int64_t b = 0; b < sb; ++b) deint_halves(xin + b * d, xd + b * d, d);
    float* gu = (float*)malloc(sizeof(float) * (size_t)((pairs > 0 ? pairs : 1) * rows));
    float* ad = (float*)malloc(sizeof(float) * (size_t)((pairs > 0 ? pairs : 1) * F));
    /* coal_s1 :838-1046 */
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t u = 0; u < nu; ++u) {
            int64_t e = ue[u];
            const uint8_t* wr = L->gu_p + e * rows * half + r * half;
            const float* sr = L->gu_s + e * rows * nb + r * nb;
            for (int64_t i = 0; i < bc[e]; ++i) {
                const float* xe = xd + bt[e * sb + i] * d;
                gu[(ub[u] + i) * rows + r] = row_dot_f32(wr, sr, xe, xe + half, nb);
            }
        }
    /* fused GeGLU + deinterleave :1049-1068 */
    for (int64_t p = 0; p < pairs; ++p) {
        float a[4096];
        for (int64_t j = 0; j < F; ++j) a[j] = act_f32(gu[p * rows + j], gu[p * rows + F + j], L->act);
        deint_halves(a, ad + p * F, F);
    }
    /* coal_s2 :1090-1318 */
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t r = 0; r < d; ++r) {
        for (int64_t b = 0; b < sb; ++b) out[b * d + r] = 0.0f;
        for (int64_t u = 0; u < nu; ++u) {
            int64_t e = ue[u];
            const uint8_t* wr = L->dn_p + e * d * dh + r * dh;
            const float* sr = L->dn_s + e * d * dnb + r * dnb;
            for (int64_t i = 0; i < bc[e]; ++i) {
                const float* ae = ad + (ub[u] + i) * F;
                float v = row_dot_f32(wr, sr, ae, ae + dh, dnb);
                out[bt[e * sb + i] * d + r] += v * bw[e * sb + i];
            }
        }
    }
    free(bc); free(bt); free(bw); free(ue); free(ub); free(xd); free(gu); free(ad);
}

void orc_experts_forward(const orc_layer* L, int64_t M, const float* moe_in,
                         const int64_t* tok_count, const int64_t* tok_idx, const float* tok_w,
                         float* moe_out, int prec, int nthreads) {
    int64_t d = L->d, F = L->F, K = L->top_k;
    nthreads = clamp_threads(nthreads);
    if (prec == ORC_F32) {
        for (int64_t t0 = 0; t0 < M; t0 += 5) {
            int64_t sb = M - t0 < 5 ? M - t0 : 5;
            coalesced_chunk_f32(L, sb, moe_in + t0 * d, tok_count + t0, tok_idx + t0 * K,
                                tok_w + t0 * K, moe_out + t0 * d, nthreads);
        }
        return;
    }
    int64_t rows = 2 * F, half = d / 2, nb = d / 32, dh = F / 2, dnb = F / 32;
    double* h = (double*)malloc(sizeof(double) * (size_t)(M * K * rows));
    double* a = (double*)malloc(sizeof(double) * (size_t)(M * K * F));
    float* af = (float*)malloc(sizeof(float) * (size_t)(M * K * F));
#pragma omp parallel for num_threads(nthreads) schedule(dynamic, 4) collapse(2)
    for (int64_t t = 0; t < M; ++t)
        for (int64_t r = 0; r < rows; ++r)
            for (int64_t k = 0; k < tok_count[t]; ++k) {
                int64_t e = tok_idx[t * K + k];
                h[(t * K + k) * rows + r] = row_dot_f64(L->gu_p + e * rows * half + r * half,
                                                        L->gu_s + e * rows * nb + r * nb,
                                                        moe_in + t * d, nb);
            }
    for (int64_t t = 0; t < M; ++t)
        for (int64_t k = 0; k < tok_count[t]; ++k)
            for (int64_t j = 0; j < F; ++j) {
                int64_t s = t * K + k;
                a[s * F + j] = act_f64(h[s * rows + j], h[s * rows + F + j], L->act);
                af[s * F + j] = (float)a[s * F + j];
            }
    /* down projection with the activations kept in fp64 */
#pragma omp parallel for num_threads(nthreads) schedule(static) collapse(2)
    for (int64_t t = 0; t < M; ++t)
        for (int64_t r = 0; r < d; ++r) {
            double acc = 0.0;
            for (int64_t k = 0; k < tok_count[t]; ++k) {
                int64_t e = tok_idx[t * K + k];
                const uint8_t* wr = L->dn_p + e * d * dh + r * dh;
                const float* sr = L->dn_s + e * d * dnb + r * dnb;
                const double* av = a + (t * K + k) * F;
                double row = 0.0;
                for (int64_t b = 0; b < dnb; ++b) {
                    double blk = 0.0;
                    for (int j = 0; j < 16; ++j) {
                        int by = wr[b * 16 + j];
                        blk += (double)((by & 15) - 8) * av[b * 32 + 2 * j] +
                               (double)((by >> 4) - 8) * av[b * 32 + 2 * j + 1];
                    }
                    row += blk * (double)sr[b];
                }
                acc += (double)tok_w[t * K + k] * row;
            }
            moe_out[t * d + r] = (float)acc;
        }
    free(h); free(a); free(af);
}

void orc_layer_forward(const orc_layer* L, int64_t M, const float* x, float* out, int flags,
                       int prec, int nthreads, int64_t* tok_count, int64_t* tok_idx,
                       float* tok_w) {
    int64_t d = L->d, K = L->top_k;
    int64_t* cnt = tok_count ? tok_count : (int64_t*)malloc(sizeof(int64_t) * (size_t)M);
    int64_t* idx = tok_idx ? tok_idx : (int64_t*)malloc(sizeof(int64_t) * (size_t)(M * K));
    float* w = tok_w ? tok_w : (float*)malloc(sizeof(float) * (size_t)(M * K));
    float* moe_in = (float*)malloc(sizeof(float) * (size_t)(M * d));
    /* routing is always the reference's fp32 arithmetic */
    orc_route(L, M, x, (flags & 4) != 0, NULL, NULL, NULL, cnt, idx, w, moe_in, ORC_F32);
    orc_experts_forward(L, M, moe_in, cnt, idx, w, out, prec, nthreads);
    if (flags & 1)
        for (int64_t t = 0; t < M; ++t) orc_rms_norm(out + t * d, L->post_norm_w, out + t * d, d);
    if (!tok_count) free(cnt);
    if (!tok_idx) free(idx);
    if (!tok_w) free(w);
    free(moe_in);
}

/* ------------------------------------------------------------ diffusion
 * run_diffusion_moe_experts_parallel diffusion_kernels.mojo:236-404 with
 * q4_moe_expert_single_thread :110-233 (8-lane FMA over block-32
 * deinterleaved rows) and the fp32 per-token combine :386-399. */
static void deint_block32(const float* x, float* xd, int64_t c) {
    for (int64_t b = 0; b < c / 32; ++b)
        for (int j = 0; j < 16; ++j) {
            xd[b * 32 + j] = x[b * 32 + 2 * j];
            xd[b * 32 + 16 + j] = x[b * 32 + 2 * j + 1];
        }
}
static void dequant_row_block32(const uint8_t* wr, const float* sr, float* wd, int64_t c) {
    for (int64_t b = 0; b < c / 32; ++b) {
        float sc = sr[b];
        for (int j = 0; j < 16; ++j) {
            wd[b * 32 + j] = (float)((int)(wr[b * 16 + j] & 15) - 8) * sc;
            wd[b * 32 + 16 + j] = (float)((int)(wr[b * 16 + j] >> 4) - 8) * sc;
        }
    }
}
static inline float dot8_f32(const float* w, const float* x, int64_t c) {
    float a[8] = {0};
    for (int64_t k = 0; k < c; k += 8)
        for (int l = 0; l < 8; ++l) a[l] = fmaf(w[k + l], x[k + l], a[l]);
    return reduce8(a);
}

void orc_diffusion_experts(const uint8_t* gu_p, const float* gu_s, const uint8_t* dn_p,
                           const float* dn_s, const uint16_t* in_f16, const int64_t* top_idx,
                           const float* top_w, uint16_t* out_f16, int64_t B, int64_t d,
                           int64_t F, int64_t top_k, int act, int prec, int nthreads) {
    int64_t rows = 2 * F;
    nthreads = clamp_threads(nthreads);
    int64_t P = B * top_k;
    float* y = (float*)malloc(sizeof(float) * (size_t)((P > 0 ? P : 1) * d));
    int64_t* slot = (int64_t*)malloc(sizeof(int64_t) * (size_t)(P > 0 ? P : 1));
    int64_t cnt[1024] = {0}, off[1024], wr_[1024];
    int64_t E = 0;
    for (int64_t i = 0; i < P; ++i)
        if (top_w[i] > 0.0f) {
            cnt[top_idx[i]]++;
            if (top_idx[i] + 1 > E) E = top_idx[i] + 1;
        }
    int64_t tot = 0;
    for (int64_t e = 0; e < E; ++e) {
        off[e] = wr_[e] = tot;
        tot += cnt[e];
    }
    int64_t* at = (int64_t*)malloc(sizeof(int64_t) * (size_t)(tot > 0 ? tot : 1));
    for (int64_t t = 0; t < B; ++t)
        for (int64_t s = 0; s < top_k; ++s) {
            slot[t * top_k + s] = -1;
            if (top_w[t * top_k + s] > 0.0f) {
                int64_t e = top_idx[t * top_k + s];
                at[wr_[e]] = t;
                slot[t * top_k + s] = wr_[e]++;
            }
        }
    float* xin = (float*)malloc(sizeof(float) * (size_t)((B > 0 ? B : 1) * d));
    for (int64_t i = 0; i < B * d; ++i) xin[i] = orc_f16_to_f32(in_f16[i]);
#pragma omp parallel for num_threads(nthreads) schedule(dynamic, 1)
    for (int64_t e = 0; e < E; ++e) {
        if (cnt[e] == 0) continue;
        int64_t n = cnt[e];
        const uint8_t* gp = gu_p + e * rows * (d / 2);
        const float* gs = gu_s + e * rows * (d / 32);
        const uint8_t* dp = dn_p + e * d * (F / 2);
        const float* ds = dn_s + e * d * (F / 32);
        float* xd = (float*)malloc(sizeof(float) * (size_t)(n * d));
        float* h = (float*)malloc(sizeof(float) * (size_t)(n * rows));
        float* ad = (float*)malloc(sizeof(float) * (size_t)(n * F));
        float* wd = (float*)malloc(sizeof(float) * (size_t)(d > F ? d : F));
        for (int64_t i = 0; i < n; ++i) deint_block32(xin + at[off[e] + i] * d, xd + i * d, d);
        if (prec == ORC_F64) {
            double* hh = (double*)malloc(sizeof(double) * (size_t)(n * rows));
            for (int64_t r = 0; r < rows; ++r)
                for (int64_t i = 0; i < n; ++i)
                    hh[i * rows + r] = row_dot_f64(gp + r * (d / 2), gs + r * (d / 32),
                                                   xin + at[off[e] + i] * d, d / 32);
            for (int64_t i = 0; i < n; ++i)
                for (int64_t j = 0; j < F; ++j)
                    h[i * F + j] = (float)act_f64(hh[i * rows + j], hh[i * rows + F + j], act);
            for (int64_t r = 0; r < d; ++r)
                for (int64_t i = 0; i < n; ++i)
                    y[(off[e] + i) * d + r] = (float)row_dot_f64(dp + r * (F / 2), ds + r * (F / 32),
                                                                 h + i * F, F / 32);
            free(hh);
        } else {
            for (int64_t r = 0; r < rows; ++r) {
                dequant_row_block32(gp + r * (d / 2), gs + r * (d / 32), wd, d);
                for (int64_t i = 0; i < n; ++i) h[i * rows + r] = dot8_f32(wd, xd + i * d, d);
            }
            /* gelu_and_mul_to_deinterleaved_f32 :78-107 */
            for (int64_t i = 0; i < n; ++i) {
                float a[4096];
                for (int64_t j = 0; j < F; ++j) a[j] = act_f32(h[i * rows + j], h[i * rows + F + j], act);
                deint_block32(a, ad + i * F, F);
            }
            for (int64_t r = 0; r < d; ++r) {
                dequant_row_block32(dp + r * (F / 2), ds + r * (F / 32), wd, F);
                for (int64_t i = 0; i < n; ++i) y[(off[e] + i) * d + r] = dot8_f32(wd, ad + i * F, F);
            }
        }
        free(xd); free(h); free(ad); free(wd);
    }
    /* accum_token_worker :386-399 */
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t t = 0; t < B; ++t)
        for (int64_t j = 0; j < d; ++j) {
            if (prec == ORC_F64) {
                double s = 0.0;
                for (int64_t k = 0; k < top_k; ++k) {
                    int64_t p = slot[t * top_k + k];
                    if (p >= 0) s += (double)y[p * d + j] * (double)top_w[t * top_k + k];
                }
                out_f16[t * d + j] = orc_f32_to_f16((float)s);
            } else {
                float s = 0.0f;
                for (int64_t k = 0; k < top_k; ++k) {
                    int64_t p = slot[t * top_k + k];
                    if (p >= 0) s = fmaf(y[p * d + j], top_w[t * top_k + k], s);
                }
                out_f16[t * d + j] = orc_f32_to_f16(s);
            }
        }
    free(y); free(slot); free(at); free(xin);
}

/* ------------------------------------------ diffusion router-subspace bypass
 * router_subspace_ffn_filter (diffusion_kernels.mojo:2253-2337).  A token
 * whose top-2 experts equal the ones it had when last evaluated, and whose
 * router logits moved by at most tau_ffn relative to that evaluation, is
 * bypassed (its routing weights zeroed); the others are listed in
 * ffn_keep_b in ascending b and their r_prev / prev_top2 rows updated.
 * The drift sums follow the reference's 8-lane SIMD loop: lane l takes the
 * experts e = l (mod 8) with fused multiply-adds, the lanes are added as a
 * halving tree (reduce8), and a tail of num_experts % 8 experts is added
 * one by one (multiply, then add). */
int64_t orc_router_subspace_ffn_filter(const float* r_curr, float* r_prev, const int64_t* top_idx,
                                       int64_t* prev_top2, const uint8_t* eb_mask,
                                       const int64_t* active_canvas_idx, int64_t* ffn_keep_b,
                                       int64_t B, int64_t num_experts, int64_t top_k, int64_t step,
                                       float tau_ffn, float* top_weights) {
    if (B <= 0) return 0;
    int64_t active = 0;
    const float tau_sq = tau_ffn * tau_ffn;
    for (int64_t b = 0; b < B; ++b) {
        const int64_t ot = active_canvas_idx ? active_canvas_idx[b] : b;
        const int accepted = eb_mask ? (eb_mask[ot] != 0) : 1;
        int bypass = 0;
        if (step >= 1 && accepted && top_k >= 2 && num_experts > 0) {
            const int64_t e0 = top_idx[b * top_k], e1 = top_idx[b * top_k + 1];
            const int64_t p0 = prev_top2[ot * 2], p1 = prev_top2[ot * 2 + 1];
            if (p0 >= 0 && p1 >= 0 && e0 == p0 && e1 == p1) {
                const float* cr = r_curr + b * num_experts;
                const float* pr = r_prev + ot * num_experts;
                float vd[8] = {0}, vn[8] = {0};
                int64_t e = 0;
                for (; e + 7 < num_experts; e += 8)
                    for (int l = 0; l < 8; ++l) {
                        const float d = cr[e + l] - pr[e + l];
                        vd[l] = fmaf(d, d, vd[l]);
                        vn[l] = fmaf(pr[e + l], pr[e + l], vn[l]);
                    }
                float diff_sq = reduce8(vd), norm_sq = reduce8(vn);
                for (; e < num_experts; ++e) {
                    const float d = cr[e] - pr[e];
                    diff_sq += d * d;
                    norm_sq += pr[e] * pr[e];
                }
                bypass = norm_sq > 1e-12f ? (diff_sq <= tau_sq * norm_sq) : (diff_sq <= 1e-12f);
            }
        }
        if (bypass) {
            if (top_weights)
                for (int64_t s = 0; s < top_k; ++s) top_weights[b * top_k + s] = 0.0f;
        } else {
            ffn_keep_b[active++] = b;
            if (top_k >= 1) prev_top2[ot * 2] = top_idx[b * top_k];
            if (top_k >= 2) prev_top2[ot * 2 + 1] = top_idx[b * top_k + 1];
            memcpy(r_prev + ot * num_experts, r_curr + b * num_experts, sizeof(float) * (size_t)num_experts);
        }
    }
    return active;
}

/* sync_moe_subspace_cache (diffusion_kernels.mojo:2345-2381) and
 * scatter_and_restore_ffn_subspace (:2386-2426), rows of `row_bytes` bytes
 * (dim * sizeof(dtype)): walking b in order with a cursor into ffn_keep_b,
 * an evaluated row is saved to the cache (and, for the scatter, taken from
 * the compacted sub-batch output first); a bypassed row is restored from
 * the cache. */
void orc_sync_moe_subspace_cache(uint8_t* moe_out, uint8_t* cache, const int64_t* active_canvas_idx,
                                 const int64_t* ffn_keep_b, int64_t B, int64_t ffn_active_len,
                                 int64_t row_bytes) {
    if (B <= 0 || row_bytes <= 0) return;
    int64_t cur = 0;
    for (int64_t b = 0; b < B; ++b) {
        const int64_t ot = active_canvas_idx ? active_canvas_idx[b] : b;
        if (cur < ffn_active_len && ffn_keep_b[cur] == b) {
            memcpy(cache + ot * row_bytes, moe_out + b * row_bytes, (size_t)row_bytes);
            ++cur;
        } else {
            memcpy(moe_out + b * row_bytes, cache + ot * row_bytes, (size_t)row_bytes);
        }
    }
}

void orc_scatter_and_restore_ffn_subspace(const uint8_t* sub_out, uint8_t* cache, uint8_t* full_out,
                                          const int64_t* active_canvas_idx, const int64_t* ffn_keep_b,
                                          int64_t B, int64_t ffn_active_len, int64_t row_bytes) {
    if (B <= 0 || row_bytes <= 0) return;
    int64_t cur = 0;
    for (int64_t b = 0; b < B; ++b) {
        const int64_t ot = active_canvas_idx ? active_canvas_idx[b] : b;
        if (cur < ffn_active_len && ffn_keep_b[cur] == b) {
            memcpy(full_out + b * row_bytes, sub_out + cur * row_bytes, (size_t)row_bytes);
            memcpy(cache + ot * row_bytes, sub_out + cur * row_bytes, (size_t)row_bytes);
            ++cur;
        } else {
            memcpy(full_out + b * row_bytes, cache + ot * row_bytes, (size_t)row_bytes);
        }
    }
}
