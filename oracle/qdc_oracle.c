/*
 * qdc_oracle.c -- CPU restatement of QwenDecisionCore.jl's per-layer row ops.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline); never
 * linked into or called by the product library.  See qdc_oracle.h for the
 * layout conventions.  Built with -ffp-contract=off so every Float32
 * multiply and add rounds separately, as in the reference's Julia loops.
 */
#include "qdc_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 1;

void qdo_set_threads(int threads) { g_threads = threads < 1 ? 1 : threads; }
int qdo_get_threads(void) { return g_threads; }

/* ---- bfloat16, src/safetensors.jl:28-30 and :38-42 ---------------------- */

float qdo_bf16_decode(uint16_t bits) {
    uint32_t wide = (uint32_t)bits << 16;
    float out;
    memcpy(&out, &wide, sizeof out);
    return out;
}

uint16_t qdo_bf16_encode(float value) {
    uint32_t bits;
    memcpy(&bits, &value, sizeof bits);
    /* rounded = bits + 0x7fff + ((bits >> 16) & 1), UInt32 wrap-around. */
    uint32_t rounded = bits + 0x00007fffu + ((bits >> 16) & 0x1u);
    return (uint16_t)(rounded >> 16);
}

void qdo_bf16_encode_array(uint16_t *out, const float *in, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = qdo_bf16_encode(in[i]);
}

void qdo_bf16_decode_array(float *out, const uint16_t *in, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = qdo_bf16_decode(in[i]);
}

/* ---- SiLU, src/backbone.jl:196-197 -------------------------------------- */

float qdo_silu(float x) {
    float e = expf(-x);
    float d = 1.0f + e;
    float s = 1.0f / d; /* inv(one(x) + exp(-x)) */
    return x * s;
}

/* ---- helpers ------------------------------------------------------------- */

/* scale = inv(sqrt(sum(abs2, v) / width + eps)), src/backbone_cpu.jl:344 */
static float rms_scale_f32(const float *v, int64_t width, float eps) {
    double acc = 0.0;
    for (int64_t i = 0; i < width; ++i) acc += (double)v[i] * (double)v[i];
    float total = (float)acc;
    float mean = total / (float)width;
    float shifted = mean + eps;
    float root = sqrtf(shifted);
    return 1.0f / root;
}

static inline float gamma_term(const float *w, int64_t i, int centered) {
    return centered ? 1.0f + w[i] : w[i];
}

/* ---- gather, src/backbone.jl:55-64 -------------------------------------- */

static int ids_in_range(const int32_t *ids, int64_t n, int64_t vocab) {
    for (int64_t t = 0; t < n; ++t)
        if (ids[t] < 0 || (int64_t)ids[t] >= vocab) return 0;
    return 1;
}

int qdo_gather_f32(float *out, const float *table, const int32_t *ids,
                   int64_t n, int64_t hidden, int64_t vocab) {
    if (!ids_in_range(ids, n, vocab)) return -1; /* checkbounds, :60 */
    for (int64_t t = 0; t < n; ++t)
        memcpy(out + t * hidden, table + (int64_t)ids[t] * hidden,
               (size_t)hidden * sizeof(float));
    return 0;
}

int qdo_gather_bf16(uint16_t *out, const uint16_t *table, const int32_t *ids,
                    int64_t n, int64_t hidden, int64_t vocab) {
    if (!ids_in_range(ids, n, vocab)) return -1;
    for (int64_t t = 0; t < n; ++t)
        memcpy(out + t * hidden, table + (int64_t)ids[t] * hidden,
               (size_t)hidden * sizeof(uint16_t));
    return 0;
}

/* ---- RMSNorm, src/backbone_cpu.jl:333-350 / :352-362 -------------------- */

void qdo_rms(float *out, const float *in, const float *weight, float eps,
             int centered, int64_t rows, int64_t width, int64_t ld_in,
             int64_t ld_out) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
    for (int64_t t = 0; t < rows; ++t) {
        const float *x = in + t * ld_in;
        float *y = out + t * ld_out;
        float scale = rms_scale_f32(x, width, eps);
        for (int64_t i = 0; i < width; ++i)
            y[i] = (x[i] * scale) * gamma_term(weight, i, centered);
    }
}

/* ---- residual + RMSNorm, src/backbone_cpu.jl:321-328 -------------------- */

static void residual_rms_row(float *r_out, float *y, const float *x,
                             const float *m, const float *weight, float eps,
                             int centered, int64_t width, float *scratch) {
    for (int64_t i = 0; i < width; ++i)
        scratch[i] = m ? x[i] + m[i] : x[i]; /* residual .= x .+ mixed */
    float scale = rms_scale_f32(scratch, width, eps);
    for (int64_t i = 0; i < width; ++i)
        y[i] = (scratch[i] * scale) * gamma_term(weight, i, centered);
    if (r_out) memcpy(r_out, scratch, (size_t)width * sizeof(float));
}

void qdo_residual_rms(float *out_r, float *out_y, const float *x,
                      const float *m, const float *weight, float eps,
                      int centered, int64_t rows, int64_t width, int64_t ld_x,
                      int64_t ld_m, int64_t ld_r, int64_t ld_y) {
#pragma omp parallel num_threads(g_threads) if (g_threads > 1)
    {
        float *scratch = (float *)malloc((size_t)width * sizeof(float));
#pragma omp for schedule(static)
        for (int64_t t = 0; t < rows; ++t)
            residual_rms_row(out_r ? out_r + t * ld_r : NULL, out_y + t * ld_y,
                             x + t * ld_x, m ? m + t * ld_m : NULL, weight,
                             eps, centered, width, scratch);
        free(scratch);
    }
}

void qdo_residual_rms_bf16(uint16_t *out_r, uint16_t *out_y, const uint16_t *x,
                           const uint16_t *m, const float *weight, float eps,
                           int centered, int64_t rows, int64_t width,
                           int64_t ld_x, int64_t ld_m, int64_t ld_r,
                           int64_t ld_y) {
#pragma omp parallel num_threads(g_threads) if (g_threads > 1)
    {
        float *r = (float *)malloc((size_t)width * sizeof(float));
#pragma omp for schedule(static)
        for (int64_t t = 0; t < rows; ++t) {
            const uint16_t *xr = x + t * ld_x;
            const uint16_t *mr = m ? m + t * ld_m : NULL;
            for (int64_t i = 0; i < width; ++i)
                r[i] = mr ? qdo_bf16_decode(xr[i]) + qdo_bf16_decode(mr[i])
                          : qdo_bf16_decode(xr[i]);
            float scale = rms_scale_f32(r, width, eps);
            uint16_t *yr = out_y + t * ld_y;
            for (int64_t i = 0; i < width; ++i)
                yr[i] = qdo_bf16_encode((r[i] * scale) *
                                        gamma_term(weight, i, centered));
            if (out_r)
                for (int64_t i = 0; i < width; ++i)
                    out_r[t * ld_r + i] = qdo_bf16_encode(r[i]);
        }
        free(r);
    }
}

/* ---- gather + residual + RMSNorm ---------------------------------------- */

int qdo_gather_rms_f32(float *out_r, float *out_y, const float *table,
                       const int32_t *ids, const float *m, const float *weight,
                       float eps, int centered, int64_t n, int64_t hidden,
                       int64_t vocab) {
    if (!ids_in_range(ids, n, vocab)) return -1;
#pragma omp parallel num_threads(g_threads) if (g_threads > 1)
    {
        float *scratch = (float *)malloc((size_t)hidden * sizeof(float));
#pragma omp for schedule(static)
        for (int64_t t = 0; t < n; ++t)
            residual_rms_row(out_r ? out_r + t * hidden : NULL,
                             out_y + t * hidden,
                             table + (int64_t)ids[t] * hidden,
                             m ? m + t * hidden : NULL, weight, eps, centered,
                             hidden, scratch);
        free(scratch);
    }
    return 0;
}

int qdo_gather_rms_bf16(uint16_t *out_r, uint16_t *out_y,
                        const uint16_t *table, const int32_t *ids,
                        const uint16_t *m, const float *weight, float eps,
                        int centered, int64_t n, int64_t hidden,
                        int64_t vocab) {
    if (!ids_in_range(ids, n, vocab)) return -1;
#pragma omp parallel num_threads(g_threads) if (g_threads > 1)
    {
        float *r = (float *)malloc((size_t)hidden * sizeof(float));
#pragma omp for schedule(static)
        for (int64_t t = 0; t < n; ++t) {
            const uint16_t *e = table + (int64_t)ids[t] * hidden;
            const uint16_t *mr = m ? m + t * hidden : NULL;
            for (int64_t i = 0; i < hidden; ++i)
                r[i] = mr ? qdo_bf16_decode(e[i]) + qdo_bf16_decode(mr[i])
                          : qdo_bf16_decode(e[i]);
            float scale = rms_scale_f32(r, hidden, eps);
            for (int64_t i = 0; i < hidden; ++i)
                out_y[t * hidden + i] = qdo_bf16_encode(
                    (r[i] * scale) * gamma_term(weight, i, centered));
            if (out_r)
                for (int64_t i = 0; i < hidden; ++i)
                    out_r[t * hidden + i] = qdo_bf16_encode(r[i]);
        }
        free(r);
    }
    return 0;
}

/* ---- RoPE tables, src/backbone_cpu.jl:90-105 ---------------------------- */

void qdo_rope_table(float theta, int rotary, int64_t n, float *cos_out,
                    float *sin_out) {
    int half = rotary / 2;
    for (int j = 0; j < half; ++j) {
        /* Float32.(0:2:(r-1)) ./ Float32(r): one Float32 division */
        float exponent = (float)(2 * j) / (float)rotary;
        /* Float32 ^: evaluated in double, rounded once */
        float power = (float)pow((double)theta, (double)exponent);
        float freq = 1.0f / power; /* inv.() */
        for (int64_t p = 0; p < n; ++p) {
            float angle = freq * (float)p; /* frequencies .* Float32(pos) */
            cos_out[p * half + j] = (float)cos((double)angle);
            sin_out[p * half + j] = (float)sin((double)angle);
        }
    }
}

/* ---- q/k norm + partial RoPE, src/backbone_cpu.jl:113-136 --------------- */

void qdo_qk_norm_rope(float *out, const float *in, int64_t tokens, int heads,
                      int dim, int64_t in_tok, int64_t in_head,
                      const float *weight, float eps, int rotary,
                      const float *cos_tab, const float *sin_tab,
                      int64_t pos_offset, int64_t seq_len) {
    int half = rotary / 2;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
    for (int64_t t = 0; t < tokens; ++t) {
        int64_t pos = pos_offset + (seq_len > 0 ? t % seq_len : t);
        const float *c = cos_tab + pos * half;
        const float *s = sin_tab + pos * half;
        for (int h = 0; h < heads; ++h) {
            const float *x = in + t * in_tok + (int64_t)h * in_head;
            float *y = out + (t * heads + h) * (int64_t)dim;
            /* cpu_full_rms!, :113-123 */
            float scale = rms_scale_f32(x, dim, eps);
            for (int i = 0; i < dim; ++i)
                y[i] = (x[i] * scale) * (1.0f + weight[i]);
            /* cpu_full_rope!, :125-136 (in place) */
            for (int i = 0; i < half; ++i) {
                float a = y[i], b = y[half + i];
                float ac = a * c[i], bs = b * s[i];
                float bc = b * c[i], as = a * s[i];
                y[i] = ac - bs;
                y[half + i] = bc + as;
            }
        }
    }
}

/* ---- gated RMSNorm, src/backbone_cpu.jl:750-755 ------------------------- */

void qdo_gated_rms(float *out, const float *o, const float *z, int64_t rows,
                   int heads, int dim, int64_t o_ld, int64_t z_ld,
                   int64_t z_off, int64_t out_ld, const float *weight,
                   float eps) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
    for (int64_t t = 0; t < rows; ++t) {
        for (int h = 0; h < heads; ++h) {
            const float *x = o + t * o_ld + (int64_t)h * dim;
            const float *g = z + t * z_ld + z_off + (int64_t)h * dim;
            float *y = out + t * out_ld + (int64_t)h * dim;
            float scale = rms_scale_f32(x, dim, eps);
            for (int i = 0; i < dim; ++i)
                y[i] = ((x[i] * scale) * weight[i]) * qdo_silu(g[i]);
        }
    }
}

/* ---- DeltaNet conv + SiLU + q/k L2 norm ---------------------------------- */

static float conv4_silu(const float *proj, int64_t ld, const float *w, int64_t t,
                        int64_t pos, int64_t c) {
    /* cpu_convolution_four!, src/backbone_cpu.jl:787-807: value starts at
     * the zero-filled output and takes the taps oldest first. */
    float value = 0.0f;
    for (int j = 0; j < 4; ++j) {
        int64_t lag = 3 - j;
        if (pos - lag < 0) continue;
        value = value + proj[(t - lag) * ld + c] * w[c * 4 + j];
    }
    return qdo_silu(value);
}

void qdo_delta_conv_norm(float *q_out, float *k_out, float *v_out,
                         const float *proj, int64_t ld, const float *conv_w,
                         int64_t tokens, int64_t seq_len, int kh, int kd,
                         int vh, int vd, float eps) {
    const int64_t kw = (int64_t)kh * kd;
    const float qmult = sqrtf((float)kd);
#pragma omp parallel num_threads(g_threads) if (g_threads > 1)
    {
        float *buf = (float *)malloc((size_t)(kd > vd ? kd : vd) * sizeof(float));
#pragma omp for schedule(static)
        for (int64_t t = 0; t < tokens; ++t) {
            int64_t pos = seq_len > 0 ? t % seq_len : t;
            for (int g = 0; g < 2; ++g) {          /* q heads, then k heads */
                float *out = g == 0 ? q_out : k_out;
                float mult = g == 0 ? qmult : 1.0f;
                for (int h = 0; h < kh; ++h) {
                    int64_t base = g * kw + (int64_t)h * kd;
                    double acc = 0.0;
                    for (int i = 0; i < kd; ++i) {
                        buf[i] = conv4_silu(proj, ld, conv_w, t, pos, base + i);
                        acc += (double)buf[i] * (double)buf[i];
                    }
                    /* inv(sqrt(squared + 1f-6) * multiplier), :421 */
                    float scale = 1.0f / (sqrtf((float)acc + eps) * mult);
                    float *dst = out + (t * kh + h) * (int64_t)kd;
                    for (int i = 0; i < kd; ++i) dst[i] = buf[i] * scale;
                }
            }
            for (int h = 0; h < vh; ++h) {
                int64_t base = 2 * kw + (int64_t)h * vd;
                float *dst = v_out + (t * vh + h) * (int64_t)vd;
                for (int i = 0; i < vd; ++i)
                    dst[i] = conv4_silu(proj, ld, conv_w, t, pos, base + i);
            }
        }
        free(buf);
    }
}

/* ---- attention output gate, src/backbone.jl:258-259 ----------------------- */

void qdo_attn_gate(float *out, const float *values, const float *gate,
                   int64_t batch, int64_t seq, int heads, int dim, int64_t v_b,
                   int64_t v_h, int64_t v_s, int64_t g_t, int64_t g_h,
                   int64_t out_t) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
    for (int64_t t = 0; t < batch * seq; ++t) {
        int64_t b = t / seq, s = t % seq;
        for (int h = 0; h < heads; ++h)
            for (int d = 0; d < dim; ++d) {
                float g = gate[t * g_t + (int64_t)h * g_h + d];
                float sig = 1.0f / (1.0f + expf(-g)); /* native_sigmoid, :196 */
                out[t * out_t + (int64_t)h * dim + d] =
                    values[b * v_b + (int64_t)h * v_h + s * v_s + d] * sig;
            }
    }
}

/* ---- DeltaNet gates, src/backbone.jl:292-297 ---------------------------- */

void qdo_delta_gates(float *beta, float *decay, const float *proj, int64_t ld,
                     int64_t start, const float *a_decay, const float *dt_bias,
                     int64_t tokens, int heads) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
    for (int64_t t = 0; t < tokens; ++t) {
        const float *row = proj + t * ld + start;
        for (int h = 0; h < heads; ++h) {
            float a = row[h] + dt_bias[h];   /* native_linear(a) .+ dt_bias */
            float b = row[heads + h];
            beta[t * heads + h] = 1.0f / (1.0f + expf(-b)); /* native_sigmoid, :196 */
            /* native_softplus, :198 */
            float sp = fmaxf(a, 0.0f) + log1pf(expf(-fabsf(a)));
            decay[t * heads + h] = a_decay[h] * sp;
        }
    }
}

/* ---- SwiGLU, src/backbone.jl:352-355 ------------------------------------ */

void qdo_swiglu(float *out_f32, uint16_t *out_bf16, const float *g,
                const float *u, int64_t rows, int64_t width, int64_t ld_g,
                int64_t ld_u, int64_t ld_out) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
    for (int64_t t = 0; t < rows; ++t) {
        const float *gr = g + t * ld_g;
        const float *ur = u + t * ld_u;
        for (int64_t i = 0; i < width; ++i) {
            float h = qdo_silu(gr[i]) * ur[i];
            if (out_f32) out_f32[t * ld_out + i] = h;
            if (out_bf16) out_bf16[t * ld_out + i] = qdo_bf16_encode(h);
        }
    }
}

/* ---- delta_solve, src/backbone.jl:279 ----------------------------------- */

void qdo_unit_lower_solve(float *x, const float *l, int64_t batch, int n,
                          int64_t width, int64_t ld_l, int64_t l_batch,
                          int64_t ld_x, int64_t x_batch) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
    for (int64_t b = 0; b < batch; ++b) {
        const float *lb = l + b * l_batch;
        float *xb = x + b * x_batch;
        for (int64_t j = 0; j < width; ++j)
            for (int i = 1; i < n; ++i) {
                float acc = xb[i * ld_x + j];
                for (int k = 0; k < i; ++k) acc = acc - lb[i * ld_l + k] * xb[k * ld_x + j];
                xb[i * ld_x + j] = acc;
            }
    }
}
