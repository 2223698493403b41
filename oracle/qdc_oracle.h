/*
 * qdc_oracle.h -- CPU restatement of QwenDecisionCore.jl's per-layer row ops.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * B200 kernels in libqdc_b200.so and the timed CPU baseline of bench.py.
 * Product code never links or calls it; only tests/, __graft_entry__.smoke()
 * and bench.py's CPU legs do.
 *
 * Every function restates one reference routine with Float32 storage and
 * Float32 arithmetic in the reference's operation order; each cites the
 * Julia file:line it follows (paths inside the QwenDecisionCore.jl project).
 * Sums of squares are accumulated in double and rounded once, because
 * Julia's pairwise Float32 `sum` order is not reproducible from C; the
 * difference is far below the 1e-5 relative parity tolerance.
 *
 * Layouts are the reference's column-major Julia matrices seen as row-major
 * C arrays: a Julia (width, tokens) matrix is `[tokens][width]` here, with
 * a leading dimension (elements between consecutive tokens).
 *
 * Parity pin: the whole tiny-model forward built on these ops (oracle/forward.py)
 * reproduces the reference's own golden logits (test/fixtures/native/
 * reference.json, 2e-5) -- see tests/test_oracle_golden.py.
 */
#ifndef QDC_ORACLE_H
#define QDC_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Threads used by the OpenMP loops below (1 = the reference's serial loops). */
void qdo_set_threads(int threads);
int qdo_get_threads(void);

/* bfloat16 storage convention, src/safetensors.jl:28-30 (decode bits<<16)
 * and :38-42 (round to nearest even by integer add, no NaN special case). */
float qdo_bf16_decode(uint16_t bits);
uint16_t qdo_bf16_encode(float value);
void qdo_bf16_encode_array(uint16_t *out, const float *in, int64_t n);
void qdo_bf16_decode_array(float *out, const uint16_t *in, int64_t n);

/* SiLU, src/backbone.jl:196-197: x * inv(1 + exp(-x)). */
float qdo_silu(float x);

/* Token-embedding gather, src/backbone.jl:55-64 (checkbounds -> -1).
 * table is [vocab][hidden] (Julia (hidden, vocab)); ids are 0-based. */
int qdo_gather_f32(float *out, const float *table, const int32_t *ids,
                   int64_t n, int64_t hidden, int64_t vocab);
int qdo_gather_bf16(uint16_t *out, const uint16_t *table, const int32_t *ids,
                    int64_t n, int64_t hidden, int64_t vocab);

/* RMSNorm, src/backbone_cpu.jl:333-350 (centered: *(1+w)) and
 * src/backbone_cpu.jl:352-362 / src/backbone.jl:200-204 (uncentered: *w).
 * out may alias in. */
void qdo_rms(float *out, const float *in, const float *weight, float eps,
             int centered, int64_t rows, int64_t width, int64_t ld_in,
             int64_t ld_out);

/* Residual add + RMSNorm, src/backbone_cpu.jl:321-328 and
 * src/backbone.jl:347-350: r = x + m (stored when out_r != NULL),
 * y = rms(r).  m == NULL means r = x (plain RMSNorm of x). */
void qdo_residual_rms(float *out_r, float *out_y, const float *x,
                      const float *m, const float *weight, float eps,
                      int centered, int64_t rows, int64_t width, int64_t ld_x,
                      int64_t ld_m, int64_t ld_r, int64_t ld_y);

/* bf16-stored variant: inputs decoded, Float32 math, outputs encoded. */
void qdo_residual_rms_bf16(uint16_t *out_r, uint16_t *out_y, const uint16_t *x,
                           const uint16_t *m, const float *weight, float eps,
                           int centered, int64_t rows, int64_t width,
                           int64_t ld_x, int64_t ld_m, int64_t ld_r,
                           int64_t ld_y);

/* Gather fused with (optional) residual add and the input RMSNorm:
 * r = E[id] (+ m), y = rms(r).  Composition of src/backbone.jl:55-64 with
 * src/backbone_cpu.jl:321-328 / :333-350. */
int qdo_gather_rms_f32(float *out_r, float *out_y, const float *table,
                       const int32_t *ids, const float *m, const float *weight,
                       float eps, int centered, int64_t n, int64_t hidden,
                       int64_t vocab);
int qdo_gather_rms_bf16(uint16_t *out_r, uint16_t *out_y,
                        const uint16_t *table, const int32_t *ids,
                        const uint16_t *m, const float *weight, float eps,
                        int centered, int64_t n, int64_t hidden,
                        int64_t vocab);

/* RoPE tables, src/backbone_cpu.jl:90-105: freq_j = inv(theta^(2j/r)),
 * angle = freq_j * pos (one Float32 multiply), cos/sin rounded to Float32.
 * Output [n][rotary/2] each. */
void qdo_rope_table(float theta, int rotary, int64_t n, float *cos_out,
                    float *sin_out);

/* Per-head q/k RMSNorm (centered), src/backbone_cpu.jl:113-123, then the
 * rotate-half partial RoPE of src/backbone_cpu.jl:125-136 on the first
 * `rotary` dims.  Input head h of token t starts at
 * in + t*in_tok + h*in_head (so q can be read straight out of the packed
 * [q;gate] projection, src/backbone.jl:226-227).  Output is dense
 * [tokens][heads][dim].  Position of token t: pos_offset + t % seq_len,
 * the row of the tables. */
void qdo_qk_norm_rope(float *out, const float *in, int64_t tokens, int heads,
                      int dim, int64_t in_tok, int64_t in_head,
                      const float *weight, float eps, int rotary,
                      const float *cos_tab, const float *sin_tab,
                      int64_t pos_offset, int64_t seq_len);

/* Gated RMSNorm of the Gated DeltaNet output, src/backbone_cpu.jl:750-755
 * (and :670-674): y = ((o*s)*w)*silu(z), uncentered w.  o head h of token t
 * at o + t*o_ld + h*dim; z at z + t*z_ld + z_off + h*dim (the packed
 * projection layout of ext/cuda_delta.jl:232-241); out at t*out_ld + h*dim. */
void qdo_gated_rms(float *out, const float *o, const float *z, int64_t rows,
                   int heads, int dim, int64_t o_ld, int64_t z_ld,
                   int64_t z_off, int64_t out_ld, const float *weight,
                   float eps);

/* DeltaNet prologue on the packed projection rows (channels
 * [q (kh*kd) | k (kh*kd) | v (vh*vd)] at the start of each row, leading
 * dimension ld): the 4-tap causal depthwise conv of src/backbone_cpu.jl:
 * 787-807 (taps accumulated oldest first into a zero, each product and sum
 * rounded; taps before the token's sequence start are absent), SiLU
 * (src/backbone.jl:196-197), then the per-head L2 normalisation of
 * src/backbone_cpu.jl:411-427 for q (multiplier sqrt(Float32(kd))) and k
 * (multiplier 1): x * inv(sqrt(sum(x^2) + eps) * multiplier).  v is only
 * activated.  Sequences of seq_len tokens are packed back to back.
 * conv_w is [channels][4] (torch conv1d weight (C, 1, 4)). */
void qdo_delta_conv_norm(float *q_out, float *k_out, float *v_out,
                         const float *proj, int64_t ld, const float *conv_w,
                         int64_t tokens, int64_t seq_len, int kh, int kd,
                         int vh, int vd, float eps);

/* Attention output gate, src/backbone.jl:258-259 (src/backbone_cpu.jl:55-56):
 * out[t][h][d] = values * inv(1 + exp(-gate)).  values element (b, h, s, d)
 * at values + b*v_b + h*v_h + s*v_s + d (t = b*seq + s); gate at
 * gate + t*g_t + h*g_h + d (the gate half of the packed [q;gate] rows);
 * out at out + t*out_t + h*dim + d. */
void qdo_attn_gate(float *out, const float *values, const float *gate,
                   int64_t batch, int64_t seq, int heads, int dim, int64_t v_b,
                   int64_t v_h, int64_t v_s, int64_t g_t, int64_t g_h,
                   int64_t out_t);

/* Gated DeltaNet gates, src/backbone.jl:292-297 (delta_gates_kernel!,
 * ext/cuda_delta.jl:168-181): beta = inv(1 + exp(-b)), decay = a_decay *
 * softplus(a + dt_bias), softplus(x) = max(x, 0) + log1p(exp(-|x|))
 * (:196-198).  a of token t, head h at proj[t*ld + start + h], b at
 * proj[t*ld + start + heads + h]; beta, decay dense [tokens][heads]. */
void qdo_delta_gates(float *beta, float *decay, const float *proj, int64_t ld,
                     int64_t start, const float *a_decay, const float *dt_bias,
                     int64_t tokens, int heads);

/* SwiGLU, src/backbone.jl:352-355: h = silu(g) * u; optional fp32 and/or
 * bf16 (src/safetensors.jl:38-42) outputs. */
/* delta_solve, src/backbone.jl:279: X_b <- UnitLowerTriangular(L_b) \ X_b
 * (forward substitution, k ascending, separately rounded Float32 multiply
 * and subtract; only the strict lower triangle of L_b is read). */
void qdo_unit_lower_solve(float *x, const float *l, int64_t batch, int n,
                          int64_t width, int64_t ld_l, int64_t l_batch,
                          int64_t ld_x, int64_t x_batch);

void qdo_swiglu(float *out_f32, uint16_t *out_bf16, const float *g,
                const float *u, int64_t rows, int64_t width, int64_t ld_g,
                int64_t ld_u, int64_t ld_out);

#ifdef __cplusplus
}
#endif
#endif
