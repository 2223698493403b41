/*
 * qdc_b200.h -- C ABI of libqdc_b200.so, the B200 (sm_100a) implementation of
 * QwenDecisionCore.jl's memory-bound per-layer row ops.
 *
 * Every entry point replaces one hook that the reference's CUDA extension
 * overrides through Julia multiple dispatch; the hook is cited (file:line
 * inside the QwenDecisionCore.jl project) beside each declaration.  The
 * reference binds its GPU code with CUDA.jl `@cuda` launches; a Julia
 * extension binds this library with `ccall`
 * (qwendecisioncore.jl_b200/julia/QwenDecisionCoreB200Ext.jl).
 *
 * Conventions
 *  - Layouts are the reference's column-major Julia matrices seen row-major:
 *    a Julia (width, tokens) Float32 matrix is `[tokens][width]` here.  Each
 *    row operand carries a leading dimension `ld_*` in ELEMENTS.
 *  - Device pointers are owned by the caller; the library never frees them.
 *    `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are
 *    stream-ordered and asynchronous unless stated otherwise.
 *  - Every call returns a qdc_status.  Arguments are validated on the host
 *    before anything is launched; on error nothing is launched and
 *    qdc_last_error() describes the failure.  No kernel traps: an
 *    out-of-vocabulary id that reaches the device raises a flag that
 *    qdc_sync() reports as QDC_EBOUNDS.
 *  - One context serves one host thread at a time (as the reference's
 *    per-model workspace lock, ext/cuda_workspace.jl:48-69); different
 *    contexts may be used concurrently.
 *  - Float32 arithmetic follows the reference's CPU operation order
 *    (src/backbone_cpu.jl) with separately rounded multiplies and adds;
 *    bf16 storage follows src/safetensors.jl:28-30,38-42.
 */
#ifndef QDC_B200_H
#define QDC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QDC_B200_ABI_VERSION 1

#if defined(__GNUC__)
#define QDC_API __attribute__((visibility("default")))
#else
#define QDC_API
#endif

typedef enum qdc_status {
    QDC_OK = 0,
    QDC_EINVAL = 1,   /* bad shape, null/misaligned pointer, bad dtype */
    QDC_EBOUNDS = 2,  /* token id outside the vocabulary */
    QDC_ECUDA = 3,    /* a CUDA runtime call failed */
    QDC_ENOMEM = 4,   /* workspace exhausted or device allocation failed */
    QDC_EDEVICE = 5   /* device is not a compute capability 10.0 GPU */
} qdc_status;

typedef enum qdc_dtype {
    QDC_F32 = 0,      /* Float32 storage */
    QDC_BF16 = 1      /* bfloat16 storage (uint16 bits), Float32 math */
} qdc_dtype;

typedef struct qdc_ctx qdc_ctx;

/* ---- library / context ---------------------------------------------------- */

QDC_API int qdc_abi_version(void);
QDC_API const char *qdc_status_string(int status);

/* Create a context bound to CUDA device `device`: the owner of a forward's
 * workspace arena and device error flag.  Replaces the per-model
 * ForwardWorkspace of ext/cuda_workspace.jl:4-46. */
QDC_API int qdc_init(int device, qdc_ctx **out);
QDC_API int qdc_destroy(qdc_ctx *ctx);

/* Context options (value 0 = off, nonzero = on); QDC_EINVAL for an unknown
 * option.
 * QDC_OPT_PDL (default on): launch this context's kernels with programmatic
 * dependent launch, so a kernel's CTAs may become resident while the
 * preceding kernel drains; every kernel still waits for its predecessor grid
 * to complete before it touches global memory.  It saves the launch latency
 * at each boundary between two of this library's kernels: 2% of a 24-layer
 * step at 8,192 tokens, 0.2% at 65,536. */
#define QDC_OPT_PDL 1
QDC_API int qdc_set_option(qdc_ctx *ctx, int option, int value);

/* Text of the last failure on this context (or on this thread, ctx NULL). */
QDC_API const char *qdc_last_error(const qdc_ctx *ctx);

/* Synchronize `stream`, then report QDC_EBOUNDS (and clear the flag) if a
 * kernel saw an out-of-vocabulary id since the last call.  Replaces the
 * synchronize in native_forward_scope's `finally`, ext/cuda_workspace.jl:62-66. */
QDC_API int qdc_sync(qdc_ctx *ctx, void *stream);

/* ---- workspace arena -------------------------------------------------------
 * Bump allocator over one device allocation per context, reused forward after
 * forward.  Replaces the slot list `scratch(T, dims)` of
 * ext/cuda_workspace.jl:71-87 and the cursor reset of :57-59. */

/* Ensure capacity >= bytes.  Growing frees and reallocates the arena, which
 * invalidates every pointer handed out before; it synchronizes the device. */
QDC_API int qdc_ws_reserve(qdc_ctx *ctx, size_t bytes);
/* Carve `bytes` (rounded up to `align`, a power of two >= 256 or 0 for 256). */
QDC_API int qdc_ws_alloc(qdc_ctx *ctx, size_t bytes, size_t align, void **out);
/* Current cursor, and pop back to a cursor taken earlier. */
QDC_API int qdc_ws_mark(qdc_ctx *ctx, size_t *mark);
QDC_API int qdc_ws_release(qdc_ctx *ctx, size_t mark);
/* cursor = 0: the start of a forward (native_forward_scope, :57-58). */
QDC_API int qdc_ws_reset(qdc_ctx *ctx);
QDC_API int qdc_ws_stats(const qdc_ctx *ctx, size_t *used, size_t *capacity,
                 size_t *high_water);

/* ---- host tables -------------------------------------------------------------
 * RoPE cos/sin tables exactly as src/backbone_cpu.jl:90-105 builds them:
 * freq_j = inv(theta^(Float32(2j)/Float32(rotary))), angle = freq_j*Float32(p)
 * (one Float32 multiply), cos/sin of the Float32 angle rounded to Float32.
 * Fills host arrays [n][rotary/2].  Pure host code; no context needed. */
QDC_API int qdc_rope_table(float theta, int rotary, int64_t n, float *cos_host,
                   float *sin_host);

/* ---- per-layer row kernels ----------------------------------------------- */

/* Token-embedding gather fused with an optional residual add and the input
 * RMSNorm:  r_t = E[ids_t] (+ add_t);  y_t = rms(r_t) * (1+g | g).
 *   table   [vocab][hidden] (Julia (hidden, vocab)), dtype storage
 *   ids     HOST int32[n], 0-based; validated before launch (QDC_EBOUNDS,
 *           src/backbone.jl:417-418) and staged into the context workspace
 *           (the reference stages them the same way, ext/cuda_workspace.jl:333-334)
 *   add     optional [n][hidden] residual (NULL: none)
 *   out_x   optional [n][hidden] r (NULL: not stored); with gamma NULL the
 *           call is the plain gather of ext/cuda_workspace.jl:317-344
 *   out_y   [n][hidden] normalized output (NULL allowed only if gamma NULL)
 *   gamma   Float32[hidden] (centered: applied as 1+g, src/backbone_cpu.jl:346)
 * Replaces native_gather (src/backbone.jl:55-64, ext/cuda_workspace.jl:330-344)
 * followed by the first layer's native_rms (src/backbone.jl:364). */
QDC_API int qdc_gather_rms(qdc_ctx *ctx, void *out_x, void *out_y, const void *table,
                   const int32_t *ids, const void *add, const float *gamma,
                   float eps, int centered, int64_t n, int64_t hidden,
                   int64_t vocab, int dtype, void *stream);

/* The plain token-embedding gather, out[t] = table[ids[t]] (bit-exact),
 * host ids validated and staged as in qdc_gather_rms.  Replaces
 * native_gather(::CuMatrix, ids) / gather_kernel! (src/backbone.jl:55-64,
 * ext/cuda_workspace.jl:317-344); the same as qdc_gather_rms with
 * out_y, add and gamma NULL. */
QDC_API int qdc_gather(qdc_ctx *ctx, void *out, const void *table, const int32_t *ids,
                       int64_t n, int64_t hidden, int64_t vocab, int dtype, void *stream);

/* As qdc_gather_rms with DEVICE ids (for graph capture / device-resident
 * batches).  Out-of-range ids are not read: their rows are filled with NaN
 * and the context flag is raised (QDC_EBOUNDS from the next qdc_sync). */
QDC_API int qdc_gather_rms_device_ids(qdc_ctx *ctx, void *out_x, void *out_y,
                              const void *table, const int32_t *ids_dev,
                              const void *add, const float *gamma, float eps,
                              int centered, int64_t n, int64_t hidden,
                              int64_t vocab, int dtype, void *stream);

/* qdc_gather_rms for callers that may not allocate device memory: no
 * context, and no cudaMalloc / cudaFree or allocating library call, ever.
 * No counterpart in the reference -- it exists for hosts whose memory
 * manager owns every device byte (a CUDA.jl pool, a serving arena), loops
 * that cannot take the device-wide synchronisation of cudaMalloc/cudaFree,
 * and deployments with a memory budget fixed at start-up.  The ids are
 * staged in a fixed 256 KiB array inside the library's device image, so a
 * call takes at most 65536 ids (more: QDC_EINVAL).  Runs on the current
 * device.  Its first call there looks the array up (cudaGetSymbolAddress)
 * and, under CUDA's lazy module loading (the default), is when the driver
 * loads the library's module onto that device and commits the array: make
 * that first call at start-up, before any stream capture begins.  The
 * looked-up address is kept for the process; cudaDeviceReset is not
 * supported.  All calls on a device share the array: calls whose work
 * overlaps on the GPU race -- serialise them (calls on one stream are
 * ordered).  Ids are validated on the host (QDC_EBOUNDS); an out-of-range id
 * that racing calls let through reaches the device as a NaN row (there is no
 * device flag).  Errors are reported through qdc_last_error(NULL). */
QDC_API int qdc_gather_rms_noalloc(void *out_x, void *out_y, const void *table,
                                   const int32_t *ids, const void *add,
                                   const float *gamma, float eps, int centered,
                                   int64_t n, int64_t hidden, int64_t vocab,
                                   int dtype, void *stream);

/* Residual add + RMSNorm:  r = x + m (m NULL: r = x);  y = rms(r)*(1+g | g);
 * r stored when out_r != NULL.  One kernel covers
 *  - native_rms (src/backbone.jl:200-204, ext/cuda_workspace.jl:139-170):
 *    m NULL, out_r NULL -- the input norm and the final norm;
 *  - native_residual_rms (src/backbone.jl:347-350, src/backbone_cpu.jl:321-328,
 *    ext/cuda_workspace.jl:179-209): the post-attention norm;
 *  - native_residual_add! (src/backbone.jl:358-361) fused with the NEXT
 *    layer's input norm (or with the final norm, src/backbone.jl:410).
 * out_r may alias x (in-place residual stream); out_y must not alias x/m. */
QDC_API int qdc_residual_rms(qdc_ctx *ctx, void *out_r, void *out_y, const void *x,
                     const void *m, const float *gamma, float eps,
                     int centered, int64_t rows, int64_t width, int64_t ld_x,
                     int64_t ld_m, int64_t ld_r, int64_t ld_y, int dtype,
                     void *stream);

/* Per-head q/k RMSNorm (centered gamma) + rotate-half partial RoPE on the
 * first `rotary` dims; dims >= rotary pass through.  Input head h of token
 * t starts at in + t*in_tok + h*in_head (q straight from the packed [q;gate]
 * projection: in_tok = heads*2*dim, in_head = 2*dim, src/backbone.jl:226-227).
 * Output dense [tokens][heads][dim].  Position of token t:
 * pos_offset + t % seq_len (seq_len <= 0: t), which must be < table_rows.
 * cos_tab/sin_tab: device [table_rows][rotary/2] from qdc_rope_table.
 * Replaces native_rms + native_rope in full_attention (src/backbone.jl:
 * 206-235; CPU src/backbone_cpu.jl:113-136; CUDA prepare_head_kernel!
 * ext/cuda_attention.jl:1-45).  K is written once per kv head, not
 * expanded per query head. */
QDC_API int qdc_qk_norm_rope(qdc_ctx *ctx, float *out, const float *in,
                     int64_t tokens, int heads, int dim, int64_t in_tok,
                     int64_t in_head, const float *gamma, float eps,
                     int rotary, const float *cos_tab, const float *sin_tab,
                     int64_t table_rows, int64_t pos_offset, int64_t seq_len,
                     void *stream);

/* qdc_qk_norm_rope with the output laid out by strides: head h of token t
 * goes to out + t*out_tok + h*out_head (out_tok = heads*dim, out_head = dim
 * is the dense layout above).  out_tok = dim, out_head = tokens*dim writes
 * the head-major (dim, tokens, heads) Julia array that the reference's
 * attention GEMMs read (prepare_head_kernel!, ext/cuda_attention.jl:1-45,
 * 128,141); the heads must not overlap. */
QDC_API int qdc_qk_norm_rope_strided(qdc_ctx *ctx, float *out, const float *in,
                                     int64_t tokens, int heads, int dim, int64_t in_tok,
                                     int64_t in_head, int64_t out_tok, int64_t out_head,
                                     const float *gamma, float eps, int rotary,
                                     const float *cos_tab, const float *sin_tab,
                                     int64_t table_rows, int64_t pos_offset,
                                     int64_t seq_len, void *stream);

/* qdc_qk_norm_rope for the query AND key heads of the same tokens in one
 * launch: q head h of token t at q_in + t*q_tok + h*q_head, k head h at
 * k_in + t*k_tok + h*k_head; outputs dense [tokens][q_heads][dim] and
 * [tokens][k_heads][dim]; q_gamma / k_gamma are the two centered gammas.
 * Replaces the two prepare_head_kernel! launches of full_attention
 * (ext/cuda_attention.jl:128,141); the key heads then cost no launch of
 * their own. */
QDC_API int qdc_q_k_norm_rope(qdc_ctx *ctx, float *q_out, float *k_out,
                              const float *q_in, const float *k_in,
                              int64_t tokens, int q_heads, int k_heads, int dim,
                              int64_t q_tok, int64_t q_head, int64_t k_tok,
                              int64_t k_head, const float *q_gamma,
                              const float *k_gamma, float eps, int rotary,
                              const float *cos_tab, const float *sin_tab,
                              int64_t table_rows, int64_t pos_offset,
                              int64_t seq_len, void *stream);

/* Gated RMSNorm of the Gated DeltaNet output:  y = ((o*s)*g)*silu(z),
 * uncentered gamma (src/backbone.jl:339-341, src/backbone_cpu.jl:750-755).
 * o head h of row t at o + t*o_ld + h*dim; z at z + t*z_ld + z_off + h*dim
 * (z read in place from the packed projection, ext/cuda_delta.jl:232-241);
 * y at out + t*out_ld + h*dim.  Replaces rms_gate_kernel!
 * (ext/cuda_delta.jl:99-116). */
QDC_API int qdc_gated_rms(qdc_ctx *ctx, float *out, const float *o, const float *z,
                  int64_t rows, int heads, int dim, int64_t o_ld, int64_t z_ld,
                  int64_t z_off, int64_t out_ld, const float *gamma,
                  float eps, void *stream);

/* Attention output gate: out[t][h][:] = values * sigmoid(gate) with
 * sigmoid(x) = inv(1 + exp(-x)) (src/backbone.jl:258-259).  values element
 * (b, h, s, d) at values + b*v_b + h*v_h + s*v_s + d -- the (batch, heads,
 * seq, dim) output of an attention kernel, read in place; gate at
 * gate + t*g_t + h*g_h + d with t = b*seq + s (the gate half of the packed
 * [q;gate] projection: g_t = heads*2*dim, g_h = 2*dim, base + dim); out at
 * out + t*out_t + h*dim + d.  Replaces merge_gate_kernel!
 * (ext/cuda_attention.jl:92-108) and the transpose before it. */
QDC_API int qdc_attn_gate(qdc_ctx *ctx, float *out, const float *values,
                          const float *gate, int64_t batch, int64_t seq,
                          int heads, int dim, int64_t v_b, int64_t v_h,
                          int64_t v_s, int64_t g_t, int64_t g_h, int64_t out_t,
                          void *stream);

/* Gated DeltaNet gates for every (token, value head):
 *   beta  = inv(1 + exp(-b)),
 *   decay = a_decay[h] * softplus(a + dt_bias[h]),
 *   softplus(x) = max(x, 0) + log1p(exp(-|x|))
 * (src/backbone.jl:292-297, :196-198).  a of token t, head h at
 * proj[t*ld_proj + start + h], b at proj[t*ld_proj + start + heads + h] (the
 * packed [qkv | z | a | b] projection rows, ext/cuda_mlp.jl:27); a_decay =
 * -exp(A_log) per head; beta and decay are dense [tokens][heads].  Replaces
 * delta_gates_kernel! (ext/cuda_delta.jl:168-181). */
QDC_API int qdc_delta_gates(qdc_ctx *ctx, float *beta, float *decay, const float *proj,
                    int64_t ld_proj, int64_t start, const float *a_decay,
                    const float *dt_bias, int64_t tokens, int heads, void *stream);

/* DeltaNet prologue in one pass over the packed projection: 4-tap causal
 * depthwise conv + SiLU on the [q | k | v] channels at the start of each
 * token row (row t at proj + t*ld_proj), then q and k L2-normalised per head
 * (q also divided by sqrt(key_dim)); eps is the reference's 1e-6.
 * conv_w: [channels][4] (torch conv1d weight (C, 1, 4)).  Tokens are
 * sequences of seq_len packed back to back (0: one sequence); the conv never
 * reaches across a sequence start.  Outputs dense q, k [tokens][key_heads]
 * [key_dim] and v [tokens][value_heads][value_dim].  Replaces
 * causal_depthwise_kernel! + qk_normalize_kernel! (ext/cuda_delta.jl:8-40,
 * 122-146; CPU src/backbone_cpu.jl:787-807, :411-427). */
QDC_API int qdc_delta_conv_norm(qdc_ctx *ctx, float *q_out, float *k_out,
                                float *v_out, const float *proj,
                                int64_t ld_proj, const float *conv_w,
                                int64_t tokens, int64_t seq_len, int key_heads,
                                int key_dim, int value_heads, int value_dim,
                                float eps, void *stream);

/* qdc_delta_conv_norm with v written at v_out + t*v_tok + h*value_dim
 * (v_tok >= value_heads*value_dim): v can go straight into the value rows of
 * the conv output `mixed` that the reference's delta-rule kernels read
 * (v_out = mixed + 2*key_heads*key_dim, v_tok = the qkv width;
 * ext/cuda_delta.jl:199-213). */
QDC_API int qdc_delta_conv_norm_strided(qdc_ctx *ctx, float *q_out, float *k_out,
                                        float *v_out, int64_t v_tok, const float *proj,
                                        int64_t ld_proj, const float *conv_w,
                                        int64_t tokens, int64_t seq_len, int key_heads,
                                        int key_dim, int value_heads, int value_dim,
                                        float eps, void *stream);

/* bf16 storage <-> Float32 on the device, n elements, out and in not
 * overlapping.  qdc_bf16_to_f32: out = bits << 16 (src/safetensors.jl:28-30),
 * exact -- the weight upload path: a checkpoint's raw BF16 bytes are copied
 * to the device and widened there, half the host -> device traffic of the
 * reference's host-side decode (src/safetensors.jl:3-35).  qdc_f32_to_bf16:
 * round to nearest even by integer add, no NaN special case
 * (src/safetensors.jl:38-42), for bf16-stored activations. */
QDC_API int qdc_bf16_to_f32(qdc_ctx *ctx, float *out, const uint16_t *in, int64_t n,
                            void *stream);
QDC_API int qdc_f32_to_bf16(qdc_ctx *ctx, uint16_t *out, const float *in, int64_t n,
                            void *stream);

/* In-place batched solve with unit lower-triangular matrices:
 *   X_b <- (I + strict_lower(L_b))^{-1} X_b,   b = 0 .. batch-1,
 * L_b an n x n matrix (1 <= n <= 64) at l + b*l_batch with row stride ld_l
 * (its diagonal and upper triangle are not read), X_b an n x width matrix
 * at x + b*x_batch with row stride ld_x; the L's and X's must not overlap.
 * Forward substitution in Float32 (fused multiply-adds, k ascending).
 * Replaces delta_solve, the chunked gated delta rule's
 * UnitLowerTriangular(system) \ rhs (src/backbone.jl:279,328-330;
 * CUDA ext/QwenDecisionCoreCUDAExt.jl:22-24), with no solver workspace. */
QDC_API int qdc_unit_lower_solve(qdc_ctx *ctx, float *x, const float *l, int64_t batch,
                                 int n, int64_t width, int64_t ld_l, int64_t l_batch,
                                 int64_t ld_x, int64_t x_batch, void *stream);

/* SwiGLU gate:  h = silu(g) * u  (src/backbone.jl:196-197,352-355).
 * g/u rows at g + t*ld_g, u + t*ld_u (the packed [gate;up] projection of
 * ext/cuda_mlp.jl:63-71 is g = P, u = P + width, ld = 2*width).  Writes
 * Float32 out_f32 and/or bf16 out_bf16 (either may be NULL, not both), both
 * with leading dimension ld_out.  Replaces mlp_gate_kernel!
 * (ext/cuda_mlp.jl:49-61) and native_mlp_gate! (src/backbone.jl:352-355). */
QDC_API int qdc_swiglu(qdc_ctx *ctx, float *out_f32, uint16_t *out_bf16,
               const float *g, const float *u, int64_t rows, int64_t width,
               int64_t ld_g, int64_t ld_u, int64_t ld_out, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* QDC_B200_H */
