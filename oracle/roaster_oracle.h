/*
 * CPU oracle for the hybrid-attention hot path. TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's CPU arithmetic for the gated full-attention layers
 * and the Gated DeltaNet layers (KKB007X/Roaster, src/model.c and src/kernels.c). It is used by
 * tests/, bench.py's CPU-baseline leg and __graft_entry__.smoke() as the checker. The product
 * path (libroaster_b200.so) never links or calls it.
 *
 * Pinning: every function here is checked against the reference's own code compiled from its
 * sources (oracle/_ref, built by oracle/Makefile) and against the committed golden vectors in
 * tests/golden/ that were produced by that build.
 *
 * Conventions shared with the CUDA path:
 *   - The KV cache is f16 ([capacity][2 kv heads][256], K and V separate). The oracle widens the
 *     cached f16 values to fp32, exactly as the reference would hold them after a widening load.
 *   - The token appended by a decode step is used at fp32 in that step (the reference never
 *     rounds it); the cache receives its f16 rounding for later steps.
 *   - Q and the output gate arrive as per-head rows with a caller-given head stride, so the
 *     interleaved projection layout [Q0|G0|Q1|G1|...] (model.c:801-805) is q = qg, gate = qg+256,
 *     stride 512.
 */
#ifndef ROASTER_ORACLE_H
#define ROASTER_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QH 16          /* attention query heads */
#define ORC_KVH 2          /* attention kv heads */
#define ORC_D 256          /* attention head dim */
#define ORC_DN_KH 16       /* DeltaNet key heads */
#define ORC_DN_VH 32       /* DeltaNet value heads */
#define ORC_DN_D 128       /* DeltaNet head dim */

float    orc_f16_to_f32(uint16_t h);
uint16_t orc_f32_to_f16(float f);           /* round to nearest even */

void orc_rmsnorm(float *out, const float *in, const float *w, size_t n, float eps);
void orc_l2norm(float *out, const float *in, size_t n, float eps);
void orc_rope64(float *x, size_t heads, size_t head_dim, size_t position);

/* One gated-attention decode step for one slot (model.c:783-861 without the projections).
 * q/gate: 16 heads at `qg_stride` floats apart; k_new/v_new: [2][256] raw projections.
 * k_cache/v_cache: f16 [>= length][2][256]; the step attends to the `length` cached tokens plus
 * the new one. out: [16][256] gated output. k_app/v_app (may be NULL): [2][256] fp32 values the
 * step appends (normed + RoPE'd K, raw V). Returns 0, or -1 on bad arguments. */
int orc_attn_decode(const float *q, const float *gate, size_t qg_stride,
                    const float *k_new, const float *v_new,
                    const float *qnorm, const float *knorm,
                    const uint16_t *k_cache, const uint16_t *v_cache,
                    size_t length, size_t position,
                    float *out, float *k_app, float *v_app);

/* Partial softmax state of one slot's decode over cached tokens [t0, t1) only (no new token, no
 * gate): m[16] natural-log max score, l[16] = sum exp(s - m), o[16][256] = normalised output.
 * Used to check the split-KV partials that cross GPUs. */
int orc_attn_decode_partial(const float *q, size_t qg_stride, const float *qnorm,
                            const uint16_t *k_cache, const uint16_t *v_cache,
                            size_t t0, size_t t1, size_t position,
                            float *m, float *l, float *o);

/* Causal prefill of T tokens for one slot (model.c:1536-1602 without the projections).
 * q/gate: token t, head h at q + t*qg_tok_stride + h*qg_stride. k/v: [T][2][256] raw.
 * The window already holds `kbase` cached tokens (f16); token t sits at RoPE position base+t
 * and attends to cache entries [0, kbase+t]. out: [T][16][256]. k_app/v_app (may be NULL):
 * [T][2][256] fp32 appended values. Multithreaded with OpenMP over (token, head). */
int orc_attn_prefill(size_t T, const float *q, const float *gate, size_t qg_stride,
                     size_t qg_tok_stride, const float *k, const float *v,
                     const float *qnorm, const float *knorm,
                     const uint16_t *k_cache, const uint16_t *v_cache,
                     size_t kbase, size_t base,
                     float *out, float *k_app, float *v_app);

/* Same as orc_attn_prefill but computes the outputs of the `nrows` tokens listed in `rows`
 * only (out: [nrows][16][256]); every token's K is still prepared and appended. For checking
 * long prompts on a sample of rows. */
int orc_attn_prefill_rows(size_t T, const float *q, const float *gate, size_t qg_stride,
                          size_t qg_tok_stride, const float *k, const float *v,
                          const float *qnorm, const float *knorm,
                          const uint16_t *k_cache, const uint16_t *v_cache,
                          size_t kbase, size_t base, const long *rows, size_t nrows, float *out);

/* One Gated DeltaNet decode step (model.c:272-323). state: [32][128][128], updated in place.
 * q,k: [16][128]; v: [32][128]; g: [32] log-decay; beta: [32]; out: [32][128]. */
void orc_delta_step(float *state, const float *q, const float *k, const float *v,
                    const float *g, const float *beta, float *out);

/* T sequential steps of the same recurrence (model.c:1644-1658 + delta_head 1507-1534).
 * q,k: [T][16][128]; v: [T][32][128]; g, beta: [T][32]; out: [T][32][128]. OpenMP over heads. */
void orc_delta_prefill(float *state, size_t T, const float *q, const float *k, const float *v,
                       const float *g, const float *beta, float *out);

/* Pre-ops of one recurrent layer for T consecutive tokens (model.c:1293-1328 per token; pf_ssm
 * 1619-1643): causal conv1d over the 3-token history + SiLU, history shift, q/k L2-norm, beta
 * sigmoid, g = a softplus(alpha + dt). qkv [T][8192]; alpha, beta [T][32]; conv_state [3][8192]
 * (updated); conv_w [8192][4]; dt, a [32]. Out: q, k [T][16][128], v [T][32][128], g, b [T][32]. */
void orc_delta_preop(size_t T, const float *qkv, const float *alpha, const float *beta,
                     float *conv_state, const float *conv_w, const float *dt, const float *a,
                     float *q, float *k, float *v, float *g, float *b);

/* Gated RMSNorm post-op (model.c:1333-1343) over `rows` rows of 128, in place. */
void orc_delta_postop(size_t rows, float *out, const float *z, const float *w);

/* k-quant matrix-vector product (matvec_q4_cpu / matvec_q6_cpu, kernels.c:405-431, 553-578):
 * out[r] = sum of the dequantised row r (Q4_K 144-byte or Q6_K 210-byte blocks of 256) times x. */
void orc_matvec_q(int is_q6, const uint8_t *m, const float *x, float *out, size_t rows, size_t cols);

#ifdef __cplusplus
}
#endif
#endif
