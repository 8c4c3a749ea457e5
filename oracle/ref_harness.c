/*
 * Drives the reference's OWN CPU implementation of the hot path (KKB007X/Roaster src/model.c,
 * src/kernels.c lines 1-721), compiled from its sources by oracle/Makefile into
 * oracle/_ref/libroaster_ref.so. TEST INFRASTRUCTURE ONLY (checker and timed CPU baseline).
 *
 * Nothing of the reference is copied here: this file #includes the reference's model.c from
 * the path given to the compiler (-I<reference>/src), which reaches its static functions
 * full_attention (model.c:783-863), pf_attention (1536-1602), recurrent_delta_step (272-323)
 * and delta_head (1507-1534). The reference's kvwindow.c and kvspill.c are compiled alongside
 * (oracle/Makefile) and driven through a small Model rig for the window tests.
 *
 * The attention functions take their inputs through projections. They are driven literally with
 * f32 (GGUF type 0) weight tensors, which the reference multiplies with kernel_matvec_f32
 * (model.c:113-121):
 *   - decode: normed = e0 and column 0 of W_q / W_k / W_v holds the wanted [Q|G], k and v, so the
 *     projections return them exactly; W_o rows are one-hot selectors of the gated output, so
 *     two calls (window length reset in between) read all 4096 values back through `residual`.
 *   - prefill: token t's normed row is e_t, so column t of each W holds token t's projection; the
 *     gated output is read from the prefill scratch (g_pf.rec) before the O projection.
 */
#include "model.c"
#include "kvwindow.h"

#include <stdlib.h>
#include <string.h>

/* ---- link stubs: the hot path never reaches these (quantized / Vulkan / window / weights). */
static void unreachable(const char *what)
{
    fprintf(stderr, "ref_harness: unexpected call to %s\n", what);
    abort();
}
int kernel_ffn_fused(const KernelFfnExpert *e, int n, const float *x, size_t i, size_t h)
{ (void)e; (void)n; (void)x; (void)i; (void)h; unreachable("kernel_ffn_fused"); return 0; }
int kernel_matmul_quant_batch(const KernelMatmulJob *j, int n)
{ (void)j; (void)n; unreachable("kernel_matmul_quant_batch"); return -1; }
void kernel_matvec_q4_k(const void *m, const float *v, float *o, size_t r, size_t c)
{ (void)m; (void)v; (void)o; (void)r; (void)c; unreachable("kernel_matvec_q4_k"); }
void kernel_matvec_q6_k(const void *m, const float *v, float *o, size_t r, size_t c)
{ (void)m; (void)v; (void)o; (void)r; (void)c; unreachable("kernel_matvec_q6_k"); }
void kernel_matvec_quant_batch(const KernelMatvecJob *j, int n)
{ (void)j; (void)n; unreachable("kernel_matvec_quant_batch"); }
int kernel_matvec_quant_begin(const KernelMatvecJob *j, int n)
{ (void)j; (void)n; unreachable("kernel_matvec_quant_begin"); return 0; }
void kernel_matvec_quant_end(void) { unreachable("kernel_matvec_quant_end"); }
int kernel_moe_prefill(const KernelMoeExpert *e, int c, const float *x, float *d, size_t i, size_t h)
{ (void)e; (void)c; (void)x; (void)d; (void)i; (void)h; unreachable("kernel_moe_prefill"); return -1; }
void kernel_vk_trim_scratch(void) {}
TensorInfo *weights_find_tensor(Weights *w, const char *n) { (void)w; (void)n; return NULL; }
CachedExpert *weights_get_expert(Weights *w, int l, int e)
{ (void)w; (void)l; (void)e; unreachable("weights_get_expert"); return NULL; }
int weights_prefetch_experts(Weights *w, int l, const int *ids, int c)
{ (void)w; (void)l; (void)ids; (void)c; unreachable("weights_prefetch_experts"); return -1; }

/* ---- synthetic f32 weights (type 0 = F32 in GGUF) */
#define ATT_LAYER 3                                 /* (3+1) % 4 == 0: a full-attention layer */

static TensorInfo t_q, t_k, t_v, t_o;
static float *W_q, *W_k, *W_v, *W_o;               /* [rows][2048] / [2048][4096] */
static ModelRefs *R;

static int ensure_weights(void)
{
    if (R)
        return 0;
    W_q = calloc((size_t)MODEL_ATTN_Q_SIZE * MODEL_HIDDEN_SIZE, sizeof(float));
    W_k = calloc((size_t)MODEL_ATTN_K_SIZE * MODEL_HIDDEN_SIZE, sizeof(float));
    W_v = calloc((size_t)MODEL_ATTN_V_SIZE * MODEL_HIDDEN_SIZE, sizeof(float));
    W_o = calloc((size_t)MODEL_HIDDEN_SIZE * 4096, sizeof(float));
    R = calloc(1, sizeof(*R));
    if (!W_q || !W_k || !W_v || !W_o || !R)
        return -1;
    t_q.type = t_k.type = t_v.type = t_o.type = 0;
    LayerRefs *L = &R->layer[ATT_LAYER];
    L->q = (TRef){ &t_q, W_q };
    L->k = (TRef){ &t_k, W_k };
    L->v = (TRef){ &t_v, W_v };
    L->o = (TRef){ &t_o, W_o };
    return 0;
}

/* Column `col` of a [rows][2048] matrix := x. */
static void set_col(float *W, size_t rows, size_t col, const float *x)
{
    for (size_t r = 0; r < rows; r++)
        W[r * MODEL_HIDDEN_SIZE + col] = x[r];
}

typedef struct {
    Model m;
    KVCache kv[MODEL_NUM_LAYERS];
    float *normed, *attn_q, *attn_k, *attn_v, *residual;
} Rig;

static int rig_init(Rig *g, size_t capacity, const float *kc, const float *vc, size_t length,
                    const float *qnorm, const float *knorm)
{
    memset(g, 0, sizeof(*g));
    KVCache *kv = &g->kv[ATT_LAYER];
    kv->capacity = capacity;
    kv->k = calloc(capacity * 512, sizeof(float));
    kv->v = calloc(capacity * 512, sizeof(float));
    g->normed = calloc(MODEL_HIDDEN_SIZE, sizeof(float));
    g->attn_q = calloc(MODEL_ATTN_Q_SIZE, sizeof(float));
    g->attn_k = calloc(MODEL_ATTN_K_SIZE, sizeof(float));
    g->attn_v = calloc(MODEL_ATTN_V_SIZE, sizeof(float));
    g->residual = calloc(MODEL_HIDDEN_SIZE, sizeof(float));
    g->m.attn_scratch = calloc(16 * capacity, sizeof(float));
    if (!kv->k || !kv->v || !g->normed || !g->attn_q || !g->attn_k || !g->attn_v ||
        !g->residual || !g->m.attn_scratch)
        return -1;
    if (length) {
        memcpy(kv->k, kc, length * 512 * sizeof(float));
        memcpy(kv->v, vc, length * 512 * sizeof(float));
    }
    kv->length = length;
    R->layer[ATT_LAYER].qnorm = qnorm;
    R->layer[ATT_LAYER].knorm = knorm;
    g->m.kv_cache = g->kv;
    g->m.refs = R;
    g->m.normed = g->normed;
    g->m.attn_q = g->attn_q;
    g->m.attn_k = g->attn_k;
    g->m.attn_v = g->attn_v;
    g->m.residual = g->residual;
    g->m.context_length = capacity;
    g->m.initialized = true;
    return 0;
}

static void rig_free(Rig *g)
{
    free(g->kv[ATT_LAYER].k);
    free(g->kv[ATT_LAYER].v);
    free(g->normed);
    free(g->attn_q);
    free(g->attn_k);
    free(g->attn_v);
    free(g->residual);
    free(g->m.attn_scratch);
}

/* One decode step through full_attention. q_gate: [16][512] interleaved Q|G; k_new, v_new:
 * [512]; kc/vc: fp32 window [length][512]. out: [4096] gated attention output; k_app/v_app:
 * [512] what the step appended. 0 = ok. */
int ref_attn_decode(const float *q_gate, const float *k_new, const float *v_new,
                    const float *qnorm, const float *knorm, const float *kc, const float *vc,
                    size_t length, size_t position, float *out, float *k_app, float *v_app)
{
    if (ensure_weights() != 0)
        return -1;
    Rig g;
    if (rig_init(&g, length + 1, kc, vc, length, qnorm, knorm) != 0) {
        rig_free(&g);
        return -1;
    }
    set_col(W_q, MODEL_ATTN_Q_SIZE, 0, q_gate);
    set_col(W_k, MODEL_ATTN_K_SIZE, 0, k_new);
    set_col(W_v, MODEL_ATTN_V_SIZE, 0, v_new);
    g.normed[0] = 1.0f;
    int rc = 0;
    for (int half = 0; half < 2 && rc == 0; half++) {
        memset(W_o, 0, (size_t)MODEL_HIDDEN_SIZE * 4096 * sizeof(float));
        for (size_t r = 0; r < MODEL_HIDDEN_SIZE; r++)
            W_o[r * 4096 + (size_t)half * MODEL_HIDDEN_SIZE + r] = 1.0f;
        g.kv[ATT_LAYER].length = length;
        g.m.position = position;
        rc = full_attention(&g.m, ATT_LAYER);
        memcpy(out + (size_t)half * MODEL_HIDDEN_SIZE, g.residual, MODEL_HIDDEN_SIZE * sizeof(float));
    }
    if (rc == 0) {
        memcpy(k_app, g.kv[ATT_LAYER].k + length * 512, 512 * sizeof(float));
        memcpy(v_app, g.kv[ATT_LAYER].v + length * 512, 512 * sizeof(float));
    }
    for (size_t r = 0; r < MODEL_ATTN_Q_SIZE; r++)
        W_q[r * MODEL_HIDDEN_SIZE] = 0.0f;
    rig_free(&g);
    return rc;
}

/* Causal prefill of T <= 256 tokens through pf_attention. q_gate: [T][16][512]; k, v: [T][512];
 * kc/vc: fp32 window [kbase][512]. out: [T][4096] gated output; k_app/v_app: [T][512]. */
int ref_attn_prefill(int T, const float *q_gate, const float *k, const float *v,
                     const float *qnorm, const float *knorm, const float *kc, const float *vc,
                     size_t kbase, size_t base, float *out, float *k_app, float *v_app)
{
    if (T <= 0 || T > PF_MAX_T || ensure_weights() != 0)
        return -1;
    Rig g;
    if (rig_init(&g, kbase + (size_t)T, kc, vc, kbase, qnorm, knorm) != 0 ||
        pf_ensure(kbase + (size_t)T) != 0) {
        rig_free(&g);
        return -1;
    }
    memset(g_pf.nrm, 0, (size_t)T * PF_H * sizeof(float));
    for (int t = 0; t < T; t++) {
        g_pf.nrm[(size_t)t * PF_H + (size_t)t] = 1.0f;
        set_col(W_q, MODEL_ATTN_Q_SIZE, (size_t)t, q_gate + (size_t)t * MODEL_ATTN_Q_SIZE);
        set_col(W_k, MODEL_ATTN_K_SIZE, (size_t)t, k + (size_t)t * 512);
        set_col(W_v, MODEL_ATTN_V_SIZE, (size_t)t, v + (size_t)t * 512);
    }
    memset(W_o, 0, (size_t)MODEL_HIDDEN_SIZE * 4096 * sizeof(float));
    int rc = pf_attention(&g.m, ATT_LAYER, T, base);
    if (rc == 0) {
        memcpy(out, g_pf.rec, (size_t)T * 4096 * sizeof(float));
        memcpy(k_app, g.kv[ATT_LAYER].k + kbase * 512, (size_t)T * 512 * sizeof(float));
        memcpy(v_app, g.kv[ATT_LAYER].v + kbase * 512, (size_t)T * 512 * sizeof(float));
    }
    memset(W_q, 0, (size_t)MODEL_ATTN_Q_SIZE * MODEL_HIDDEN_SIZE * sizeof(float));
    memset(W_k, 0, (size_t)MODEL_ATTN_K_SIZE * MODEL_HIDDEN_SIZE * sizeof(float));
    memset(W_v, 0, (size_t)MODEL_ATTN_V_SIZE * MODEL_HIDDEN_SIZE * sizeof(float));
    rig_free(&g);
    return rc;
}

/* A reusable full_attention rig for the timed CPU baseline: the caller fills the fp32 window
 * (ref_decode_ctx_k / _v) once and times ref_decode_ctx_step. full_attention also runs its
 * Q/K/V/O projections as f32 matvecs; ref_decode_ctx_projections runs exactly those four
 * kernel_matvec_f32 calls so the baseline can subtract their time and report the attention
 * work alone. */
typedef struct RefDecodeCtx { Rig g; } RefDecodeCtx;

RefDecodeCtx *ref_decode_ctx_new(size_t capacity, const float *qnorm, const float *knorm)
{
    if (ensure_weights() != 0)
        return NULL;
    RefDecodeCtx *c = calloc(1, sizeof(*c));
    if (!c)
        return NULL;
    if (rig_init(&c->g, capacity, NULL, NULL, 0, qnorm, knorm) != 0) {
        rig_free(&c->g);
        free(c);
        return NULL;
    }
    return c;
}

float *ref_decode_ctx_k(RefDecodeCtx *c) { return c->g.kv[ATT_LAYER].k; }
float *ref_decode_ctx_v(RefDecodeCtx *c) { return c->g.kv[ATT_LAYER].v; }

void ref_decode_ctx_free(RefDecodeCtx *c)
{
    if (!c)
        return;
    rig_free(&c->g);
    free(c);
}

/* Run full_attention once over a window of `length` cached tokens (plus the appended one). */
int ref_decode_ctx_step(RefDecodeCtx *c, size_t length, size_t position)
{
    c->g.kv[ATT_LAYER].length = length;
    c->g.m.position = position;
    c->g.normed[0] = 1.0f;
    return full_attention(&c->g.m, ATT_LAYER);
}

/* The four projection matvecs full_attention issues (model.c:796-800 and 862), same shapes. */
void ref_decode_ctx_projections(RefDecodeCtx *c)
{
    static float qg[MODEL_ATTN_Q_SIZE];
    kernel_matvec_f32(W_q, c->g.normed, qg, MODEL_ATTN_Q_SIZE, MODEL_HIDDEN_SIZE);
    kernel_matvec_f32(W_k, c->g.normed, c->g.attn_k, MODEL_ATTN_K_SIZE, MODEL_HIDDEN_SIZE);
    kernel_matvec_f32(W_v, c->g.normed, c->g.attn_v, MODEL_ATTN_V_SIZE, MODEL_HIDDEN_SIZE);
    kernel_matvec_f32(W_o, qg, c->g.residual, MODEL_HIDDEN_SIZE, 4096);
}

/* A reusable pf_attention rig for the timed prefill CPU baseline (model.c:1536-1602): the caller
 * fills the fp32 window once (ref_prefill_ctx_k / _v) and times ref_prefill_ctx_chunk, one
 * prompt chunk of T <= 256 tokens appended after `kbase` cached tokens. The chunk's normed rows
 * are zero, so its projections return zeros; the attention work does not depend on the values.
 * ref_prefill_ctx_projections runs the same Q/K/V and O projection calls (pf_mm / pf_mm1 on the
 * f32 weights) so the baseline can subtract their time and report the attention work alone. */
typedef struct RefPrefillCtx { Rig g; } RefPrefillCtx;

RefPrefillCtx *ref_prefill_ctx_new(size_t capacity, const float *qnorm, const float *knorm)
{
    if (ensure_weights() != 0 || pf_ensure(capacity) != 0)
        return NULL;
    RefPrefillCtx *c = calloc(1, sizeof(*c));
    if (!c)
        return NULL;
    if (rig_init(&c->g, capacity, NULL, NULL, 0, qnorm, knorm) != 0) {
        rig_free(&c->g);
        free(c);
        return NULL;
    }
    memset(g_pf.nrm, 0, (size_t)PF_MAX_T * PF_H * sizeof(float));
    return c;
}

float *ref_prefill_ctx_k(RefPrefillCtx *c) { return c->g.kv[ATT_LAYER].k; }
float *ref_prefill_ctx_v(RefPrefillCtx *c) { return c->g.kv[ATT_LAYER].v; }

void ref_prefill_ctx_free(RefPrefillCtx *c)
{
    if (!c)
        return;
    rig_free(&c->g);
    free(c);
}

int ref_prefill_ctx_chunk(RefPrefillCtx *c, int T, size_t kbase, size_t base)
{
    if (T <= 0 || T > PF_MAX_T || kbase + (size_t)T > c->g.kv[ATT_LAYER].capacity)
        return -1;
    c->g.kv[ATT_LAYER].length = kbase;
    return pf_attention(&c->g.m, ATT_LAYER, T, base);
}

int ref_prefill_ctx_projections(RefPrefillCtx *c, int T)
{
    (void)c;
    const LayerRefs *L = &R->layer[ATT_LAYER];
    const TRef *refs[3] = { &L->q, &L->k, &L->v };
    float *outs[3] = { g_pf.qkv, g_pf.k, g_pf.v };
    const size_t rws[3] = { MODEL_ATTN_Q_SIZE, MODEL_ATTN_K_SIZE, MODEL_ATTN_V_SIZE };
    if (pf_mm(refs, outs, rws, 3, g_pf.nrm, PF_H, T) != 0)
        return -1;
    return pf_mm1(&L->o, g_pf.res, MODEL_HIDDEN_SIZE, g_pf.rec, 4096, T);
}

/* recurrent_delta_step on a caller state [32][128][128]. */
void ref_delta_step(float *state, const float *q, const float *k, const float *v,
                    const float *g, const float *beta, float *out)
{
    SSMState s;
    memset(&s, 0, sizeof(s));
    s.state = state;
    s.state_elements = (size_t)MODEL_LINEAR_V_HEADS * 128 * 128;
    recurrent_delta_step(&s, q, k, v, g, beta, out);
}

/* T tokens of delta_head per value head, heads in parallel (the recurrence of pf_ssm,
 * model.c:1644-1658, without its norm/gate post-ops). q,k: [T][16][128]; v: [T][32][128];
 * g, beta: [T][32]; out: [T][32][128]. */
void ref_delta_prefill(float *state, int T, const float *q, const float *k, const float *v,
                       const float *g, const float *beta, float *out)
{
    #pragma omp parallel for schedule(static)
    for (int vh = 0; vh < MODEL_LINEAR_V_HEADS; vh++) {
        const int kh = vh % MODEL_LINEAR_K_HEADS;
        float *st = state + (size_t)vh * 128 * 128;
        for (int t = 0; t < T; t++)
            delta_head(st, q + ((size_t)t * 16 + kh) * 128, k + ((size_t)t * 16 + kh) * 128,
                       v + ((size_t)t * 32 + vh) * 128, g[(size_t)t * 32 + vh],
                       beta[(size_t)t * 32 + vh], out + ((size_t)t * 32 + vh) * 128);
    }
}

/* ---- a whole Gated DeltaNet layer through pf_ssm (model.c:1604-1660).
 * The four projections are one-hot f32 matvecs: token t's normed row is e_t and column t of
 * W_qkv / W_gate / W_alpha / W_beta holds its qkv [8192], z [4096], alpha [32], beta [32]. pf_ssm
 * then runs, on exactly those inputs, its per-token conv1d + SiLU + L2-norm + beta/g prep
 * (1619-1643), the delta_head recurrence (1644-1658) and the gated RMSNorm (1655-1658). The
 * layer output is read from the prefill scratch (g_pf.rec) before the ssm_out projection.
 * T <= 256. state [32][128][128] and conv_state [3][8192] are updated in place. */
#define DN_LAYER 0                                  /* (0+1) % 4 != 0: a recurrent layer */
static TensorInfo t_qkv, t_gate, t_al, t_be, t_so;
static float *W_qkv, *W_gate, *W_al, *W_be, *W_so;

static void set_col_n(float *W, size_t rows, size_t col, const float *x)
{
    for (size_t r = 0; r < rows; r++)
        W[r * MODEL_HIDDEN_SIZE + col] = x[r];
}

int ref_delta_layer_prefill(int T, const float *qkv, const float *z, const float *alpha,
                            const float *beta, const float *conv_w, const float *dt, const float *a,
                            const float *ssm_norm, float *state, float *conv_state, float *out)
{
    if (T <= 0 || T > PF_MAX_T || ensure_weights() != 0)
        return -1;
    if (!W_qkv) {
        W_qkv = calloc((size_t)MODEL_LINEAR_QKV_SIZE * MODEL_HIDDEN_SIZE, sizeof(float));
        W_gate = calloc((size_t)MODEL_LINEAR_GATE_SIZE * MODEL_HIDDEN_SIZE, sizeof(float));
        W_al = calloc((size_t)MODEL_LINEAR_V_HEADS * MODEL_HIDDEN_SIZE, sizeof(float));
        W_be = calloc((size_t)MODEL_LINEAR_V_HEADS * MODEL_HIDDEN_SIZE, sizeof(float));
        W_so = calloc((size_t)MODEL_HIDDEN_SIZE * MODEL_LINEAR_V_SIZE, sizeof(float));
        if (!W_qkv || !W_gate || !W_al || !W_be || !W_so)
            return -1;
        t_qkv.type = t_gate.type = t_al.type = t_be.type = t_so.type = 0;
    }
    LayerRefs *L = &R->layer[DN_LAYER];
    L->qkv = (TRef){ &t_qkv, W_qkv };
    L->gate = (TRef){ &t_gate, W_gate };
    L->alpha = (TRef){ &t_al, W_al };
    L->beta = (TRef){ &t_be, W_be };
    L->ssm_out = (TRef){ &t_so, W_so };
    L->conv = conv_w;
    L->dt = dt;
    L->a = a;
    L->ssm_norm = ssm_norm;
    static SSMState ss[MODEL_NUM_LAYERS];
    memset(ss, 0, sizeof(ss));
    ss[DN_LAYER].state = state;
    ss[DN_LAYER].conv_state = conv_state;
    ss[DN_LAYER].state_elements = (size_t)MODEL_LINEAR_V_HEADS * 128 * 128;
    ss[DN_LAYER].conv_elements = (size_t)(MODEL_SSM_CONV_KERNEL - 1) * MODEL_LINEAR_QKV_SIZE;
    static Model m;
    memset(&m, 0, sizeof(m));
    m.refs = R;
    m.ssm_state = ss;
    m.initialized = true;
    if (pf_ensure((size_t)T) != 0)
        return -1;
    memset(g_pf.nrm, 0, (size_t)T * PF_H * sizeof(float));
    for (int t = 0; t < T; t++) {
        g_pf.nrm[(size_t)t * PF_H + (size_t)t] = 1.0f;
        set_col_n(W_qkv, MODEL_LINEAR_QKV_SIZE, (size_t)t, qkv + (size_t)t * MODEL_LINEAR_QKV_SIZE);
        set_col_n(W_gate, MODEL_LINEAR_GATE_SIZE, (size_t)t, z + (size_t)t * MODEL_LINEAR_GATE_SIZE);
        set_col_n(W_al, MODEL_LINEAR_V_HEADS, (size_t)t, alpha + (size_t)t * MODEL_LINEAR_V_HEADS);
        set_col_n(W_be, MODEL_LINEAR_V_HEADS, (size_t)t, beta + (size_t)t * MODEL_LINEAR_V_HEADS);
    }
    const int rc = pf_ssm(&m, DN_LAYER, T);
    if (rc == 0)
        memcpy(out, g_pf.rec, (size_t)T * MODEL_LINEAR_V_SIZE * sizeof(float));
    for (int t = 0; t < T; t++) {
        const float zero[MODEL_LINEAR_QKV_SIZE] = {0};
        set_col_n(W_qkv, MODEL_LINEAR_QKV_SIZE, (size_t)t, zero);
        set_col_n(W_gate, MODEL_LINEAR_GATE_SIZE, (size_t)t, zero);
        set_col_n(W_al, MODEL_LINEAR_V_HEADS, (size_t)t, zero);
        set_col_n(W_be, MODEL_LINEAR_V_HEADS, (size_t)t, zero);
    }
    return rc;
}

/* ---- the attention window (kvwindow.c) over a rig holding only the 10 attention layers' KV.
 * Appends follow forward_impl / prefill_chunk: kvw_ensure_room(n) first (model.c:1265, 1798),
 * then the rows land at the window's end and position advances. Context changes go through
 * model_set_context (model.c:1870-1899). */
typedef struct RefWin {
    Model m;
    KVCache kv[MODEL_NUM_LAYERS];
    KVSpill sp;
    int att[MODEL_NUM_LAYERS], na;
} RefWin;

RefWin *ref_kvw_new(size_t ctx, int slide, size_t keep, size_t pin, const char *spill_path)
{
    RefWin *w = calloc(1, sizeof(*w));
    if (!w)
        return NULL;
    for (int l = 0; l < MODEL_NUM_LAYERS; l++) {
        if (!model_is_attention_layer(l))
            continue;
        w->kv[l].k = locked_calloc_checked(ctx * KV_FLOATS_PER_TOKEN, sizeof(float));
        w->kv[l].v = locked_calloc_checked(ctx * KV_FLOATS_PER_TOKEN, sizeof(float));
        w->kv[l].capacity = ctx;
        w->att[w->na++] = l;
    }
    kvspill_init(&w->sp, spill_path);
    w->m.kv_cache = w->kv;
    w->m.context_length = ctx;
    w->m.slide = slide != 0;
    w->m.slide_keep = keep;
    w->m.slide_pin = pin;
    w->m.spill = &w->sp;
    w->m.attn_scratch = calloc(16 * ctx, sizeof(float));
    w->m.initialized = true;
    return w;
}

void ref_kvw_free(RefWin *w)
{
    if (!w)
        return;
    kvspill_clear(&w->sp);
    for (int l = 0; l < MODEL_NUM_LAYERS; l++) {
        locked_buffer_free(w->kv[l].k);
        locked_buffer_free(w->kv[l].v);
    }
    free(w->m.attn_scratch);
    free(w);
}

int ref_kvw_layers(const RefWin *w) { return w->na; }

/* k, v: [na][n][512] rows for the n new tokens of every attention layer. */
int ref_kvw_append(RefWin *w, size_t n, const float *k, const float *v)
{
    if (kvw_ensure_room(&w->m, n) != 0)
        return -1;
    for (int a = 0; a < w->na; a++) {
        KVCache *kv = &w->kv[w->att[a]];
        memcpy(kv->k + kv->length * KV_FLOATS_PER_TOKEN, k + (size_t)a * n * KV_FLOATS_PER_TOKEN,
               n * KV_FLOATS_PER_TOKEN * sizeof(float));
        memcpy(kv->v + kv->length * KV_FLOATS_PER_TOKEN, v + (size_t)a * n * KV_FLOATS_PER_TOKEN,
               n * KV_FLOATS_PER_TOKEN * sizeof(float));
        kv->length += n;
    }
    w->m.position += n;
    return 0;
}

int ref_kvw_evict(RefWin *w, size_t n) { return kvw_evict(&w->m, n); }
int ref_kvw_restore(RefWin *w, size_t n) { return kvw_restore(&w->m, n); }
int ref_kvw_rollback(RefWin *w, size_t p0, size_t s0) { return kvw_rollback(&w->m, p0, s0); }
int ref_kvw_set_context(RefWin *w, size_t ctx) { return model_set_context(&w->m, ctx); }
size_t ref_kvw_len(const RefWin *w) { return kvw_len(&w->m); }
size_t ref_kvw_spilled(const RefWin *w) { return kvw_spilled(&w->m); }
size_t ref_kvw_head(const RefWin *w) { return kvw_head(&w->m); }
size_t ref_kvw_max_chunk(const RefWin *w) { return kvw_max_chunk(&w->m); }
size_t ref_kvw_position(const RefWin *w) { return w->m.position; }
size_t ref_kvw_context(const RefWin *w) { return w->m.context_length; }

/* The window rows [0, len) of attention layer index a. */
void ref_kvw_read(const RefWin *w, int a, float *k, float *v)
{
    const KVCache *kv = &w->kv[w->att[a]];
    memcpy(k, kv->k, kv->length * KV_FLOATS_PER_TOKEN * sizeof(float));
    memcpy(v, kv->v, kv->length * KV_FLOATS_PER_TOKEN * sizeof(float));
}

int ref_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---- k-quant projections: the reference's matvec_q4_cpu / matvec_q6_cpu (kernels.c:405-431,
 * 553-578) are static in kernels.c; they are one kernel_dot_q4_k / kernel_dot_q6_k call per row
 * under an OpenMP loop, reproduced here around the reference's own (public) dot functions. */
void ref_matvec_q(int is_q6, const void *matrix, const float *x, float *out, size_t rows, size_t cols)
{
    const size_t rb = (cols / 256) * (is_q6 ? 210 : 144);
    const uint8_t *m = (const uint8_t *)matrix;
    #pragma omp parallel for schedule(static) if (rows * (cols / 256) >= 16384)
    for (size_t r = 0; r < rows; r++)
        out[r] = is_q6 ? kernel_dot_q6_k(m + r * rb, x, cols) : kernel_dot_q4_k(m + r * rb, x, cols);
}

/* ---- the reference's state file ("RSTA" v2, state.c:7-81) through its own model_state_save /
 * model_state_load, on a Model rig with host fp32 windows of `ctx` rows for the attention
 * layers and the DeltaNet state + conv history of the recurrent layers (the sizes of
 * kv_cache_init / ssm_state_init, model.c:355-461). No spill store: the window holds every
 * token, so `position` equals the window length. */
#include "state.h"

typedef struct RefState {
    Model m;
    KVCache kv[MODEL_NUM_LAYERS];
    SSMState ss[MODEL_NUM_LAYERS];
} RefState;

void ref_state_free(RefState *r)
{
    if (!r)
        return;
    for (int l = 0; l < MODEL_NUM_LAYERS; l++) {
        free(r->kv[l].k);
        free(r->kv[l].v);
        free(r->ss[l].state);
        free(r->ss[l].conv_state);
    }
    free(r);
}

RefState *ref_state_new(size_t ctx)
{
    RefState *r = calloc(1, sizeof(*r));
    if (!r)
        return NULL;
    for (int l = 0; l < MODEL_NUM_LAYERS; l++) {
        if (model_is_attention_layer(l)) {
            r->kv[l].k = calloc(ctx * KV_FLOATS_PER_TOKEN, sizeof(float));
            r->kv[l].v = calloc(ctx * KV_FLOATS_PER_TOKEN, sizeof(float));
            r->kv[l].capacity = ctx;
            if (!r->kv[l].k || !r->kv[l].v) {
                ref_state_free(r);
                return NULL;
            }
        } else {
            r->ss[l].state_elements = (size_t)MODEL_LINEAR_V_HEADS * MODEL_LINEAR_HEAD_DIM * MODEL_LINEAR_HEAD_DIM;
            r->ss[l].conv_elements = (size_t)(MODEL_SSM_CONV_KERNEL - 1) * MODEL_LINEAR_QKV_SIZE;
            r->ss[l].state = calloc(r->ss[l].state_elements, sizeof(float));
            r->ss[l].conv_state = calloc(r->ss[l].conv_elements, sizeof(float));
            if (!r->ss[l].state || !r->ss[l].conv_state) {
                ref_state_free(r);
                return NULL;
            }
        }
    }
    r->m.kv_cache = r->kv;
    r->m.ssm_state = r->ss;
    r->m.context_length = ctx;
    r->m.initialized = true;
    return r;
}

float *ref_state_k(RefState *r, int layer) { return r->kv[layer].k; }
float *ref_state_v(RefState *r, int layer) { return r->kv[layer].v; }
float *ref_state_ssm(RefState *r, int layer) { return r->ss[layer].state; }
float *ref_state_conv(RefState *r, int layer) { return r->ss[layer].conv_state; }
int ref_state_is_attention(int layer) { return model_is_attention_layer(layer) ? 1 : 0; }
int ref_state_layers(void) { return MODEL_NUM_LAYERS; }

void ref_state_set_len(RefState *r, size_t len)
{
    for (int l = 0; l < MODEL_NUM_LAYERS; l++)
        if (model_is_attention_layer(l))
            r->kv[l].length = len;
    r->m.position = len;
}

size_t ref_state_len(const RefState *r, int layer) { return r->kv[layer].length; }
size_t ref_state_position(const RefState *r) { return r->m.position; }

int ref_state_save(RefState *r, const char *path)
{
    FILE *f = fopen(path, "wb");
    if (!f)
        return -1;
    const int rc = model_state_save(&r->m, f);
    return fclose(f) == 0 ? rc : -1;
}

int ref_state_load(RefState *r, const char *path)
{
    FILE *f = fopen(path, "rb");
    if (!f)
        return -1;
    const int rc = model_state_load(&r->m, f);
    fclose(f);
    return rc;
}
