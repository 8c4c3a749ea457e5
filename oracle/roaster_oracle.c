/*
 * CPU oracle for the hybrid-attention hot path. TEST INFRASTRUCTURE ONLY: it is the checker
 * for tests/, bench.py's CPU-baseline leg and __graft_entry__.smoke(); the product library
 * never calls it. Restates the reference's arithmetic (KKB007X/Roaster) in plain C; each
 * function cites the reference lines it follows. Parity of this restatement is pinned against
 * the reference compiled from its own sources (oracle/_ref) and the golden vectors in
 * tests/golden/.
 */
#include "roaster_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- f16 <-> f32 */

/* IEEE binary16 -> binary32, all classes (the reference widens with F16C `_cvtsh_ss`,
 * src/kernels.c:56-96, which is exact). */
float orc_f16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 31u, m = h & 1023u, bits;
    if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {                      /* subnormal: normalise */
            int shift = 0;
            while (!(m & 1024u)) { m <<= 1; shift++; }
            m &= 1023u;
            bits = sign | ((uint32_t)(127 - 15 - shift + 1) << 23) | (m << 13);
        }
    } else {
        bits = sign | ((e - 15 + 127) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* binary32 -> binary16, round to nearest even, overflow to inf, NaN kept quiet. */
uint16_t orc_f32_to_f16(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u)                                    /* inf / nan */
        return sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u);
    if (ax >= 0x477ff000u)                                    /* rounds to >= 65520 */
        return sign | 0x7c00u;
    if (ax < 0x33000000u)                                     /* < 2^-25: rounds to 0 */
        return sign;
    int e = (int)(ax >> 23) - 127;
    uint32_t mant = (ax & 0x7fffffu) | 0x800000u;             /* 24-bit significand */
    int shift;                                                /* bits dropped */
    uint32_t base;
    if (e < -14) {                                            /* subnormal result */
        shift = 13 + (-14 - e);
        base = 0;
    } else {
        shift = 13;
        base = (uint32_t)(e + 15) << 10;
        mant &= 0x7fffffu;
    }
    uint32_t q = mant >> shift, rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1);
    uint32_t r = base + q;
    if (rem > half || (rem == half && (q & 1u)))
        r++;
    return sign | (uint16_t)r;
}

/* ---------------------------------------------------------------- primitives */

/* kernel_rmsnorm, src/kernels.c:584-605: x * (1/sqrt(mean(x^2)+eps)) * w. */
void orc_rmsnorm(float *out, const float *in, const float *w, size_t n, float eps)
{
    float ss = 0.0f;
    for (size_t i = 0; i < n; i++)
        ss += in[i] * in[i];
    const float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (size_t i = 0; i < n; i++)
        out[i] = in[i] * inv * w[i];
}

/* kernel_l2norm, src/kernels.c:607-622: x / sqrt(sum(x^2)+eps). */
void orc_l2norm(float *out, const float *in, size_t n, float eps)
{
    float ss = 0.0f;
    for (size_t i = 0; i < n; i++)
        ss += in[i] * in[i];
    const float inv = 1.0f / sqrtf(ss + eps);
    for (size_t i = 0; i < n; i++)
        out[i] = in[i] * inv;
}

/* apply_rope_64, src/model.c:759-781: NeoX rotate-half on dims [0,32) x [32,64) of each head,
 * theta 1e7, inv_freq_j = theta^(-2j/64), all in fp32 libm. Dims 64.. are untouched. */
void orc_rope64(float *x, size_t heads, size_t head_dim, size_t position)
{
    float c[32], s[32];
    for (int j = 0; j < 32; j++) {
        const float f = powf(10000000.0f, -2.0f * (float)j / 64.0f);
        const float ang = (float)position * f;
        c[j] = cosf(ang);
        s[j] = sinf(ang);
    }
    for (size_t h = 0; h < heads; h++) {
        float *r = x + h * head_dim;
        for (int j = 0; j < 32; j++) {
            const float lo = r[j], hi = r[j + 32];
            r[j] = lo * c[j] - hi * s[j];
            r[j + 32] = hi * c[j] + lo * s[j];
        }
    }
}

static float dot(const float *a, const float *b, size_t n)
{
    float acc = 0.0f;
    for (size_t i = 0; i < n; i++)
        acc += a[i] * b[i];
    return acc;
}

static float sigm(float g)
{
    return 1.0f / (1.0f + expf(-g));
}

/* ---------------------------------------------------------------- attention */

/* Prepare one token: split q/gate rows, q/k RMSNorm, RoPE (model.c:801-819 and the per-token
 * prep of pf_attention, model.c:1553-1568). qo: [16][256], ko: [2][256]. */
static void prep_token(const float *q, size_t qg_stride, const float *k,
                       const float *qnorm, const float *knorm, size_t pos,
                       float *qo, float *ko)
{
    for (int h = 0; h < ORC_QH; h++)
        orc_rmsnorm(qo + h * ORC_D, q + (size_t)h * qg_stride, qnorm, ORC_D, 1e-6f);
    for (int h = 0; h < ORC_KVH; h++)
        orc_rmsnorm(ko + h * ORC_D, k + h * ORC_D, knorm, ORC_D, 1e-6f);
    orc_rope64(qo, ORC_QH, ORC_D, pos);
    orc_rope64(ko, ORC_KVH, ORC_D, pos);
}

/* Three-pass softmax attention of one query row over `len` keys whose rows are fetched by
 * `row(t)` (model.c:830-856 / 1572-1600). Scores scratch has len floats. */
static void attend_row(const float *qh, size_t len,
                       const float *(*krow)(const void *, size_t, int),
                       const float *(*vrow)(const void *, size_t, int),
                       const void *ctx, int kvh, float *scores, float *out)
{
    const float scale = 1.0f / 16.0f;
    float mx = -INFINITY;
    for (size_t t = 0; t < len; t++) {
        scores[t] = dot(qh, krow(ctx, t, kvh), ORC_D) * scale;
        if (scores[t] > mx)
            mx = scores[t];
    }
    float sum = 0.0f;
    for (size_t t = 0; t < len; t++) {
        scores[t] = expf(scores[t] - mx);
        sum += scores[t];
    }
    const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
    for (int d = 0; d < ORC_D; d++)
        out[d] = 0.0f;
    for (size_t t = 0; t < len; t++) {
        const float *vr = vrow(ctx, t, kvh);
        const float p = scores[t] * inv;
        for (int d = 0; d < ORC_D; d++)
            out[d] += p * vr[d];
    }
}

/* A widened window: cached f16 rows [0, ncached) followed by fp32 rows appended this call. */
typedef struct {
    const float *kc, *vc;       /* widened cache, [ncached][2][256] */
    size_t ncached;
    const float *ka, *va;       /* appended, [..][2][256] */
} Window;

static const float *win_k(const void *c, size_t t, int h)
{
    const Window *w = (const Window *)c;
    return t < w->ncached ? w->kc + (t * 2 + h) * ORC_D : w->ka + ((t - w->ncached) * 2 + h) * ORC_D;
}

static const float *win_v(const void *c, size_t t, int h)
{
    const Window *w = (const Window *)c;
    return t < w->ncached ? w->vc + (t * 2 + h) * ORC_D : w->va + ((t - w->ncached) * 2 + h) * ORC_D;
}

static float *widen(const uint16_t *src, size_t n)
{
    float *dst = (float *)malloc((n ? n : 1) * sizeof(float));
    if (!dst)
        return NULL;
    for (size_t i = 0; i < n; i++)
        dst[i] = orc_f16_to_f32(src[i]);
    return dst;
}

int orc_attn_decode(const float *q, const float *gate, size_t qg_stride,
                    const float *k_new, const float *v_new,
                    const float *qnorm, const float *knorm,
                    const uint16_t *k_cache, const uint16_t *v_cache,
                    size_t length, size_t position,
                    float *out, float *k_app, float *v_app)
{
    return orc_attn_prefill(1, q, gate, qg_stride, 0, k_new, v_new, qnorm, knorm,
                            k_cache, v_cache, length, position, out, k_app, v_app);
}

int orc_attn_prefill(size_t T, const float *q, const float *gate, size_t qg_stride,
                     size_t qg_tok_stride, const float *k, const float *v,
                     const float *qnorm, const float *knorm,
                     const uint16_t *k_cache, const uint16_t *v_cache,
                     size_t kbase, size_t base,
                     float *out, float *k_app, float *v_app)
{
    if (!q || !gate || !k || !v || !qnorm || !knorm || !out || T == 0)
        return -1;
    if (kbase && (!k_cache || !v_cache))
        return -1;
    const size_t n = kbase * ORC_KVH * ORC_D;
    float *kc = widen(k_cache, n), *vc = widen(v_cache, n);
    float *qp = (float *)malloc(T * ORC_QH * ORC_D * sizeof(float));
    float *kp = (float *)malloc(T * ORC_KVH * ORC_D * sizeof(float));
    int rc = -1;
    if (!kc || !vc || !qp || !kp)
        goto done;
    /* Prepare every token and append its K/V first (model.c:1553-1569). */
    for (size_t t = 0; t < T; t++)
        prep_token(q + t * qg_tok_stride, qg_stride, k + t * ORC_KVH * ORC_D, qnorm, knorm,
                   base + t, qp + t * ORC_QH * ORC_D, kp + t * ORC_KVH * ORC_D);
    {
        Window w = { kc, vc, kbase, kp, v };
        const size_t maxlen = kbase + T;
        int bad = 0;
        #pragma omp parallel
        {
            float *scores = (float *)malloc(maxlen * sizeof(float));
            if (!scores) {
                #pragma omp atomic write
                bad = 1;
            }
            #pragma omp for schedule(dynamic, 4)
            for (long idx = 0; idx < (long)(T * ORC_QH); idx++) {
                if (!scores)
                    continue;
                const size_t t = (size_t)idx / ORC_QH;
                const int h = (int)(idx % ORC_QH);
                float *o = out + (t * ORC_QH + h) * ORC_D;
                attend_row(qp + (t * ORC_QH + h) * ORC_D, kbase + t + 1, win_k, win_v, &w,
                           h / 8, scores, o);
                const float *g = gate + t * qg_tok_stride + (size_t)h * qg_stride;
                for (int d = 0; d < ORC_D; d++)
                    o[d] *= sigm(g[d]);
            }
            free(scores);
        }
        if (bad)
            goto done;
    }
    if (k_app)
        memcpy(k_app, kp, T * ORC_KVH * ORC_D * sizeof(float));
    if (v_app)
        memcpy(v_app, v, T * ORC_KVH * ORC_D * sizeof(float));
    rc = 0;
done:
    free(kc);
    free(vc);
    free(qp);
    free(kp);
    return rc;
}

int orc_attn_prefill_rows(size_t T, const float *q, const float *gate, size_t qg_stride,
                          size_t qg_tok_stride, const float *k, const float *v,
                          const float *qnorm, const float *knorm,
                          const uint16_t *k_cache, const uint16_t *v_cache,
                          size_t kbase, size_t base, const long *rows, size_t nrows, float *out)
{
    if (!q || !gate || !k || !v || !qnorm || !knorm || !out || !rows || T == 0)
        return -1;
    if (kbase && (!k_cache || !v_cache))
        return -1;
    const size_t n = kbase * ORC_KVH * ORC_D;
    float *kc = widen(k_cache, n), *vc = widen(v_cache, n);
    float *kp = (float *)malloc(T * ORC_KVH * ORC_D * sizeof(float));
    int rc = -1;
    if (!kc || !vc || !kp)
        goto done;
    for (size_t t = 0; t < T; t++) {
        for (int h = 0; h < ORC_KVH; h++)
            orc_rmsnorm(kp + (t * ORC_KVH + h) * ORC_D, k + (t * ORC_KVH + h) * ORC_D, knorm, ORC_D, 1e-6f);
        orc_rope64(kp + t * ORC_KVH * ORC_D, ORC_KVH, ORC_D, base + t);
    }
    {
        Window w = { kc, vc, kbase, kp, v };
        int bad = 0;
        #pragma omp parallel
        {
            float *scores = (float *)malloc((kbase + T) * sizeof(float));
            float qh[ORC_D];
            if (!scores) {
                #pragma omp atomic write
                bad = 1;
            }
            #pragma omp for schedule(dynamic, 1)
            for (long idx = 0; idx < (long)(nrows * ORC_QH); idx++) {
                if (!scores)
                    continue;
                const size_t i = (size_t)idx / ORC_QH;
                const int h = (int)(idx % ORC_QH);
                const long t = rows[i];
                if (t < 0 || (size_t)t >= T)
                    continue;
                orc_rmsnorm(qh, q + (size_t)t * qg_tok_stride + (size_t)h * qg_stride, qnorm, ORC_D, 1e-6f);
                orc_rope64(qh, 1, ORC_D, base + (size_t)t);
                float *o = out + (i * ORC_QH + h) * ORC_D;
                attend_row(qh, kbase + (size_t)t + 1, win_k, win_v, &w, h / 8, scores, o);
                const float *g = gate + (size_t)t * qg_tok_stride + (size_t)h * qg_stride;
                for (int d = 0; d < ORC_D; d++)
                    o[d] *= sigm(g[d]);
            }
            free(scores);
        }
        if (bad)
            goto done;
    }
    rc = 0;
done:
    free(kc);
    free(vc);
    free(kp);
    return rc;
}

int orc_attn_decode_partial(const float *q, size_t qg_stride, const float *qnorm,
                            const uint16_t *k_cache, const uint16_t *v_cache,
                            size_t t0, size_t t1, size_t position,
                            float *m, float *l, float *o)
{
    if (!q || !qnorm || !m || !l || !o || t1 < t0)
        return -1;
    float qp[ORC_QH * ORC_D];
    for (int h = 0; h < ORC_QH; h++)
        orc_rmsnorm(qp + h * ORC_D, q + (size_t)h * qg_stride, qnorm, ORC_D, 1e-6f);
    orc_rope64(qp, ORC_QH, ORC_D, position);
    const size_t len = t1 - t0;
    float *s = (float *)malloc((len ? len : 1) * sizeof(float));
    if (!s)
        return -1;
    for (int h = 0; h < ORC_QH; h++) {
        const int kvh = h / 8;
        float mx = -INFINITY, sum = 0.0f;
        float kr[ORC_D];
        for (size_t t = 0; t < len; t++) {
            const uint16_t *src = k_cache + ((t0 + t) * 2 + kvh) * ORC_D;
            for (int d = 0; d < ORC_D; d++)
                kr[d] = orc_f16_to_f32(src[d]);
            s[t] = dot(qp + h * ORC_D, kr, ORC_D) / 16.0f;
            if (s[t] > mx)
                mx = s[t];
        }
        for (size_t t = 0; t < len; t++) {
            s[t] = expf(s[t] - mx);
            sum += s[t];
        }
        float *oh = o + h * ORC_D;
        for (int d = 0; d < ORC_D; d++)
            oh[d] = 0.0f;
        for (size_t t = 0; t < len; t++) {
            const uint16_t *src = v_cache + ((t0 + t) * 2 + kvh) * ORC_D;
            const float p = s[t] / sum;
            for (int d = 0; d < ORC_D; d++)
                oh[d] += p * orc_f16_to_f32(src[d]);
        }
        m[h] = mx;
        l[h] = sum;
    }
    free(s);
    return 0;
}

/* ---------------------------------------------------------------- Gated DeltaNet */

/* One value head of the delta rule (recurrent_delta_step, model.c:272-323; delta_head,
 * model.c:1507-1534). st: [128 key rows][128 value cols].
 *   A = S^T k, B = S^T q, kq = k.q (one pass over the old state)
 *   delta = (v - d*A) * beta,  out = (d*B + kq*delta) / sqrt(128)
 *   S <- d*S + k (x) delta,    d = exp(g) */
static void delta_one(float *st, const float *qh, const float *kh, const float *vh,
                      float g, float b, float *out)
{
    const float scale = 1.0f / sqrtf(128.0f);
    const float d = expf(g);
    float A[ORC_DN_D], B[ORC_DN_D], delta[ORC_DN_D], kq = 0.0f;
    for (int c = 0; c < ORC_DN_D; c++)
        A[c] = B[c] = 0.0f;
    for (int r = 0; r < ORC_DN_D; r++) {
        const float *row = st + r * ORC_DN_D;
        kq += kh[r] * qh[r];
        for (int c = 0; c < ORC_DN_D; c++) {
            A[c] += row[c] * kh[r];
            B[c] += row[c] * qh[r];
        }
    }
    for (int c = 0; c < ORC_DN_D; c++) {
        delta[c] = (vh[c] - d * A[c]) * b;
        out[c] = (d * B[c] + kq * delta[c]) * scale;
    }
    for (int r = 0; r < ORC_DN_D; r++) {
        float *row = st + r * ORC_DN_D;
        for (int c = 0; c < ORC_DN_D; c++)
            row[c] = d * row[c] + kh[r] * delta[c];
    }
}

/* Value head vh reads key head vh % 16 (model.c:285: tiled, not vh / 2). */
void orc_delta_step(float *state, const float *q, const float *k, const float *v,
                    const float *g, const float *beta, float *out)
{
    for (int vh = 0; vh < ORC_DN_VH; vh++) {
        const int kh = vh % ORC_DN_KH;
        delta_one(state + (size_t)vh * ORC_DN_D * ORC_DN_D, q + kh * ORC_DN_D, k + kh * ORC_DN_D,
                  v + vh * ORC_DN_D, g[vh], beta[vh], out + vh * ORC_DN_D);
    }
}

void orc_delta_prefill(float *state, size_t T, const float *q, const float *k, const float *v,
                       const float *g, const float *beta, float *out)
{
    #pragma omp parallel for schedule(static)
    for (int vh = 0; vh < ORC_DN_VH; vh++) {
        const int kh = vh % ORC_DN_KH;
        float *st = state + (size_t)vh * ORC_DN_D * ORC_DN_D;
        for (size_t t = 0; t < T; t++)
            delta_one(st, q + (t * ORC_DN_KH + kh) * ORC_DN_D, k + (t * ORC_DN_KH + kh) * ORC_DN_D,
                      v + (t * ORC_DN_VH + vh) * ORC_DN_D, g[t * ORC_DN_VH + vh],
                      beta[t * ORC_DN_VH + vh], out + (t * ORC_DN_VH + vh) * ORC_DN_D);
    }
}

/* ---------------------------------------------------------------- Gated DeltaNet pre/post ops */

/* Logistic function in the form that never overflows exp (kernel_sigmoid, kernels.c:628-638). */
static float orc_sigmoid(float x)
{
    if (x >= 0.0f)
        return 1.0f / (1.0f + expf(-x));
    const float e = expf(x);
    return e / (1.0f + e);
}

/* Pre-ops of one recurrent layer for T consecutive tokens: the decode block model.c:1293-1328
 * applied token by token, which is also pf_ssm's prep loop (model.c:1619-1643).
 *   conv:  cv[c] = sum_{j<3} hist[j][c] w[c][j] + in[c] w[c][3]     (kernel_conv1d_causal_f32,
 *          kernels.c:693-719; hist holds the 3 previous raw inputs, oldest first)
 *   SiLU:  cv[c] *= sigmoid(cv[c])                                  (kernels.c:644-651)
 *   history: hist <- [hist[1], hist[2], in]                         (model.c:1299-1306)
 *   q = cv[0:2048], k = cv[2048:4096] L2-normalised per 128 (eps 1e-6, kernels.c:607-622),
 *   v = cv[4096:8192]; beta' = sigmoid(beta), g = a softplus(alpha + dt) with softplus(x) = x
 *   for x > 20 (model.c:1324-1328).
 * qkv [T][8192], alpha/beta [T][32] in; conv_state [3][8192] updated; conv_w [8192][4];
 * q, k [T][16][128], v [T][32][128], g, b [T][32] out. */
void orc_delta_preop(size_t T, const float *qkv, const float *alpha, const float *beta,
                     float *conv_state, const float *conv_w, const float *dt, const float *a,
                     float *q, float *k, float *v, float *g, float *b)
{
    const size_t Q = 8192;
    float *cv = malloc(Q * sizeof(float));
    for (size_t t = 0; t < T; t++) {
        const float *in = qkv + t * Q;
        for (size_t c = 0; c < Q; c++) {
            float sum = 0.0f;
            for (size_t j = 0; j < 3; j++)
                sum += conv_state[j * Q + c] * conv_w[c * 4 + j];
            sum += in[c] * conv_w[c * 4 + 3];
            cv[c] = sum * orc_sigmoid(sum);
        }
        memmove(conv_state, conv_state + Q, 2 * Q * sizeof(float));
        memcpy(conv_state + 2 * Q, in, Q * sizeof(float));
        for (int h = 0; h < 16; h++) {
            orc_l2norm(q + (t * 16 + h) * 128, cv + h * 128, 128, 1e-6f);
            orc_l2norm(k + (t * 16 + h) * 128, cv + 2048 + h * 128, 128, 1e-6f);
        }
        memcpy(v + t * 4096, cv + 4096, 4096 * sizeof(float));
        for (int h = 0; h < 32; h++) {
            b[t * 32 + h] = 1.0f / (1.0f + expf(-beta[t * 32 + h]));
            const float x = alpha[t * 32 + h] + dt[h];
            g[t * 32 + h] = a[h] * (x > 20.0f ? x : log1pf(expf(x)));
        }
    }
    free(cv);
}

/* Gated RMSNorm of `rows` value-head rows (model.c:1333-1343, pf_ssm 1655-1658): per row of 128,
 * out = rmsnorm(out) * w (eps 1e-6), then out *= z sigmoid(z). */
void orc_delta_postop(size_t rows, float *out, const float *z, const float *w)
{
    for (size_t r = 0; r < rows; r++) {
        float *x = out + r * 128;
        const float *zr = z + r * 128;
        orc_rmsnorm(x, x, w, 128, 1e-6f);
        for (int j = 0; j < 128; j++)
            x[j] *= zr[j] * (1.0f / (1.0f + expf(-zr[j])));
    }
}

/* Q4_K block (kernels.c:137-200): d, dmin (f16), 12 bytes of 6-bit scales/mins unpacked as in
 * q4_k_get_scales (kernels.c:155-174), 128 bytes of nibbles; group g of 64 weights takes the low
 * nibbles of qs[32g..32g+31] (scale/min 2g) then their high nibbles (2g+1);
 * weight = d sc q - dmin m. */
static float orc_dot_q4_block(const uint8_t *b, const float *x)
{
    const float d = orc_f16_to_f32((uint16_t)(b[0] | (b[1] << 8)));
    const float dmin = orc_f16_to_f32((uint16_t)(b[2] | (b[3] << 8)));
    const uint8_t *sc = b + 4, *qs = b + 16;
    float sum = 0.0f;
    for (int j = 0; j < 8; j++) {
        int s, m;
        if (j < 4) {
            s = sc[j] & 63;
            m = sc[j + 4] & 63;
        } else {
            s = (sc[j + 4] & 0x0F) | ((sc[j - 4] >> 6) << 4);
            m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
        }
        const int g = j >> 1, hi = j & 1;
        float part = 0.0f, xs = 0.0f;
        for (int i = 0; i < 32; i++) {
            const int q = hi ? (qs[32 * g + i] >> 4) : (qs[32 * g + i] & 15);
            part += (float)q * x[32 * j + i];
            xs += x[32 * j + i];
        }
        sum += d * (float)s * part - dmin * (float)m * xs;
    }
    return sum;
}

/* Q6_K block (kernels.c:437-488): ql[128], qh[64], int8 scales[16], d; for half n and l < 32 the
 * weights 128n + l, +32, +64, +96 are the low nibbles of ql[64n+l], ql[64n+32+l], then their high
 * nibbles, each with two bits of qh[32n+l] (bits 0-1, 2-3, 4-5, 6-7) on top, minus 32, scaled by
 * d * scales[8n + l/16 + 0, 2, 4, 6]. */
static float orc_dot_q6_block(const uint8_t *b, const float *x)
{
    const uint8_t *ql = b, *qh = b + 128;
    const int8_t *sc = (const int8_t *)(b + 192);
    const float d = orc_f16_to_f32((uint16_t)(b[208] | (b[209] << 8)));
    float sum = 0.0f;
    for (int n = 0; n < 2; n++)
        for (int l = 0; l < 32; l++) {
            const int a = ql[64 * n + l], c = ql[64 * n + 32 + l], h = qh[32 * n + l];
            const int q[4] = {(a & 15) | ((h & 3) << 4), (c & 15) | (((h >> 2) & 3) << 4),
                              (a >> 4) | (((h >> 4) & 3) << 4), (c >> 4) | (((h >> 6) & 3) << 4)};
            for (int k = 0; k < 4; k++)
                sum += d * (float)sc[8 * n + l / 16 + 2 * k] * (float)(q[k] - 32) * x[128 * n + 32 * k + l];
        }
    return sum;
}

void orc_matvec_q(int is_q6, const uint8_t *m, const float *x, float *out, size_t rows, size_t cols)
{
    const size_t nb = cols / 256, bs = is_q6 ? 210 : 144;
    for (size_t r = 0; r < rows; r++) {
        float acc = 0.0f;
        for (size_t b = 0; b < nb; b++) {
            const uint8_t *blk = m + (r * nb + b) * bs;
            acc += is_q6 ? orc_dot_q6_block(blk, x + 256 * b) : orc_dot_q4_block(blk, x + 256 * b);
        }
        out[r] = acc;
    }
}
