// Gated DeltaNet prefill on sm_100a tensor cores: the chunked (WY) form of the delta rule.
//
// Replaces the per-token loop of pf_ssm (reference src/model.c:1644-1658, which calls
// delta_head, model.c:1507-1534, once per token and value head). Per value head vh (key head
// vh % 16) and token t, with d_t = exp(g_t):
//     delta_t = beta_t (v_t - d_t S_{t-1}^T k_t),  S_t = d_t S_{t-1} + k_t delta_t^T,
//     o_t = S_t^T q_t / sqrt(128).
// Over a chunk of C = 64 tokens starting from state S_0, with G_i = sum_{l<=i} g_l and
// gamma_i = exp(G_i) (row i = token i of the chunk):
//     L_ij  = beta_i exp(G_i - G_j) k_i.k_j        (j < i)      T = (I + L)^-1
//     M_ij  = exp(G_i - G_j) q_i.k_j               (j <= i)
//     U = T diag(beta) V,  W = T diag(beta gamma) K,  Delta = U - W S_0
//     O = (diag(gamma) Q S_0 + M Delta) / sqrt(128)
//     S_C = gamma_C S_0 + K^T diag(exp(G_C - G_j)) Delta
// which is the same recurrence regrouped (no approximation).
//
// One CTA per (prompt, value head) walks the prompt's chunks in order. Everything is computed
// transposed, so that each product lands in tensor memory with one value (or key) dimension
// per TMEM lane and one thread owns each lane:
//   (a) [K;Q] K^T            128 x 64, K = 128 keys
//   (b) U^T = V^T (T b)^T,  W^T = K^T (T bg)^T       128 x 64 each, K = 64 tokens
//   (c) S_0^T W^T,  (d1) S_0^T Q^T                    128 x 64, A = S_0^T from TMEM
//   (d2) Delta^T M^T                                  128 x 64
//   (e) Delta''^T K                                   128 x 128 (state update)
// The fp32 state S^T stays in TMEM for the whole prompt (128 columns). T = (I + L)^-1 is formed
// on the CUDA cores of the producer warps (16 x 16 diagonal blocks by substitution, then three
// levels of block products between hardware barriers).
//
// Precision: every operand is split into two f16 parts, x = hi + lo, and each product is
// hi*hi + hi*lo + lo*hi with fp32 accumulation -- about 22 significant bits, which keeps the
// state within 1e-6 of the sequential fp32 recurrence. Before a split each operand row is scaled
// by a power of two so its largest magnitude is in [1, 2) (exact, and undone on the result):
// a scale along a product's M or N dimension factors out of the result; scales along the
// contraction dimension (the token rows of K and V) are folded into the other operand.
//
// Roles (384 threads): warps 0-3 own TMEM lanes 0-127 and do the chunk arithmetic; thread 0
// also issues every tcgen05.mma. Warps 4-11 load the next chunk's q/k/v rows into registers
// while the current chunk runs, then scale, split and store them once the chunk's last MMA
// has committed, then write the finished chunk's outputs from tensor memory (two warps per TMEM
// lane quarter, 32 tokens each), and form the new chunk's T block once (a) lands -- L from the K
// rows of (a), T = (I + L)^-1, and the B operands of (b) -- while the arithmetic warps build M.
#include "ptx.cuh"
#include "runtime.h"
#include "tcgen05.cuh"
#include "../../include/roaster_cuda.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstring>
#include <vector>

namespace rb {
namespace {

constexpr int kC = 64;                 // chunk length (tokens)
constexpr int kD = 128;                // head dim
constexpr int kThreads = 384;
constexpr int kProdThreads = 256;
constexpr int kMaxJobs = 64;
constexpr uint32_t kTmemCols = 512;
constexpr double kLog2eD = 1.4426950408889634;
constexpr float kOutScale = 0.08838834764831845f;   // 1 / sqrt(128)

// TMEM columns
constexpr uint32_t kColS = 0;          // master state S^T (fp32)
constexpr uint32_t kColS0 = 128;       // S_0^T split: hi [128,192), lo [192,256); also (e)'s result
constexpr uint32_t kColA = 256;        // (a), later (c)
constexpr uint32_t kColU = 320;        // U^T, later (d2)
constexpr uint32_t kColW = 384;        // W^T
constexpr uint32_t kColD1 = 448;       // (d1)

// Shared-memory regions (byte offsets from a 1024-aligned base). Tiles are 128-byte-swizzled
// [rows][128 B] blocks; a "half" is 8 KB (64 rows) or 16 KB (128 rows).
constexpr uint32_t kOffKQH = 0;        // [K c0 | Q c0 | K c1 | Q c1] hi, 4 x 8 KB
constexpr uint32_t kOffKQL = 32768;    // same, lo
constexpr uint32_t kOffV = 65536;      // V hi [c0|c1] 16 KB, V lo 16 KB
constexpr uint32_t kOffB = 98304;      // BV hi, BV lo, BK hi, BK lo (8 KB each);
                                       // later Delta^T hi|lo
constexpr uint32_t kOffW = 131072;     // T (fp32 scratch), then W' hi|lo, then Delta''^T hi|lo
constexpr uint32_t kOffM = 163840;     // M hi, M lo (8 KB each)
constexpr uint32_t kOffConst = 180224; // ChunkConst[2]
constexpr int kLd = 68;                // fp32 scratch row stride of L and T (floats; rows 16-byte aligned)

struct ChunkConst {
    float glf[kC];                     // G_j * log2(e) (summed in double, rounded once)
    float beta[kC];
    float isk[kC], isq[kC], isv[kC];   // inverse row scales of K, Q, V
    float gq[kC];                      // exp(G_j) / s^q_j
    float bv[kC];                      // beta_j / s^v_j
    float bk[kC];                      // beta_j exp(G_j) / s^k_j
    float df[kC];                      // exp(G_C - G_j) / s^k_j
    float gC;                          // exp(G_C)
    float pad[3];
};
static_assert(sizeof(ChunkConst) % 16 == 0, "");
constexpr uint32_t kOffCons = kOffConst + 2 * sizeof(ChunkConst);   // consumer scratch
struct ConsScratch {
    float iu_v[kC], iu_k[kC];
    float imu[2][kC];                  // M row scales, by chunk parity (read by the output epilogue)
    float sig[2][kD], rho[2][kD];      // per value row: 1 / scale of S_0 and of Delta, by chunk parity
    float red[4];
};
constexpr uint32_t kOffBars = kOffCons + ((sizeof(ConsScratch) + 15) / 16) * 16;
constexpr uint32_t kOffL = 188416;     // L, then L' (fp32, row stride kLd) while T is formed
constexpr uint32_t kOffE = kOffL + 64 * kLd * 4;   // decay factors 2^(G_i - G_j), j <= i (fp32, stride kLd)
constexpr size_t kSmemBytes = kOffE + 64 * kLd * 4 + 1024;
static_assert(kOffBars + 128 <= kOffL, "barriers overlap L");
static_assert(kSmemBytes <= 232448, "shared memory exceeds a CTA's");

struct DJob {
    float *state;
    const float *q, *k, *v, *g, *beta;
    float *out;
    long long T;
};

struct DPParams {
    DJob jobs[kMaxJobs];
    unsigned *err;
};

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ float ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Power of two s with amax * s in [1, 2) (1 for zero or non-finite amax).
__device__ __forceinline__ float pow2_scale(float amax)
{
    const int e = (int)((__float_as_uint(amax) >> 23) & 255u) - 127;
    if (!(amax > 0.f) || e == 128)
        return 1.f;
    const int ec = e < -100 ? -100 : (e > 100 ? 100 : e);
    return __uint_as_float((uint32_t)(127 - ec) << 23);
}

// x = hi + lo for a pair (a, b): packed f16x2 hi and lo words (a in the low half).
__device__ __forceinline__ void split2(float a, float b, uint32_t &hw, uint32_t &lw)
{
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
    hw = *reinterpret_cast<const uint32_t *>(&h);
    lw = *reinterpret_cast<const uint32_t *>(&l);
}

// 1 / s for a power of two s in [2^-100, 2^100] (exact, no divide).
__device__ __forceinline__ float pow2_inv(float s)
{
    return __uint_as_float((254u << 23) - __float_as_uint(s));
}

__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w)
{
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

__device__ __forceinline__ void sts64(uint32_t a, uint32_t x, uint32_t y)
{
    asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(a), "r"(x), "r"(y) : "memory");
}

// Row r (64 values, times s) of a K-major swizzled tile pair (hi, lo): 8 x 16-byte units.
__device__ __forceinline__ void store_row_split(uint32_t hi, uint32_t lo, int r, const float (&x)[kC], float s)
{
#pragma unroll
    for (int u = 0; u < 8; u++) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int p = 0; p < 4; p++)
            split2(x[8 * u + 2 * p] * s, x[8 * u + 2 * p + 1] * s, h[p], l[p]);
        const uint32_t off = (uint32_t)r * 128u + (((uint32_t)u ^ (uint32_t)(r & 7)) << 4);
        sts128(hi + off, h[0], h[1], h[2], h[3]);
        sts128(lo + off, l[0], l[1], l[2], l[3]);
    }
}

__device__ __forceinline__ float row_amax(const float (&x)[kC])
{
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < kC; i++)
        m = fmaxf(m, fabsf(x[i]));
    return m;
}

__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&x)[kC])
{
    float a[32], b[32];
    tc::tmem_ld32(taddr, a);
    tc::tmem_ld32(taddr + 32, b);
    tc::tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; i++) {
        x[i] = a[i];
        x[i + 32] = b[i];
    }
}

// T = (I + L)^-1 for the 64 x 64 strictly lower L in 16 x 16 blocks (fp32 scratch, row stride
// kLd), by the 256 producer threads; the threads always reach the same barriers (named barrier
// BAR): no step here waits on anything else.
//  1. Forward substitution through each diagonal block (I + L_ii), one right-hand-side column per
//     thread: the unit columns give T_ii = (I + L_ii)^-1, the columns of the blocks L_im (m < i)
//     give L'_im = T_ii L_im, written over L_im (160 columns; L_ii itself is only read).
//  2. By distance d = 1..3: T_ij = -sum_{m=j}^{i-1} L'_im T_mj, one step per distance with the
//     (4 - d) blocks split into 1 x 4 strips, one per thread (k = q / 64, rr = q / 4 % 16,
//     cc = 4 (q % 4)): T and the results move as 16-byte words and L' as a broadcast.
__device__ __forceinline__ void fma4(float4 &a, float s, const float4 &t)
{
    a.x = fmaf(s, t.x, a.x);
    a.y = fmaf(s, t.y, a.y);
    a.z = fmaf(s, t.z, a.z);
    a.w = fmaf(s, t.w, a.w);
}

template <int D>
__device__ __forceinline__ void inv_level(const float *Lp, float *Tm, int q)
{
    const int k = q >> 6, rr = (q >> 2) & 15, c4 = 4 * (q & 3);
    {
        const float *lrow = Lp + (16 * (k + D) + rr) * kLd + 16 * k;
        const float *tcol = Tm + 16 * k * kLd + 16 * k + c4;
        float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
#pragma unroll
        for (int m = 0; m < 16 * D; m += 2) {
            fma4(a0, lrow[m], *reinterpret_cast<const float4 *>(tcol + m * kLd));
            fma4(a1, lrow[m + 1], *reinterpret_cast<const float4 *>(tcol + (m + 1) * kLd));
        }
        *reinterpret_cast<float4 *>(Tm + (16 * (k + D) + rr) * kLd + 16 * k + c4) =
            make_float4(-(a0.x + a1.x), -(a0.y + a1.y), -(a0.z + a1.z), -(a0.w + a1.w));
    }
}

// NU 16-byte units (8 values each, times s) of row r of a K-major swizzled tile pair (hi, lo),
// starting at unit u0.
template <int NU>
__device__ __forceinline__ void store_units(uint32_t hi, uint32_t lo, int r, int u0, const float (&x)[8 * NU], float s)
{
#pragma unroll
    for (int u = 0; u < NU; u++) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int p = 0; p < 4; p++)
            split2(x[8 * u + 2 * p] * s, x[8 * u + 2 * p + 1] * s, hw[p], lw[p]);
        const uint32_t off = (uint32_t)r * 128u + ((((uint32_t)(u0 + u)) ^ (uint32_t)(r & 7)) << 4);
        sts128(hi + off, hw[0], hw[1], hw[2], hw[3]);
        sts128(lo + off, lw[0], lw[1], lw[2], lw[3]);
    }
}

// B operands of (b) for the 16 rows of block rb: rows of T diag(beta / s^v) (BV, tasks 0-15) and
// T diag(beta gamma / s^k) (BK, tasks 16-31), each split hi + lo with its own power-of-two scale;
// G threads (adjacent lanes, t = G task + h) per row, 64 / G columns each.
template <int G>
__device__ __forceinline__ void b_rows(const float *Tm, const ChunkConst &C, ConsScratch *cs, uint32_t bbase, int rb,
                                       int t)
{
    constexpr int NV = 64 / G;
    const int task = t / G, h = t % G, i = 16 * rb + (task & 15);
    const bool isv = task < 16;
    const float *bsrc = isv ? C.bv : C.bk;
    float x[NV];
#pragma unroll
    for (int j4 = 0; j4 < NV; j4 += 4) {
        const int j = NV * h + j4;
        const float4 t4 = *reinterpret_cast<const float4 *>(Tm + i * kLd + j);
        const float4 b4 = *reinterpret_cast<const float4 *>(bsrc + j);
        x[j4] = j <= i ? t4.x * b4.x : 0.f;
        x[j4 + 1] = j + 1 <= i ? t4.y * b4.y : 0.f;
        x[j4 + 2] = j + 2 <= i ? t4.z * b4.z : 0.f;
        x[j4 + 3] = j + 3 <= i ? t4.w * b4.w : 0.f;
    }
    float m = 0.f;
#pragma unroll
    for (int jj = 0; jj < NV; jj++)
        m = fmaxf(m, fabsf(x[jj]));
#pragma unroll
    for (int o = 1; o < G; o <<= 1)
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float u = pow2_scale(m);
    const uint32_t hi = bbase + (isv ? 0u : 16384u);
    store_units<NV / 8>(hi, hi + 8192, i, (NV / 8) * h, x, u);
    if (h == 0) {
        if (isv)
            cs->iu_v[i] = pow2_inv(u);
        else
            cs->iu_k[i] = pow2_inv(u);
    }
    fence_proxy_async();
}

template <int BAR>
__device__ __forceinline__ void tri_inverse(float *Lw, float *Tm, int q, const ChunkConst &C, ConsScratch *cs,
                                            uint32_t bbase)
{
    if (q < 160) {
        int i, c;                                    // block row, column within [0, 16 i + 16)
        bool unit;
        if (q < 64) {
            i = q >> 4;
            c = 16 * i + (q & 15);
            unit = true;
        } else {
            const int u = q - 64;
            i = u < 16 ? 1 : (u < 48 ? 2 : 3);
            c = u - (i == 1 ? 0 : (i == 2 ? 16 : 48));
            unit = false;
        }
        const float *Lii = Lw + 16 * i * kLd + 16 * i;
        float y[16];
#pragma unroll
        for (int rr = 0; rr < 16; rr++) {
            float acc = unit ? (16 * i + rr == c ? 1.f : 0.f) : Lw[(16 * i + rr) * kLd + c];
#pragma unroll
            for (int m = 0; m < rr; m++)
                acc = fmaf(-Lii[rr * kLd + m], y[m], acc);
            y[rr] = acc;
        }
        float *dst = unit ? Tm : Lw;
#pragma unroll
        for (int rr = 0; rr < 16; rr++)
            dst[(16 * i + rr) * kLd + c] = y[rr];
    }
    named_bar_sync(BAR, 256);
    if (q < 192)
        inv_level<1>(Lw, Tm, q);
    named_bar_sync(BAR, 256);
    if (q < 128)
        inv_level<2>(Lw, Tm, q);
    named_bar_sync(BAR, 256);
    if (q < 64)
        inv_level<3>(Lw, Tm, q);
    named_bar_sync(BAR, 256);
    // the B operands of (b): 64 threads per 16-row block, two per row
    b_rows<2>(Tm, C, cs, bbase, q >> 6, q & 63);
}

__global__ void __launch_bounds__(kThreads, 1) deltanet_prefill_kernel(const __grid_constant__ DPParams p)
{
    extern __shared__ unsigned char smem_raw[];
    const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;
    unsigned char *gbase = smem_raw + (base - smem_addr(smem_raw));
    ChunkConst *cc = reinterpret_cast<ChunkConst *>(gbase + kOffConst);
    ConsScratch *cs = reinterpret_cast<ConsScratch *>(gbase + kOffCons);
    unsigned long long *bars = reinterpret_cast<unsigned long long *>(gbase + kOffBars);
    const uint32_t in_full = smem_addr(&bars[0]), mma_bar = smem_addr(&bars[1]);
    const uint32_t done_bar = smem_addr(&bars[2]), drain_bar = smem_addr(&bars[3]);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(&bars[4]);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(&bars[5]);
    const uint32_t out_bar = smem_addr(&bars[6]);     // producers have read a chunk's outputs from TMEM
    const uint32_t a_bar = smem_addr(&bars[7]);       // (a) of the chunk has landed in TMEM
    const uint32_t t_bar = smem_addr(&bars[8]);       // producers have stored the B operands of (b)
    const uint32_t b_bar = smem_addr(&bars[9]);       // (b) has finished reading V
    const uint32_t cd_bar = smem_addr(&bars[10]);     // (c, d1) have finished reading Q (and W')

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int vh = blockIdx.x, kh = vh & 15;
    const DJob &J = p.jobs[blockIdx.y];
    const long long T = J.T;
    const int nchunks = (int)((T + kC - 1) / kC);

    if (tid == 0) {
        mbar_init(in_full, kProdThreads / 32);
        mbar_init(mma_bar, 1);
        mbar_init(done_bar, 1);
        mbar_init(drain_bar, 1);
        mbar_init(out_bar, kProdThreads / 32);
        mbar_init(a_bar, 1);
        mbar_init(t_bar, kProdThreads / 32);
        mbar_init(b_bar, 1);
        mbar_init(cd_bar, 1);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 0) {
        tc::tmem_alloc(smem_addr(tmem_slot), kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tb = *tmem_slot;

    auto set_abort = [&]() {
        atomicOr(p.err, kErrWaitTimeout);
        *abort_flag = 1;
    };

    if (warp >= 4) {
        // ============================================================ producers
        const int pw = warp - 4;                       // 0..7, rows pw + 8 s
        float4 buf[24];
        float gv0 = 0.f, gv1 = 0.f, bv0 = 0.f, bv1 = 0.f, dfa = 0.f, dfb = 0.f;
        double ga = 0.0, gb = 0.0;
        auto issue_loads = [&](int n) {
            const long long t0 = (long long)n * kC;
            const int tc_ = (int)(T - t0 < kC ? T - t0 : kC);
#pragma unroll
            for (int s = 0; s < 24; s++) {
                const int rr = pw + 8 * s, which = rr >> 6, j = rr & 63;
                float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
                if (j < tc_) {
                    const long long t = t0 + j;
                    const float *src = which == 0 ? J.k + (t * 16 + kh) * kD
                                     : which == 1 ? J.q + (t * 16 + kh) * kD
                                                  : J.v + (t * 32 + vh) * kD;
                    x = __ldg(reinterpret_cast<const float4 *>(src) + lane);
                }
                buf[s] = x;
            }
            if (pw == 0) {
                gv0 = gv1 = bv0 = bv1 = 0.f;
                if (lane < tc_) {
                    gv0 = __ldg(J.g + (t0 + lane) * 32 + vh);
                    bv0 = __ldg(J.beta + (t0 + lane) * 32 + vh);
                }
                if (lane + 32 < tc_) {
                    gv1 = __ldg(J.g + (t0 + lane + 32) * 32 + vh);
                    bv1 = __ldg(J.beta + (t0 + lane + 32) * 32 + vh);
                }
            }
        };
        issue_loads(0);
        for (int n = 0; n < nchunks; n++) {
            ChunkConst &C = cc[n & 1];
            // scale, split and store this chunk's rows s0 .. s0 + 7 of the 24 a warp holds
            // (rows pw + 8 s: s 0-7 K, 8-15 Q, 16-23 V)
            auto stage = [&](int s0) {
#pragma unroll
                for (int s = s0; s < s0 + 8; s++) {
                    const int rr = pw + 8 * s, which = rr >> 6, j = rr & 63;
                    const float4 x = buf[s];
                    // non-negative floats order like their bit patterns: one warp max-reduction
                    const float m0 = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
                    const float sc = pow2_scale(__uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m0))));
                    uint32_t h0, l0, h1, l1;
                    split2(x.x * sc, x.y * sc, h0, l0);
                    split2(x.z * sc, x.w * sc, h1, l1);
                    const uint32_t c = (uint32_t)lane >> 4;                    // 64-column chunk
                    const uint32_t unit = ((uint32_t)(lane & 15) >> 1) ^ (uint32_t)(j & 7);
                    const uint32_t inner = (uint32_t)j * 128u + (unit << 4) + (uint32_t)(lane & 1) * 8u;
                    uint32_t hi, lo;
                    if (which == 2) {
                        hi = base + kOffV + c * 8192u;
                        lo = hi + 16384u;
                    } else {
                        hi = base + kOffKQH + c * 16384u + (uint32_t)which * 8192u;
                        lo = hi + (kOffKQL - kOffKQH);
                    }
                    sts64(hi + inner, h0, h1);
                    sts64(lo + inner, l0, l1);
                    if (lane == 0) {
                        const float inv = pow2_inv(sc);
                        if (which == 0) C.isk[j] = inv;
                        else if (which == 1) C.isq[j] = inv;
                        else C.isv[j] = inv;
                    }
                }
            };
            // V once (b) of chunk n - 1 has read it, Q once (c, d1) have, K once the chunk's last
            // MMAs (d2, e) have committed
            auto gate = [&](uint32_t bar) -> bool {
                const bool w = n == 0 || mbar_wait_sleep(bar, (uint32_t)(n - 1) & 1u, 64);
                if (!bar_all(3, kProdThreads, w && !*abort_flag)) {
                    if (tid == kThreads - kProdThreads)
                        set_abort();
                    return false;
                }
                return true;
            };
            if (!gate(b_bar))
                break;
            // g prefix sums (pw == 0) and, after the V rows, the chunk's decay factors E (the
            // arithmetic warps finished reading chunk n - 1's E, in M, before they issued its (b))
            if (pw == 0) {
                // prefix sums of g * log2(e) in double
                double a = (double)gv0 * kLog2eD, b = (double)gv1 * kLog2eD;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const double ua = __shfl_up_sync(0xffffffffu, a, o);
                    const double ub = __shfl_up_sync(0xffffffffu, b, o);
                    if (lane >= o) {
                        a += ua;
                        b += ub;
                    }
                }
                b += __shfl_sync(0xffffffffu, a, 31);
                const double gl_last = __shfl_sync(0xffffffffu, b, 31);
                ga = a;
                gb = b;
                C.glf[lane] = (float)a;
                C.glf[lane + 32] = (float)b;
                C.beta[lane] = bv0;
                C.beta[lane + 32] = bv1;
                dfa = ex2((float)(gl_last - a));
                dfb = ex2((float)(gl_last - b));
                if (lane == 0)
                    C.gC = ex2((float)gl_last);
            }
            stage(16);
            named_bar_sync(3, kProdThreads);
            {
                float *Ew = reinterpret_cast<float *>(gbase + kOffE);
                const int pq = tid - (kThreads - kProdThreads);
#pragma unroll 4
                for (int e = pq; e < kC * kC; e += kProdThreads) {
                    const int i = e >> 6, j = e & 63;
                    Ew[i * kLd + j] = j <= i ? ex2(C.glf[i] - C.glf[j]) : 0.f;
                }
            }
            if (!gate(cd_bar))
                break;
            stage(8);
            if (!gate(done_bar))
                break;
            stage(0);
            named_bar_sync(3, kProdThreads);
            if (pw == 0) {
                // per-token factors that need every row scale
                const float e0 = ex2((float)ga), e1 = ex2((float)gb);
                C.gq[lane] = e0 * C.isq[lane];
                C.gq[lane + 32] = e1 * C.isq[lane + 32];
                C.bv[lane] = bv0 * C.isv[lane];
                C.bv[lane + 32] = bv1 * C.isv[lane + 32];
                C.bk[lane] = bv0 * e0 * C.isk[lane];
                C.bk[lane + 32] = bv1 * e1 * C.isk[lane + 32];
                C.df[lane] = dfa * C.isk[lane];
                C.df[lane + 32] = dfb * C.isk[lane + 32];
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(in_full);
            if (n > 0) {
                // outputs of chunk n - 1 (a full chunk: only the last can be short), whose MMAs
                // completed before done_bar's phase n - 1; the arithmetic warps wait on out_bar
                // before the MMAs that overwrite these columns
                tc::fence_after_sync();
                const int q4 = warp & 3, half = pw >> 2;          // TMEM lane quarter, 32-token half
                const int rr = 32 * q4 + lane;                     // value row
                const uint32_t lq = (uint32_t)(32 * q4) << 16;
                const int pb = (n - 1) & 1;
                const ChunkConst &Cp = cc[pb];
                const float sg = cs->sig[pb][rr] * kOutScale, rh = cs->rho[pb][rr] * kOutScale;
#pragma unroll 1
                for (int h = 0; h < 2; h++) {
                    const int c0 = 32 * half + 16 * h;             // first token of this group
                    float d1[16], d2[16];
                    tc::tmem_ld16(tb + lq + kColD1 + c0, d1);
                    tc::tmem_ld16(tb + lq + kColU + c0, d2);
                    tc::tmem_wait_ld();
                    float *o = J.out + (((long long)(n - 1) * kC + c0) * 32 + vh) * kD + rr;
#pragma unroll
                    for (int i = 0; i < 16; i++)
                        o[(long long)i * 32 * kD] = Cp.gq[c0 + i] * sg * d1[i] + cs->imu[pb][c0 + i] * rh * d2[i];
                }
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(out_bar);
            }
            // ---- T block of chunk n: L from the K rows of (a), T = (I + L)^-1, B operands of (b)
            {
                const bool w = mbar_wait_sleep(a_bar, (uint32_t)n & 1u, 64);
                if (!bar_all(3, kProdThreads, w && !*abort_flag)) {
                    if (tid == kThreads - kProdThreads)
                        set_abort();
                    break;
                }
                tc::fence_after_sync();
                const int pq = tid - (kThreads - kProdThreads);   // 0..255
                float *Lw = reinterpret_cast<float *>(gbase + kOffL);
                const float *Ew = reinterpret_cast<const float *>(gbase + kOffE);
                float *Tm = reinterpret_cast<float *>(gbase + kOffW);
                const int q4 = warp & 3, half = pw >> 2;
                if (q4 < 2) {
                    // row i of L, columns 32 half .. 32 half + 31 (TMEM lanes 0-63 hold (a)'s K rows)
                    const int i = 32 * q4 + lane;
                    float x[32];
                    tc::tmem_ld32(tb + ((uint32_t)(32 * q4) << 16) + kColA + 32 * half, x);
                    tc::tmem_wait_ld();
                    const float f = C.beta[i] * C.isk[i];
#pragma unroll
                    for (int j4 = 0; j4 < 32; j4 += 4) {
                        const int j = 32 * half + j4;
                        const float4 e4 = *reinterpret_cast<const float4 *>(Ew + i * kLd + j);
                        const float4 s4 = *reinterpret_cast<const float4 *>(&C.isk[j]);
                        float4 l;
                        l.x = j < i ? f * e4.x * x[j4] * s4.x : 0.f;
                        l.y = j + 1 < i ? f * e4.y * x[j4 + 1] * s4.y : 0.f;
                        l.z = j + 2 < i ? f * e4.z * x[j4 + 2] * s4.z : 0.f;
                        l.w = j + 3 < i ? f * e4.w * x[j4 + 3] * s4.w : 0.f;
                        *reinterpret_cast<float4 *>(Lw + i * kLd + j) = l;
                    }
                }
                tc::fence_before_sync();
                named_bar_sync(3, kProdThreads);
                tri_inverse<3>(Lw, Tm, pq, C, cs, base + kOffB);
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(t_bar);
            }
            // keep the next chunk's loads (96 registers) from being hoisted above the work before
            asm volatile("" ::: "memory");
            if (n + 1 < nchunks)
                issue_loads(n + 1);
        }
    } else {
        // ============================================================ chunk arithmetic
        const int r = tid;                                  // TMEM lane: value (or key) index
        const uint32_t lrow = (uint32_t)(32 * warp) << 16;  // lane offset of this warp
        // shared-memory operand descriptors (the layout is static; MMAs add compile-time offsets)
        const uint64_t dKQH = tc::smem_desc(base + kOffKQH, 16, 1024), dKQL = tc::smem_desc(base + kOffKQL, 16, 1024);
        const uint64_t dKQHm = tc::smem_desc(base + kOffKQH, 16384, 1024);     // K' as MN-major operand
        const uint64_t dKQLm = tc::smem_desc(base + kOffKQL, 16384, 1024);
        const uint64_t dVm = tc::smem_desc(base + kOffV, 8192, 1024);          // V' (MN-major); lo at +16 KB
        const uint64_t dVk = tc::smem_desc(base + kOffW, 16, 1024);            // Delta''^T (K-major)
        const uint64_t dB = tc::smem_desc(base + kOffB, 16, 1024);             // BV, BK; later Delta^T
        const uint64_t dWm = tc::smem_desc(base + kOffW, 8192, 1024);          // W' (MN-major)
        const uint64_t dM = tc::smem_desc(base + kOffM, 16, 1024);
        float inv_sigma = 1.f, inv_rho = 1.f, inv_rho2 = 1.f, inv_omega = 1.f;
        uint32_t mphase = 0;
        bool ok = true;

        auto wait_mma = [&]() -> bool {
            const bool w = mbar_wait_sleep(mma_bar, mphase & 1u, 32);
            mphase++;
            const bool all = bar_all(1, 128, w && !*abort_flag);
            if (!all && tid == 0)
                set_abort();
            if (all)
                tc::fence_after_sync();
            return all;
        };

        // S_0^T of chunk m split into TMEM columns [128, 256) from the master, with row scale sigma
        // (its inverse also kept for the output epilogue).
        auto write_s0 = [&](int m) {
            float amax = 0.f;
#pragma unroll 1
            for (int c = 0; c < kD; c += 32) {
                float x[32];
                tc::tmem_ld32(tb + lrow + kColS + c, x);
                tc::tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i++)
                    amax = fmaxf(amax, fabsf(x[i]));
            }
            const float sg = pow2_scale(amax);
            inv_sigma = pow2_inv(sg);
            cs->sig[m & 1][r] = inv_sigma;
#pragma unroll 1
            for (int c = 0; c < kD; c += 32) {
                float x[32];
                tc::tmem_ld32(tb + lrow + kColS + c, x);
                tc::tmem_wait_ld();
                uint32_t h[16], l[16];
#pragma unroll
                for (int i = 0; i < 16; i++)
                    split2(x[2 * i] * sg, x[2 * i + 1] * sg, h[i], l[i]);
                tc::tmem_st16(tb + lrow + kColS0 + (c >> 1), h);
                tc::tmem_st16(tb + lrow + kColS0 + 64 + (c >> 1), l);
            }
            tc::tmem_wait_st();
        };

        // Outputs and state update of chunk n (its last MMAs have committed to done_bar).
        auto finish = [&](int n, bool last) -> bool {
            const bool w = mbar_wait_sleep(done_bar, (uint32_t)n & 1u, 32);
            if (!bar_all(1, 128, w && !*abort_flag)) {
                if (tid == 0)
                    set_abort();
                return false;
            }
            tc::fence_after_sync();
            const ChunkConst &C = cc[n & 1];
            const long long t0 = (long long)n * kC;
            const int tcn = (int)(T - t0 < kC ? T - t0 : kC);
            if (last) {
                // the last chunk's outputs (the producer warps write the others)
                float d1[kC], d2[kC];
                tmem_ld64(tb + lrow + kColD1, d1);
                tmem_ld64(tb + lrow + kColU, d2);
                float *o = J.out + (t0 * 32 + vh) * kD + r;
#pragma unroll
                for (int i = 0; i < kC; i++) {
                    if (i < tcn)
                        o[(long long)i * 32 * kD] =
                            kOutScale * (C.gq[i] * inv_sigma * d1[i] + cs->imu[n & 1][i] * inv_rho * d2[i]);
                }
            }
            const float gC = C.gC;
#pragma unroll 1
            for (int c = 0; c < kD; c += 32) {
                float s[32], e[32];
                tc::tmem_ld32(tb + lrow + kColS + c, s);
                tc::tmem_ld32(tb + lrow + kColS0 + c, e);
                tc::tmem_wait_ld();
                uint32_t w32[32];
#pragma unroll
                for (int i = 0; i < 32; i++)
                    w32[i] = __float_as_uint(fmaf(gC, s[i], e[i] * inv_rho2));
                tc::tmem_st32(tb + lrow + kColS + c, w32);
            }
            tc::tmem_wait_st();
            if (!last)
                write_s0(n + 1);
            tc::fence_before_sync();
            return true;
        };

        // initial state: S^T into the master (thread r holds column r of S)
        {
            const float *S = J.state + (size_t)vh * kD * kD;
#pragma unroll 1
            for (int c = 0; c < kD; c += 32) {
                uint32_t w32[32];
#pragma unroll
                for (int i = 0; i < 32; i++)
                    w32[i] = __float_as_uint(__ldg(S + (size_t)(c + i) * kD + r));
                tc::tmem_st32(tb + lrow + kColS + c, w32);
            }
            tc::tmem_wait_st();
            write_s0(0);
            tc::fence_before_sync();
        }

        for (int n = 0; n < nchunks && ok; n++) {
            const ChunkConst &C = cc[n & 1];
            // ---- inputs of chunk n staged
            {
                const bool w = mbar_wait_sleep(in_full, (uint32_t)n & 1u, 64);
                if (!bar_all(1, 128, w && !*abort_flag)) {
                    if (tid == 0)
                        set_abort();
                    ok = false;
                    break;
                }
            }
            // ---- (a): [K;Q] K^T
            if (tid == 0) {
                tc::fence_after_sync();
                const uint32_t id = tc::idesc_f16(128, 64, 0, 0);
#pragma unroll
                for (int pp = 0; pp < 3; pp++) {
                    const uint64_t A = pp == 2 ? dKQL : dKQH, B = pp == 1 ? dKQL : dKQH;
#pragma unroll
                    for (int kk = 0; kk < 8; kk++) {
                        const uint32_t off = (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u;
                        tc::mma_ss_f16(tb + kColA, tc::desc_adv(A, off), tc::desc_adv(B, off), id, (pp | kk) ? 1u : 0u);
                    }
                }
                tc::commit(mma_bar);
                tc::commit(a_bar);
            }
            // ---- state update of the previous chunk and S_0 of this one, while (a) runs and the
            //      producers form the T block
            if (n > 0 && !finish(n - 1, false)) {
                ok = false;
                break;
            }
            // ---- (d1) S_0^T Q'^T (A = S_0^T from TMEM) as soon as S_0 is split and the producers
            //      have read chunk n - 1's outputs from its columns
            {
                bool ob = true;
                if (n > 0 && tid == 0)
                    ob = mbar_wait_sleep(out_bar, (uint32_t)(n - 1) & 1u, 64);
                if (!bar_all(1, 128, ob && !*abort_flag)) {
                    if (tid == 0)
                        set_abort();
                    ok = false;
                    break;
                }
            }
            if (tid == 0) {
                tc::fence_after_sync();
                const uint32_t idd = tc::idesc_f16(128, 64, 0, 0);
#pragma unroll
                for (int pp = 0; pp < 3; pp++) {
                    const uint32_t Aa = tb + kColS0 + (pp == 2 ? 64u : 0u);
                    const uint64_t Qb = tc::desc_adv(pp == 1 ? dKQL : dKQH, 8192u);
#pragma unroll
                    for (int kk = 0; kk < 8; kk++)
                        tc::mma_ts_f16(tb + kColD1, Aa + kk * 8u,
                                       tc::desc_adv(Qb, (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u), idd,
                                       (pp | kk) ? 1u : 0u);
                }
            }
            if (!wait_mma()) {
                ok = false;
                break;
            }
            // ---- M from the Q rows of (a) (warps 2-3; the producers take the K rows: L and T)
            if (r >= kC) {
                float x[kC];
                tmem_ld64(tb + lrow + kColA, x);
                const int i = r - kC;
                const float f = C.isq[i];
                const float *Er = reinterpret_cast<const float *>(gbase + kOffE) + i * kLd;
#pragma unroll
                for (int j4 = 0; j4 < kC; j4 += 4) {
                    const float4 e4 = *reinterpret_cast<const float4 *>(Er + j4);
                    const float4 s4 = *reinterpret_cast<const float4 *>(&C.isk[j4]);
                    x[j4] = j4 <= i ? f * e4.x * x[j4] * s4.x : 0.f;
                    x[j4 + 1] = j4 + 1 <= i ? f * e4.y * x[j4 + 1] * s4.y : 0.f;
                    x[j4 + 2] = j4 + 2 <= i ? f * e4.z * x[j4 + 2] * s4.z : 0.f;
                    x[j4 + 3] = j4 + 3 <= i ? f * e4.w * x[j4 + 3] * s4.w : 0.f;
                }
                const float mu = pow2_scale(row_amax(x));
                store_row_split(base + kOffM, base + kOffM + 8192, i, x, mu);
                cs->imu[n & 1][i] = pow2_inv(mu);
                fence_proxy_async();
            }
            // the producers have stored the B operands of (b)
            {
                bool ob = true;
                if (tid == 0)
                    ob = mbar_wait_sleep(t_bar, (uint32_t)n & 1u, 64);
                if (!bar_all(1, 128, ob && !*abort_flag)) {
                    if (tid == 0)
                        set_abort();
                    ok = false;
                    break;
                }
            }
            // ---- (b): U^T = V'^T BV'^T, W^T = K'^T BK'^T
            if (tid == 0) {
                tc::fence_after_sync();
                const uint32_t id = tc::idesc_f16(128, 64, 1, 0);
#pragma unroll
                for (int pp = 0; pp < 3; pp++) {
                    const uint64_t Ka = pp == 2 ? dKQLm : dKQHm;
                    const uint64_t Bk = tc::desc_adv(dB, pp == 1 ? 24576u : 16384u);
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        tc::mma_ss_f16(tb + kColW, tc::desc_adv(Ka, kk * 2048u), tc::desc_adv(Bk, kk * 32u), id,
                                       (pp | kk) ? 1u : 0u);
                }
                tc::commit(mma_bar);             // W^T first: its split overlaps the U^T products
#pragma unroll
                for (int pp = 0; pp < 3; pp++) {
                    const uint64_t Va = tc::desc_adv(dVm, pp == 2 ? 16384u : 0u);
                    const uint64_t Bv = tc::desc_adv(dB, pp == 1 ? 8192u : 0u);
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        tc::mma_ss_f16(tb + kColU, tc::desc_adv(Va, kk * 2048u), tc::desc_adv(Bv, kk * 32u), id,
                                       (pp | kk) ? 1u : 0u);
                }
                tc::commit(b_bar);
            }
            if (!wait_mma()) {
                ok = false;
                break;
            }
            // ---- W' = omega W^T (uniform power-of-two scale), B operand of (c)
            {
                float x[kC];
                tmem_ld64(tb + lrow + kColW, x);
                const float m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(row_amax(x))));
                if (lane == 0)
                    cs->red[warp] = m;
                named_bar_sync(1, 128);
                const float om = pow2_scale(fmaxf(fmaxf(cs->red[0], cs->red[1]), fmaxf(cs->red[2], cs->red[3])));
                inv_omega = pow2_inv(om);
                store_row_split(base + kOffW, base + kOffW + 16384, r, x, om);
                fence_proxy_async();
                tc::fence_before_sync();
            }
            named_bar_sync(1, 128);
            // ---- (c) S_0^T W', A = S_0^T from TMEM (its commit also covers (d1) and the U^T half of (b))
            if (tid == 0) {
                tc::fence_after_sync();
                const uint32_t idc = tc::idesc_f16(128, 64, 0, 1);
#pragma unroll
                for (int pp = 0; pp < 3; pp++) {
                    const uint32_t Aa = tb + kColS0 + (pp == 2 ? 64u : 0u);
                    const uint64_t Wb = tc::desc_adv(dWm, pp == 1 ? 16384u : 0u);
#pragma unroll
                    for (int kk = 0; kk < 8; kk++)
                        tc::mma_ts_f16(tb + kColA, Aa + kk * 8u, tc::desc_adv(Wb, kk * 2048u), idc, (pp | kk) ? 1u : 0u);
                }
                tc::commit(mma_bar);
                tc::commit(cd_bar);
            }
            if (!wait_mma()) {
                ok = false;
                break;
            }
            // ---- Delta^T = U^T - S_0^T W^T; its split (A of d2) and Delta''^T (A of e)
            {
                float dl[kC];
                {
                    float u[kC], c[kC];
                    tmem_ld64(tb + lrow + kColU, u);
                    tmem_ld64(tb + lrow + kColA, c);
                    const float f = inv_sigma * inv_omega;
#pragma unroll
                    for (int i = 0; i < kC; i++)
                        dl[i] = u[i] * cs->iu_v[i] - c[i] * (cs->iu_k[i] * f);
                }
                const float rho = pow2_scale(row_amax(dl));
                inv_rho = pow2_inv(rho);
                cs->rho[n & 1][r] = inv_rho;
                store_row_split(base + kOffB, base + kOffB + 16384, r, dl, rho);
#pragma unroll
                for (int j = 0; j < kC; j++)
                    dl[j] *= C.df[j];
                const float rho2 = pow2_scale(row_amax(dl));
                inv_rho2 = pow2_inv(rho2);
                store_row_split(base + kOffW, base + kOffW + 16384, r, dl, rho2);
                fence_proxy_async();
                tc::fence_before_sync();
            }
            named_bar_sync(1, 128);
            // ---- (d2) Delta^T M^T and (e) Delta''^T K -> done_bar
            if (tid == 0) {
                tc::fence_after_sync();
                const uint32_t idd = tc::idesc_f16(128, 64, 0, 0);
                const uint32_t ide = tc::idesc_f16(128, 128, 0, 1);
#pragma unroll
                for (int pp = 0; pp < 3; pp++) {
                    const uint64_t Da = tc::desc_adv(dB, pp == 2 ? 16384u : 0u);
                    const uint64_t Mb = tc::desc_adv(dM, pp == 1 ? 8192u : 0u);
                    const uint64_t Ea = tc::desc_adv(dVk, pp == 2 ? 16384u : 0u);
                    const uint64_t Kb = pp == 1 ? dKQLm : dKQHm;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {
                        const uint32_t acc = (pp | kk) ? 1u : 0u;
                        tc::mma_ss_f16(tb + kColU, tc::desc_adv(Da, kk * 32u), tc::desc_adv(Mb, kk * 32u), idd, acc);
                        tc::mma_ss_f16(tb + kColS0, tc::desc_adv(Ea, kk * 32u), tc::desc_adv(Kb, kk * 2048u), ide, acc);
                    }
                }
                tc::commit(done_bar);
            }
        }
        // last chunk: outputs, state update, state back to global memory
        if (ok && nchunks > 0 && finish(nchunks - 1, true)) {
            tc::fence_after_sync();
            float *S = J.state + (size_t)vh * kD * kD;
#pragma unroll 1
            for (int c = 0; c < kD; c += 32) {
                float x[32];
                tc::tmem_ld32(tb + lrow + kColS + c, x);
                tc::tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i++)
                    S[(size_t)(c + i) * kD + r] = x[i];
            }
        }
        if (tid == 0) {
            // every MMA issued must finish before tensor memory is released
            tc::commit(drain_bar);
            mbar_wait(drain_bar, 0);
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0)
        tc::tmem_dealloc(tb, kTmemCols);
}

bool g_attr = false;

int launch(const KernelDeltaPrefillJob *jobs, int n)
{
    Runtime &R = rt();
    DPParams prm;
    memset(static_cast<void *>(&prm), 0, sizeof(prm));
    int m = 0;
    for (int i = 0; i < n; i++) {
        const KernelDeltaPrefillJob &j = jobs[i];
        if (!j.state || !j.q || !j.k || !j.v || !j.g || !j.beta || !j.out)
            return fail("kernel_deltanet_prefill_batch: job %d has a null pointer", i);
        if (!aligned16(j.q) || !aligned16(j.k) || !aligned16(j.v))
            return fail("kernel_deltanet_prefill_batch: job %d q/k/v not 16-byte aligned", i);
        if (j.T == 0)
            continue;
        prm.jobs[m++] = DJob{j.state, j.q, j.k, j.v, j.g, j.beta, j.out, (long long)j.T};
    }
    if (m == 0)
        return 0;
    prm.err = R.err_word;
    if (!g_attr) {
        if (check(cudaFuncSetAttribute(deltanet_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBytes), "deltanet prefill smem attribute") != 0)
            return -1;
        g_attr = true;
    }
    deltanet_prefill_kernel<<<dim3(32, m), kThreads, kSmemBytes, R.stream>>>(prm);
    return launched("deltanet_prefill_kernel");
}

}  // namespace

int deltanet_prefill_batch(const KernelDeltaPrefillJob *jobs, int n)
{
    if (n < 0 || (n > 0 && !jobs))
        return fail("kernel_deltanet_prefill_batch: bad job array");
    for (int i = 0; i < n; i += kMaxJobs) {
        const int m = n - i < kMaxJobs ? n - i : kMaxJobs;
        if (launch(jobs + i, m) != 0)
            return -1;
    }
    return 0;
}

}  // namespace rb

using namespace rb;

extern "C" int kernel_deltanet_prefill_batch(const KernelDeltaPrefillJob *jobs, int n)
{
    if (ensure() != 0)
        return -1;
    return deltanet_prefill_batch(jobs, n);
}

extern "C" int kernel_deltanet_prefill(float *state, size_t T, const float *q, const float *k, const float *v,
                                       const float *g, const float *beta, float *out)
{
    if (ensure() != 0)
        return -1;
    if (!state || !q || !k || !v || !g || !beta || !out)
        return fail("kernel_deltanet_prefill: null pointer");
    if (T == 0)
        return 0;
    // host q, k [T][16][128], v [T][32][128], g, beta [T][32] in; out [T][32][128]
    const size_t nq = T * 16 * 128, nv = T * 32 * 128, nh = T * 32;
    const size_t oq = 0, ok_ = nq, ov = 2 * nq, og = 2 * nq + nv, ob = og + nh;
    const size_t in_f = ob + nh, out_f = nv;
    const size_t in_pad = (in_f + 3) / 4 * 4;
    float *h = static_cast<float *>(pinned((in_pad + out_f) * sizeof(float)));
    float *d = static_cast<float *>(dstage((in_pad + out_f) * sizeof(float)));
    if (!h || !d)
        return -1;
    memcpy(h + oq, q, nq * 4);
    memcpy(h + ok_, k, nq * 4);
    memcpy(h + ov, v, nv * 4);
    memcpy(h + og, g, nh * 4);
    memcpy(h + ob, beta, nh * 4);
    cudaStream_t s = rt().stream;
    if (check(cudaMemcpyAsync(d, h, in_f * 4, cudaMemcpyHostToDevice, s), "stage in") != 0)
        return -1;
    KernelDeltaPrefillJob j{state, d + oq, d + ok_, d + ov, d + og, d + ob, d + in_pad, T};
    if (deltanet_prefill_batch(&j, 1) != 0)
        return -1;
    if (check(cudaMemcpyAsync(h + in_pad, d + in_pad, out_f * 4, cudaMemcpyDeviceToHost, s), "stage out") != 0)
        return -1;
    if (kernel_cuda_synchronize() != 0)
        return -1;
    memcpy(out, h + in_pad, out_f * 4);
    return 0;
}
