// Gated GQA attention, causal prefill, on sm_100a tensor cores (tcgen05 + TMEM).
//
// Replaces the attention part of pf_attention (reference src/model.c:1553-1600):
//   per token t: RMSNorm(q_h) * qnorm, RMSNorm(k) * knorm, partial NeoX RoPE (dims 0..63,
//   theta 1e7) at position base + t, append K/V at window index kbase + t; then for each query
//   head h (kv head h / 8): softmax over window entries [0, kbase + t] of q.k / 16, times V,
//   times sigmoid(gate).
//
// Two kernels.
//  1. prefill_prep_kernel (HBM-bound, one CTA per token): norms + RoPE; writes the prepared
//     queries as f16 to scratch and appends K/V (f16) to the cache.
//  2. prefill_attn_kernel (tensor-bound): a work item is (prompt, query head, 128-token query
//     tile); persistent CTAs take items longest-first. Per CTA (416 threads):
//       warp 0      one thread issues every tcgen05.mma and commit;
//       warps 1-3, 12  producers: 16-byte cp.async into 128-byte-swizzled tiles -- the Q tile
//                   (128 x 256 f16, 64 KB) once per item, then each 128-key K and V tile as
//                   two 32 KB halves through a 5-stage ring, in the order the MMAs use them;
//       warps 4-11  softmax + epilogue: two warps per query row (= TMEM lane), each owning half
//                   of the tile's columns and half of the output dims.
//     Tensor memory (512 columns): S_j = Q K_j^T (128 x 128 fp32) double-buffered in columns
//     [0,128) and [128,256); each softmax warp writes its 64 columns of P_j as packed f16 back
//     into the S buffer, and O += P_j V_j reads P straight from TMEM (A operand in tensor
//     memory, V as an MN-major B operand); O (128 x 256 fp32) lives in columns [256, 512).
//     128-key tiles make every QK^T MMA N = 128: a tcgen05.mma with both operands in shared
//     memory costs about as much to issue at N = 64 as at N = 128 (measured), so the wider tile
//     halves the issue cost per key. The MMA issue order S_0, S_1, PV_0, S_2, PV_1, ... overlaps
//     each QK^T with the softmax of the previous tile. The running max is raised only when a
//     tile exceeds it by more than 2^8 (log2 units), so O is rescaled (a TMEM read-modify-write)
//     rarely; P values stay <= 256.
//
// Synchronisation (all mbarrier waits bounded; a timeout sets the device error word):
//   q_full / q_empty       Q tile of the current item loaded / all its QK^T MMAs done
//   kv_full[s] / kv_empty[s]  ring stage loaded / consumed by its MMA
//   s_full[b]              S buffer b written (tcgen05.commit)
//   p_full[b]              P of buffer b written by all 256 softmax threads
//   pv_done[k % 2]         O += P_k V_k finished (two barriers so no waiter is ever two phases
//                          behind: a commit fires only after every earlier MMA, so when S_j is
//                          complete every PV up to j-2 is too)
// Producers signal each stage from the copy hardware as soon as its cp.async copies land
// (cp.async.mbarrier.arrive.noinc); the MMA thread, after acquiring a stage, orders those
// generic-proxy writes before the tensor core's async-proxy reads with fence.proxy.async.
#include "ptx.cuh"
#include "runtime.h"
#include "tcgen05.cuh"
#include "../../include/roaster_cuda.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cmath>
#include <cstring>
#include <queue>
#include <vector>


namespace rb {
namespace {

constexpr int kD = 256;
constexpr int kBM = 128;                     // query rows per item
constexpr int kBN = 128;                     // keys per tile (S MMAs with N = 128)
constexpr int kStages = 5;
constexpr int kChunkQ = kBM * 128;           // one 64-dim chunk of the Q tile (16 KB)
constexpr int kQBytes = 4 * kChunkQ;         // 64 KB
// A ring stage holds half of a K or V tile (32 KB):
//   K half h: dims [128h, 128h + 128) of all 128 keys, [2 dim chunks][128 keys][128 B]
//   V half h: keys [64h, 64h + 64) with all 256 dims, [4 dim chunks][64 keys][128 B]
// Fills follow the order the MMAs consume them -- K_0, K_1, V_0, K_2, V_1, ..., V_{nt-1} (each
// as two halves) -- so K runs two tiles ahead of the tensor core; a half-stage is released as
// soon as the MMAs reading it complete.
__host__ __device__ constexpr unsigned kfill(int j) { return j == 0 ? 0u : 4u * (unsigned)j - 2u; }
__host__ __device__ constexpr unsigned vfill(int j, int nt) { return j + 1 == nt ? 4u * (unsigned)j + 2u : 4u * (unsigned)j + 4u; }
constexpr int kStageBytes = 32768;
constexpr int kKChunk = kBN * 128;           // 16 KB: one 64-dim chunk of 128 keys
constexpr int kVChunk = 64 * 128;            // 8 KB: one 64-dim chunk of 64 keys
constexpr int kThreads = 320;                 // MMA warp, TMA warp, 8 softmax warps (2-9)
constexpr int kMaxJobs = 64;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescale = 8.0f;

struct PJob {
    const __half *qp;           // prepared queries of this job, [T][16][256] f16
    const void *gate;
    const __half *k_cache, *v_cache;
    float *out;
    long long qg_stride, qg_tok_stride, kbase, T;
    int dtype, pad;
};

struct PParams {
    PJob jobs[kMaxJobs];
    const CUtensorMap *maps;    // per job: prepared Q, K cache, V cache (global memory)
    const unsigned *sched;      // (job << 26) | (head << 22) | query tile, grouped by CTA
    const int *cta_off;         // [grid + 1]
    unsigned *err;
    int njobs;
};

struct Smem {
    unsigned char q[kQBytes];                   // 1024-byte aligned (swizzle atoms)
    unsigned char kv[kStages][kStageBytes];
    unsigned long long q_full, q_empty, kv_full[kStages], kv_empty[kStages];
    unsigned long long s_full[2], p_full[2], pv_done[2], drain;
    float lsum[2][kBM];                         // row-sum halves of the two softmax warps of a row
    uint32_t tmem_base;
    int abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

__device__ __forceinline__ bool aborted(Smem &sm) { return *(volatile int *)&sm.abort != 0; }

// Bounded wait whose outcome is the same for every lane of the warp (the warp then runs
// warp-collective tcgen05 loads/stores together).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity)
{
    const bool ok = mbar_wait(bar, parity);
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void set_abort(const PParams &p, Smem &sm)
{
    atomicOr(p.err, kErrWaitTimeout);
    *(volatile int *)&sm.abort = 1;
}

struct Item {
    int job, head, kvh;
    long long t0, rows, kend;     // first query token of the tile, valid rows, keys needed
    int nt;                       // key tiles
};

__device__ __forceinline__ Item decode_item(const PParams &p, unsigned e)
{
    Item it;
    it.job = (int)(e >> 26);
    it.head = (int)((e >> 22) & 15u);
    it.kvh = it.head >> 3;
    const PJob &J = p.jobs[it.job];
    it.t0 = (long long)(e & 0x3FFFFFu) * kBM;
    it.rows = J.T - it.t0 < kBM ? J.T - it.t0 : kBM;
    it.kend = J.kbase + it.t0 + it.rows;
    it.nt = (int)((it.kend + kBN - 1) / kBN);
    return it;
}

// One box of a 3-D tensor map (in global memory) into shared memory, completion as transaction
// bytes on `bar`. x (the innermost coordinate) is a multiple of 64 f16 elements here.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int x, int y, int z, uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

// 2^x on the special-function unit (flush-to-zero: results below 2^-126 become 0, which only
// drops probabilities that are negligible against the row maximum).
__device__ __forceinline__ float ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 32 consecutive gate values of one row, through the read-only path (no aliasing with `out`).
__device__ __forceinline__ void load_gate32(const void *base, long long idx, int dtype, float (&g)[32])
{
    if (dtype == KERNEL_DTYPE_BF16) {
        const uint4 *src = reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(base) + idx);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint4 u = __ldg(src + i);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                g[8 * i + 2 * k] = __uint_as_float(w[k] << 16);
                g[8 * i + 2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
            }
        }
    } else {
        const float4 *src = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(base) + idx);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 v = __ldg(src + i);
            g[4 * i] = v.x;
            g[4 * i + 1] = v.y;
            g[4 * i + 2] = v.z;
            g[4 * i + 3] = v.w;
        }
    }
}

// ---------------------------------------------------------------------------- prep kernel

struct PrepJob {
    const void *q, *k, *v;
    const float *q_norm, *k_norm;
    __half *qp, *k_cache, *v_cache;
    long long qg_stride, qg_tok_stride, kbase, base, tok0;
    int dtype, pad;
};

struct PrepParams {
    PrepJob jobs[kMaxJobs];
    float inv_freq[32];
    int njobs;
};

// Eight consecutive inputs (dims 8 lane .. 8 lane + 7 of one row) as fp32; 16-byte loads.
__device__ __forceinline__ void load8(const void *base, long long idx, int dtype, float (&x)[8])
{
    if (dtype == KERNEL_DTYPE_BF16) {
        const uint4 u = __ldg(reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(base) + idx));
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            x[2 * k] = __uint_as_float(w[k] << 16);
            x[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
        }
    } else {
        const float4 *src = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(base) + idx);
        const float4 a = __ldg(src), b = __ldg(src + 1);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    }
}

// One CTA per token. The token's 32 RoPE angles (position * inv_freq[j], rotated with one
// sincosf each) are shared by its 18 rotated rows; then warp w handles rows w, w + 8, w + 16 of
// the token's 16 q heads, 2 k heads and 2 v heads, lane l holding dims 8l .. 8l+7.
__global__ void __launch_bounds__(256) prefill_prep_kernel(const __grid_constant__ PrepParams p)
{
    __shared__ float rc[32], rs[32];
    const int gtok = blockIdx.x;
    int lo = 0, hi = p.njobs - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (p.jobs[mid].tok0 <= gtok)
            lo = mid;
        else
            hi = mid - 1;
    }
    const PrepJob &J = p.jobs[lo];
    const long long t = gtok - J.tok0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x < 32) {
        const float pos = (float)(J.base + t);
        float sn, cs;
        sincosf(pos * p.inv_freq[threadIdx.x], &sn, &cs);
        rc[threadIdx.x] = cs;
        rs[threadIdx.x] = sn;
    }
    __syncthreads();
    for (int row = warp; row < 20; row += 8) {
        float x[8];
        const bool isq = row < 16, isk = row >= 16 && row < 18;
        const int h = isq ? row : (isk ? row - 16 : row - 18);
        if (isq)
            load8(J.q, t * J.qg_tok_stride + (long long)h * J.qg_stride + lane * 8, J.dtype, x);
        else
            load8(isk ? J.k : J.v, t * 512 + h * 256 + lane * 8, J.dtype, x);
        if (isq || isk) {
            float ss = 0.f;
#pragma unroll
            for (int e = 0; e < 8; e++)
                ss = fmaf(x[e], x[e], ss);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
                ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float inv = 1.0f / sqrtf(ss / (float)kD + 1e-6f);
            const float4 *w4 = reinterpret_cast<const float4 *>((isq ? J.q_norm : J.k_norm) + lane * 8);
            const float4 wa = __ldg(w4), wb = __ldg(w4 + 1);
            const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
            for (int e = 0; e < 8; e++)
                x[e] = x[e] * inv * w[e];
            // RoPE: dims j and j + 32 (j < 32) live on lanes l and l + 4 (l < 4)
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const float other = __shfl_xor_sync(0xffffffffu, x[e], 4);
                if (lane < 8) {
                    const int j = (lane & 3) * 8 + e;
                    x[e] = lane < 4 ? x[e] * rc[j] - other * rs[j] : x[e] * rc[j] + other * rs[j];
                }
            }
        }
        __half hv[8];
#pragma unroll
        for (int e = 0; e < 8; e++)
            hv[e] = __float2half_rn(x[e]);
        __half *dst;
        if (isq)
            dst = J.qp + (t * 16 + h) * kD + lane * 8;
        else
            dst = (isk ? J.k_cache : J.v_cache) + ((J.kbase + t) * 2 + h) * kD + lane * 8;
        *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(hv);
    }
}

// ---------------------------------------------------------------------------- attention kernel

__global__ void __launch_bounds__(kThreads, 1) prefill_attn_kernel(const __grid_constant__ PParams p)
{
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    Smem &sm = *reinterpret_cast<Smem *>(smem_raw + ((1024u - (raw & 1023u)) & 1023u));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int i0 = p.cta_off[blockIdx.x], i1 = p.cta_off[blockIdx.x + 1];

    if (tid == 0) {
        mbar_init(smem_addr(&sm.q_full), 1);
        mbar_init(smem_addr(&sm.q_empty), 1);
        for (int s = 0; s < kStages; s++) {
            mbar_init(smem_addr(&sm.kv_full[s]), 1);
            mbar_init(smem_addr(&sm.kv_empty[s]), 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(smem_addr(&sm.s_full[b]), 1);
            mbar_init(smem_addr(&sm.p_full[b]), 256);
            mbar_init(smem_addr(&sm.pv_done[b]), 1);
        }
        mbar_init(smem_addr(&sm.drain), 1);
        sm.abort = 0;
        mbar_init_fence();
    }
    if (warp == 0) {
        tc::tmem_alloc(smem_addr(&sm.tmem_base), kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tbase = sm.tmem_base;
    const uint32_t sq = smem_addr(sm.q);

    if (warp == 0) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idS = tc::idesc_f16(kBM, kBN, 0, 0);
            const uint64_t qd = tc::smem_desc(sq, 16, 1024);
            const uint32_t idO = tc::idesc_f16(kBM, kD, 0, 1);
            unsigned fill = 0, g = 0, nitem = 0;
            bool ok = true;
            auto wait = [&](unsigned long long &bar, unsigned parity) {
                if (ok && !mbar_wait(smem_addr(&bar), parity)) {
                    set_abort(p, sm);
                    ok = false;
                }
                return ok;
            };
            auto acquire = [&](unsigned f) {                 // ring fill f loaded
                if (!wait(sm.kv_full[f % kStages], (f / kStages) & 1))   // TMA writes: async proxy
                    return 0u;
                return smem_addr(sm.kv[f % kStages]);
            };
            // O += P_g V_g; V_g occupies fills fv (keys 0-63) and fv + 1 (keys 64-127)
            auto pv = [&](unsigned gg, unsigned fv, bool first) {
                if (!wait(sm.p_full[gg & 1], (gg >> 1) & 1))
                    return;
                const uint32_t v0 = acquire(fv), v1 = ok ? acquire(fv + 1) : 0u;
                if (!ok)
                    return;
                tc::fence_after_sync();
                const uint64_t vd0 = tc::smem_desc(v0, kVChunk, 1024), vd1 = tc::smem_desc(v1, kVChunk, 1024);
#pragma unroll
                for (int kk = 0; kk < kBN / 16; kk++) {
                    // P for keys 0-63 sits in columns [0, 32) of the tile, keys 64-127 in [64, 96)
                    tc::mma_ts_f16(tbase + kColO, tbase + (gg & 1) * kBN + (kk < 4 ? kk * 8 : 32 + kk * 8),
                                   tc::desc_adv(kk < 4 ? vd0 : vd1, (kk & 3) * 2048), idO, (first && kk == 0) ? 0u : 1u);
                    if (kk == 3)
                        tc::commit(smem_addr(&sm.kv_empty[fv % kStages]));
                }
                tc::commit(smem_addr(&sm.pv_done[gg & 1]));
                tc::commit(smem_addr(&sm.kv_empty[(fv + 1) % kStages]));
            };
            for (int idx = i0; idx < i1 && ok && !aborted(sm); idx++, nitem++) {
                const Item it = decode_item(p, p.sched[idx]);
                if (!wait(sm.q_full, nitem & 1))
                    break;
                tc::fence_after_sync();
                const unsigned fbase = fill;
                for (int j = 0; j < it.nt && ok; j++) {
                    const unsigned fk = fbase + kfill(j);
                    const uint32_t k0 = acquire(fk), k1 = ok ? acquire(fk + 1) : 0u;
                    if (!ok)
                        break;
                    tc::fence_after_sync();
                    const unsigned gj = g + j;
                    const uint64_t kd0 = tc::smem_desc(k0, 16, 1024), kd1 = tc::smem_desc(k1, 16, 1024);
#pragma unroll
                    for (int kk = 0; kk < kD / 16; kk++) {
                        tc::mma_ss_f16(tbase + (gj & 1) * kBN, tc::desc_adv(qd, (kk >> 2) * kChunkQ + (kk & 3) * 32),
                                       tc::desc_adv(kk < 8 ? kd0 : kd1, ((kk >> 2) & 1) * kKChunk + (kk & 3) * 32), idS,
                                       kk > 0 ? 1u : 0u);
                        if (kk == 7)
                            tc::commit(smem_addr(&sm.kv_empty[fk % kStages]));
                    }
                    tc::commit(smem_addr(&sm.s_full[gj & 1]));
                    tc::commit(smem_addr(&sm.kv_empty[(fk + 1) % kStages]));
                    if (j == it.nt - 1)
                        tc::commit(smem_addr(&sm.q_empty));
                    if (j >= 1)
                        pv(gj - 1, fbase + vfill(j - 1, it.nt), j - 1 == 0);
                }
                if (ok)
                    pv(g + it.nt - 1, fbase + vfill(it.nt - 1, it.nt), it.nt == 1);
                g += it.nt;
                fill += 4 * it.nt;
            }
            // every MMA issued must finish before tensor memory is released
            tc::commit(smem_addr(&sm.drain));
            mbar_wait(smem_addr(&sm.drain), 0);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- producer (TMA)
        // One thread issues every tile copy: the Q tile as four 64-dim boxes of 128 rows, each
        // K half as two 64-dim x 128-key boxes, each V half as four 64-dim x 64-key boxes. The
        // tensor maps (one per job and tensor, in global memory) clip at the valid extent, so
        // rows past the end of a prompt arrive as zeros; the hardware writes the 128-byte
        // swizzle the MMAs read.
        if (lane == 0) {
            unsigned fill = 0, nitem = 0;
            bool ok = true;
            for (int idx = i0; idx < i1 && ok && !aborted(sm); idx++, nitem++) {
                const Item it = decode_item(p, p.sched[idx]);
                const CUtensorMap *mq = p.maps + 3 * it.job, *mk = mq + 1, *mv = mq + 2;
                if (nitem > 0 && !mbar_wait(smem_addr(&sm.q_empty), (nitem - 1) & 1)) {
                    set_abort(p, sm);
                    ok = false;
                    break;
                }
                const uint32_t qb = smem_addr(&sm.q_full);
                mbar_arrive_expect_tx(qb, kQBytes);
#pragma unroll
                for (int c = 0; c < 4; c++)
                    tma_load_3d(sq + c * kChunkQ, mq, 64 * c, it.head, (int)it.t0, qb);
                for (int step = 0; step <= it.nt && ok; step++) {
                    for (int part = 0; part < 4; part++) {
                        // step s: K_s (parts 0, 1) if s < nt, then V_{s-1} (parts 2, 3) if s >= 1
                        const int j = part < 2 ? step : step - 1;
                        if ((part < 2 && step == it.nt) || (part >= 2 && step == 0))
                            continue;
                        const int s = fill % kStages;
                        const unsigned f = fill / kStages;
                        if (f > 0 && !mbar_wait(smem_addr(&sm.kv_empty[s]), (f - 1) & 1)) {
                            set_abort(p, sm);
                            ok = false;
                            break;
                        }
                        const uint32_t st = smem_addr(sm.kv[s]), fb = smem_addr(&sm.kv_full[s]);
                        const int key0 = j * kBN;
                        mbar_arrive_expect_tx(fb, kStageBytes);
                        if (part < 2) {
                            // K half: dims [128 part, +128) of the tile's 128 keys
                            tma_load_3d(st, mk, 128 * part, it.kvh, key0, fb);
                            tma_load_3d(st + kKChunk, mk, 128 * part + 64, it.kvh, key0, fb);
                        } else {
                            // V half: keys [64 (part - 2), +64), all 256 dims
#pragma unroll
                            for (int c = 0; c < 4; c++)
                                tma_load_3d(st + c * kVChunk, mv, 64 * c, it.kvh, key0 + 64 * (part - 2), fb);
                        }
                        fill++;
                    }
                }
            }
            // nothing of ours may still be landing when the CTA retires
            for (unsigned f = fill > (unsigned)kStages ? fill - kStages : 0u; f < fill; f++)
                mbar_wait(smem_addr(&sm.kv_full[f % kStages]), (f / kStages) & 1);
        }
    } else {
        // ---------------------------------------------------------------- softmax + epilogue
        // Two warps per query row: warps 2-5 take score columns 0-63 (and output dims 0-127),
        // warps 6-9 columns 64-127 (dims 128-255); warp w owns TMEM lanes 32 (w % 4) ... Both read the whole row for its max, so the
        // pair agrees on it without exchanging values (a pair barrier then keeps P writes behind
        // both reads); the row sums meet in shared memory once per query tile.
        const int half = warp >= 6 ? 1 : 0;
        const int row = (warp & 3) * 32 + lane;            // query row = TMEM lane
        const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
        const int c0 = 64 * half;
        const float sc = kLog2e / 16.0f;
        unsigned g = 0;
        bool ok = true;
        for (int idx = i0; idx < i1 && ok && !aborted(sm); idx++) {
            const Item it = decode_item(p, p.sched[idx]);
            const PJob &J = p.jobs[it.job];
            const bool qvalid = row < it.rows;
            const long long tq = it.t0 + row;
            const long long qlimit = qvalid ? J.kbase + tq : -1;  // last key this row may see
            const long long it_qmin = J.kbase + it.t0;            // smallest last key of the tile
            float m_run = -INFINITY, l = 0.f;
            for (int j = 0; j < it.nt; j++) {
                const unsigned gj = g + j;
                const uint32_t sb = tbase + lane_base + (gj & 1) * kBN;
                if (!warp_wait(smem_addr(&sm.s_full[gj & 1]), (gj >> 1) & 1)) {
                    if (lane == 0)
                        set_abort(p, sm);
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                // causal mask only where the tile reaches past some row's last key
                const long long key0 = (long long)j * kBN;
                const bool masked = key0 + kBN - 1 > it_qmin;
                const int lim = masked ? (int)(qlimit - key0 < -1 ? -1 : qlimit - key0) : kBN;  // keys <= lim visible
                // pass 1: max over the whole row (tree reduction, 32 columns at a time)
                float mt = -INFINITY;
#pragma unroll 1
                for (int c = 0; c < kBN; c += 32) {
                    float x[32];
                    tc::tmem_ld32(sb + c, x);
                    tc::tmem_wait_ld();
                    if (masked) {
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            x[i] = c + i <= lim ? x[i] : -INFINITY;
                    }
#pragma unroll
                    for (int w = 16; w >= 1; w >>= 1)
#pragma unroll
                        for (int i = 0; i < w; i++)
                            x[i] = fmaxf(x[i], x[i + w]);
                    mt = fmaxf(mt, x[0]);
                }
                mt *= sc;                                            // row max in log2 units
                // the partner warp reads this warp's columns in its pass 1; P overwrites them next
                named_bar_sync(1 + (warp & 3), 64);
                float m_new = m_run;
                if (mt > m_run + kRescale || (m_run == -INFINITY && mt != -INFINITY))
                    m_new = mt;
                const float m_use = m_new == -INFINITY ? 0.f : m_new;
                const float alpha = m_run == -INFINITY ? 0.f : ex2(m_run - m_use);
                // pass 2 over this warp's 64 columns: P = 2^(s sc - m) as f16, packed two per
                // column into [c0, c0 + 32) (chunk c's P lands at c0 + (c - c0)/2, columns this
                // warp has already read)
                float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll 1
                for (int c = c0; c < c0 + 64; c += 32) {
                    float x[32];
                    tc::tmem_ld32(sb + c, x);
                    tc::tmem_wait_ld();
                    if (masked) {
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            x[i] = c + i <= lim ? x[i] : -INFINITY;
                    }
                    uint32_t w[16];
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        const float e0 = ex2(fmaf(x[i], sc, -m_use)), e1 = ex2(fmaf(x[i + 1], sc, -m_use));
                        const float e2 = ex2(fmaf(x[i + 2], sc, -m_use)), e3 = ex2(fmaf(x[i + 3], sc, -m_use));
                        s0 += e0;
                        s1 += e1;
                        s2 += e2;
                        s3 += e3;
                        w[i >> 1] = pack_f16x2(e0, e1);
                        w[(i >> 1) + 1] = pack_f16x2(e2, e3);
                    }
                    tc::tmem_st16(sb + c0 + ((c - c0) >> 1), w);
                }
                const float sum = (s0 + s1) + (s2 + s3);
                l = l * alpha + sum;
                tc::tmem_wait_st();
                const bool need = m_run != -INFINITY && m_new != m_run;
                if (__any_sync(0xffffffffu, need)) {
                    // O holds sums relative to m_run: rescale this warp's half once PV_{j-1} landed
                    const unsigned pj = gj - 1;
                    if (!warp_wait(smem_addr(&sm.pv_done[pj & 1]), (pj >> 1) & 1)) {
                        if (lane == 0)
                            set_abort(p, sm);
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const float f = need ? alpha : 1.0f;
#pragma unroll 1
                    for (int c = 128 * half; c < 128 * half + 128; c += 32) {
                        float o[32];
                        tc::tmem_ld32(tbase + lane_base + kColO + c, o);
                        tc::tmem_wait_ld();
                        uint32_t ow[32];
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            ow[i] = __float_as_uint(o[i] * f);
                        tc::tmem_st32(tbase + lane_base + kColO + c, ow);
                    }
                    tc::tmem_wait_st();
                }
                m_run = m_new;
                tc::fence_before_sync();
                mbar_arrive(smem_addr(&sm.p_full[gj & 1]));
            }
            if (!ok)
                break;
            // epilogue: O / l * sigmoid(gate) for this warp's 128 output dims
            const unsigned pl = g + it.nt - 1;
            if (!warp_wait(smem_addr(&sm.pv_done[pl & 1]), (pl >> 1) & 1)) {
                if (lane == 0)
                    set_abort(p, sm);
                ok = false;
                break;
            }
            tc::fence_after_sync();
            sm.lsum[half][row] = l;
            named_bar_sync(1 + (warp & 3), 64);
            const float lt = sm.lsum[0][row] + sm.lsum[1][row];
            const float inv_l = lt > 0.f ? 1.0f / lt : 0.f;
            const int d0 = 128 * half;
            const long long gbase = (qvalid ? tq : it.t0) * J.qg_tok_stride + (long long)it.head * J.qg_stride + d0;
            float *orow = J.out + (tq * 16 + it.head) * kD + d0;
            float gv[32], gn[32];
            load_gate32(J.gate, gbase, J.dtype, gn);
#pragma unroll 1
            for (int c = 0; c < 128; c += 32) {
#pragma unroll
                for (int i = 0; i < 32; i++)
                    gv[i] = gn[i];
                if (c + 32 < 128)
                    load_gate32(J.gate, gbase + c + 32, J.dtype, gn);     // next chunk in flight
                float o[32];
                tc::tmem_ld32(tbase + lane_base + kColO + d0 + c, o);
                tc::tmem_wait_ld();
                if (qvalid) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        float4 r;
                        r.x = o[i] * inv_l / (1.0f + __expf(-gv[i]));
                        r.y = o[i + 1] * inv_l / (1.0f + __expf(-gv[i + 1]));
                        r.z = o[i + 2] * inv_l / (1.0f + __expf(-gv[i + 2]));
                        r.w = o[i + 3] * inv_l / (1.0f + __expf(-gv[i + 3]));
                        *reinterpret_cast<float4 *>(orow + c + i) = r;
                    }
                }
            }
            // the pair's partner may still be reading lsum for this tile; the next write is a
            // full query tile later, after its named barrier
            tc::fence_before_sync();
            g += it.nt;
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0)
        tc::tmem_dealloc(tbase, kTmemCols);
}

bool g_attn_attr = false;

int validate(const KernelAttnPrefillJob &j, int i)
{
    if (!j.q || !j.gate || !j.k || !j.v || !j.q_norm || !j.k_norm || !j.k_cache || !j.v_cache || !j.out)
        return fail("attn prefill: job %d has a null pointer", i);
    if (j.T == 0 || j.T > (1ull << 22) * kBM)
        return fail("attn prefill: job %d T=%zu out of range", i, j.T);
    if (j.kbase + j.T > j.capacity)
        return fail("attn prefill: job %d window overflow (kbase %zu + T %zu > capacity %zu)", i, j.kbase,
                    j.T, j.capacity);
    if (j.dtype != KERNEL_DTYPE_F32 && j.dtype != KERNEL_DTYPE_BF16)
        return fail("attn prefill: job %d bad dtype %d", i, j.dtype);
    if (!aligned16(j.k_cache) || !aligned16(j.v_cache) || !aligned16(j.out))
        return fail("attn prefill: job %d cache/out not 16-byte aligned", i);
    if (j.qg_stride < 256 || j.qg_tok_stride < 16 * j.qg_stride / 2 || (j.qg_stride & 7) ||
        (j.qg_tok_stride & 7))
        return fail("attn prefill: job %d bad q/gate strides (>= 256, multiples of 8)", i);
    if (!aligned16(j.gate) || !aligned16(j.q) || !aligned16(j.k) || !aligned16(j.v) ||
        !aligned16(j.q_norm) || !aligned16(j.k_norm))
        return fail("attn prefill: job %d q/gate/k/v/norm weights not 16-byte aligned", i);
    return 0;
}

int prefill_launch(const KernelAttnPrefillJob *jobs, int n)
{
    Runtime &R = rt();
    long long total_t = 0;
    for (int i = 0; i < n; i++) {
        if (validate(jobs[i], i) != 0)
            return -1;
        total_t += (long long)jobs[i].T;
    }
    // items: (job, head, query tile), longest first onto the least-loaded CTA
    std::vector<std::pair<long long, unsigned>> items;
    for (int i = 0; i < n; i++) {
        const long long T = (long long)jobs[i].T, kb = (long long)jobs[i].kbase;
        const long long nq = (T + kBM - 1) / kBM;
        for (long long qt = 0; qt < nq; qt++) {
            const long long rows = std::min<long long>(kBM, T - qt * kBM);
            const long long nt = (kb + qt * kBM + rows + kBN - 1) / kBN;
            for (int h = 0; h < 16; h++)
                items.emplace_back(nt + 2, ((unsigned)i << 26) | ((unsigned)h << 22) | (unsigned)qt);
        }
    }
    // prompt by prompt, each prompt's items longest first: the CTAs then work on one or two
    // prompts' K/V at a time, which stays in L2, instead of every prompt's at once
    std::stable_sort(items.begin(), items.end(),
                     [](const std::pair<long long, unsigned> &a, const std::pair<long long, unsigned> &b) {
                         const unsigned ja = a.second >> 26, jb = b.second >> 26;
                         return ja != jb ? ja < jb : a.first > b.first;
                     });
    const int grid = (int)std::min<size_t>(items.size(), (size_t)R.num_sms);
    std::vector<std::vector<unsigned>> per(grid);
    {
        std::priority_queue<std::pair<long long, int>, std::vector<std::pair<long long, int>>,
                            std::greater<std::pair<long long, int>>> heap;
        for (int c = 0; c < grid; c++)
            heap.emplace(0ll, c);
        for (const auto &it : items) {
            auto top = heap.top();
            heap.pop();
            per[top.second].push_back(it.second);
            heap.emplace(top.first + it.first, top.second);
        }
    }
    std::vector<unsigned> sched;
    std::vector<int> off(grid + 1, 0);
    sched.reserve(items.size());
    for (int c = 0; c < grid; c++) {
        off[c] = (int)sched.size();
        sched.insert(sched.end(), per[c].begin(), per[c].end());
    }
    off[grid] = (int)sched.size();
    // scratch: prepared queries (f16), then the schedule
    const size_t qp_bytes = (size_t)total_t * 16 * kD * sizeof(__half);
    const size_t sched_off = (qp_bytes + 255) / 256 * 256;
    const size_t off_off = sched_off + (sched.size() * 4 + 255) / 256 * 256;
    const size_t maps_off = (off_off + off.size() * 4 + 255) / 256 * 256;
    unsigned char *ws = static_cast<unsigned char *>(scratch(maps_off + (size_t)n * 3 * sizeof(CUtensorMap)));
    if (!ws)
        return -1;
    // tensor maps: per job the prepared queries [T][16][256], and the K and V windows
    // [kbase + T][2][256] (f16), each clipped at its valid extent
    std::vector<CUtensorMap> maps((size_t)n * 3);
    {
        long long t0 = 0;
        for (int i = 0; i < n; i++) {
            const KernelAttnPrefillJob &s = jobs[i];
            const uint64_t qdims[3] = {256, 16, (uint64_t)s.T}, qstr[2] = {512, 8192};
            const uint64_t kdims[3] = {256, 2, (uint64_t)(s.kbase + s.T)}, kstr[2] = {512, 1024};
            const uint32_t qbox[3] = {64, 1, kBM}, kbox[3] = {64, 1, kBN}, vbox[3] = {64, 1, 64};
            const __half *qpi = reinterpret_cast<const __half *>(ws) + t0 * 16 * kD;
            if (encode_tmap_f16_3d(&maps[3 * i], qpi, qdims, qstr, qbox) != 0 ||
                encode_tmap_f16_3d(&maps[3 * i + 1], s.k_cache, kdims, kstr, kbox) != 0 ||
                encode_tmap_f16_3d(&maps[3 * i + 2], s.v_cache, kdims, kstr, vbox) != 0)
                return -1;
            t0 += (long long)s.T;
        }
    }
    cudaStream_t st = R.stream;
    if (check(cudaMemcpyAsync(ws + sched_off, sched.data(), sched.size() * 4, cudaMemcpyHostToDevice, st),
              "prefill schedule") != 0 ||
        check(cudaMemcpyAsync(ws + off_off, off.data(), off.size() * 4, cudaMemcpyHostToDevice, st),
              "prefill schedule offsets") != 0 ||
        check(cudaMemcpyAsync(ws + maps_off, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice,
                              st), "prefill tensor maps") != 0)
        return -1;

    PrepParams pp;
    memset(static_cast<void *>(&pp), 0, sizeof(pp));
    PParams ap;
    memset(static_cast<void *>(&ap), 0, sizeof(ap));
    long long tok0 = 0;
    __half *qp = reinterpret_cast<__half *>(ws);
    for (int i = 0; i < n; i++) {
        const KernelAttnPrefillJob &s = jobs[i];
        PrepJob &d = pp.jobs[i];
        d.q = s.q;
        d.k = s.k;
        d.v = s.v;
        d.q_norm = s.q_norm;
        d.k_norm = s.k_norm;
        d.qp = qp + tok0 * 16 * kD;
        d.k_cache = reinterpret_cast<__half *>(s.k_cache);
        d.v_cache = reinterpret_cast<__half *>(s.v_cache);
        d.qg_stride = (long long)s.qg_stride;
        d.qg_tok_stride = (long long)s.qg_tok_stride;
        d.kbase = (long long)s.kbase;
        d.base = (long long)s.base;
        d.tok0 = tok0;
        d.dtype = s.dtype;
        PJob &a = ap.jobs[i];
        a.qp = d.qp;
        a.gate = s.gate;
        a.k_cache = d.k_cache;
        a.v_cache = d.v_cache;
        a.out = s.out;
        a.qg_stride = d.qg_stride;
        a.qg_tok_stride = d.qg_tok_stride;
        a.kbase = d.kbase;
        a.T = (long long)s.T;
        a.dtype = s.dtype;
        tok0 += (long long)s.T;
    }
    memcpy(pp.inv_freq, R.inv_freq, sizeof(pp.inv_freq));
    pp.njobs = n;
    prefill_prep_kernel<<<(unsigned)total_t, 256, 0, st>>>(pp);
    if (launched("prefill_prep_kernel") != 0)
        return -1;
    ap.maps = reinterpret_cast<const CUtensorMap *>(ws + maps_off);
    ap.sched = reinterpret_cast<const unsigned *>(ws + sched_off);
    ap.cta_off = reinterpret_cast<const int *>(ws + off_off);
    ap.err = R.err_word;
    ap.njobs = n;
    if (!g_attn_attr) {
        if (check(cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBytes), "prefill smem attribute") != 0)
            return -1;
        g_attn_attr = true;
    }
    prefill_attn_kernel<<<grid, kThreads, kSmemBytes, st>>>(ap);
    return launched("prefill_attn_kernel");
}

}  // namespace

int attn_prefill_batch(const KernelAttnPrefillJob *jobs, int n)
{
    if (n < 0 || (n > 0 && !jobs))
        return fail("attn prefill: bad job array");
    for (int i = 0; i < n; i += kMaxJobs) {
        if (prefill_launch(jobs + i, std::min(kMaxJobs, n - i)) != 0)
            return -1;
    }
    return 0;
}

}  // namespace rb

using namespace rb;

extern "C" int kernel_attn_prefill_batch(const KernelAttnPrefillJob *jobs, int n)
{
    if (ensure() != 0)
        return -1;
    return attn_prefill_batch(jobs, n);
}

extern "C" int kernel_attn_prefill(const float *q_gate, const float *k, const float *v, const float *q_norm,
                                   const float *k_norm, uint16_t *k_cache, uint16_t *v_cache, size_t capacity,
                                   size_t kbase, size_t base, size_t T, float *out)
{
    if (ensure() != 0)
        return -1;
    if (!q_gate || !k || !v || !q_norm || !k_norm || !out || T == 0)
        return fail("kernel_attn_prefill: bad arguments");
    // device staging: q_gate [T][8192], k, v [T][512], norms [2][256]; out [T][4096]
    const size_t nqg = T * 8192, nkv = T * 512, nout = T * 4096;
    const size_t in_f = nqg + 2 * nkv + 512;
    float *d = static_cast<float *>(dstage((in_f + nout) * sizeof(float)));
    if (!d)
        return -1;
    cudaStream_t st = rt().stream;
    if (check(cudaMemcpyAsync(d, q_gate, nqg * 4, cudaMemcpyHostToDevice, st), "stage q") != 0 ||
        check(cudaMemcpyAsync(d + nqg, k, nkv * 4, cudaMemcpyHostToDevice, st), "stage k") != 0 ||
        check(cudaMemcpyAsync(d + nqg + nkv, v, nkv * 4, cudaMemcpyHostToDevice, st), "stage v") != 0 ||
        check(cudaMemcpyAsync(d + nqg + 2 * nkv, q_norm, 256 * 4, cudaMemcpyHostToDevice, st), "stage qn") != 0 ||
        check(cudaMemcpyAsync(d + nqg + 2 * nkv + 256, k_norm, 256 * 4, cudaMemcpyHostToDevice, st), "stage kn") != 0)
        return -1;
    KernelAttnPrefillJob j;
    memset(&j, 0, sizeof(j));
    j.q = d;
    j.gate = d + 256;
    j.qg_stride = 512;
    j.qg_tok_stride = 8192;
    j.k = d + nqg;
    j.v = d + nqg + nkv;
    j.q_norm = d + nqg + 2 * nkv;
    j.k_norm = d + nqg + 2 * nkv + 256;
    j.k_cache = k_cache;
    j.v_cache = v_cache;
    j.capacity = capacity;
    j.kbase = kbase;
    j.base = base;
    j.T = T;
    j.out = d + in_f;
    j.dtype = KERNEL_DTYPE_F32;
    if (attn_prefill_batch(&j, 1) != 0)
        return -1;
    if (check(cudaMemcpyAsync(out, d + in_f, nout * 4, cudaMemcpyDeviceToHost, st), "stage out") != 0)
        return -1;
    return kernel_cuda_synchronize();
}

