// Gated GQA attention, decode: split-KV, bandwidth-bound, one launch per step for any number
// of slots.
//
// Replaces reference src/model.c:801-861 (full_attention without its projections): per query
// head h (kv head h/8) RMSNorm(q) * qnorm, RMSNorm(k) * knorm, partial NeoX RoPE on dims 0..63
// (theta 1e7), K/V append at the window index `length`, softmax(q.k/16) over the window plus the
// new token, times V, times sigmoid(gate).
//
// Work decomposition. A work item is (slot, kv head, split): a run of consecutive cached
// positions of one kv head; each slot's window is cut into equal splits of about
// total/(SMs x items_per_sm) positions. The host assigns items to persistent CTAs (one per SM)
// longest-first onto the least-loaded CTA and passes each CTA its item list.
// In each CTA
//   * warps 4-7 (producers) stream 32-position stages of K and V into a 5-stage shared-memory
//     ring with 16-byte cp.async copies: one warp instruction moves one 512-byte row (one kv
//     head of one position), placed in a [4 chunks][32 pos][128 B] tile with the 16-byte units of
//     row p XOR-swizzled by (p & 7), so the warp matrix loads below are bank-conflict free.
//     Completion is tracked per stage on an mbarrier (cp.async.mbarrier.arrive). Rows past the
//     window end are never read. The producers run ahead across item boundaries, so the stream
//     stays busy while the consumers finish an item. (Per-row bulk copies are request-rate
//     bound on B200: 512-byte requests top out near 2.4 TB/s, while 16-byte cp.async from four
//     warps streams 512-byte rows at a 1 KB pitch -- this cache's layout -- at about 6.7 TB/s.)
//   * warps 0-3 (consumers) take every 4th stage. The 8 query heads of the GQA group share each
//     tile: S^T[16 pos x 8 heads] = K[16 x 256] Q^T with f16 mma.sync (fp32 accumulate; K is the
//     A operand via ldmatrix, Q^T the B operand held in registers), an online softmax across the
//     stage's 32 positions with warp shuffles (exp2 domain), then O^T[256 x 8] += V^T P^T with
//     V^T loaded by ldmatrix.trans and P^T made by transposing the probability fragment in
//     registers (movmatrix). The 16-position x 8-head tile is exactly one m16n8k16 shape, so no
//     MMA lane is padding.
//   * at the end of an item the 4 warps' (m, l, O) are merged and written as one partial record;
//     the last item of a (slot, kv head) to finish (an atomic counter) merges all of them plus
//     the new token's own partial (scored at fp32 by the split-0 item, which also appends the
//     token's K/V to the f16 cache), applies the gate and writes the output.
//
// Every mbarrier wait is bounded; a timeout sets the device error word instead of hanging.
#include "ptx.cuh"
#include "runtime.h"
#include "../../include/roaster_cuda.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <utility>
#include <vector>

namespace rb {
namespace {

constexpr int kHD = 256;                          // head dim
constexpr int kTile = 32;                         // positions per stage
constexpr int kStages = 5;
constexpr int kCons = 4;                          // consumer warps
constexpr int kProd = 4;                          // producer warps
constexpr int kThreads = (kCons + kProd) * 32;
constexpr int kChunkBytes = kTile * 128;          // one 64-dim chunk of kTile positions (4 KB)
constexpr int kHalfBytes = 4 * kChunkBytes;       // K (or V) of one stage: [4 chunks][kTile][128 B]
constexpr int kStageBytes = 2 * kHalfBytes;       // K then V
constexpr int kMaxJobs = 64;
constexpr int kPF = KERNEL_ATTN_PARTIAL_FLOATS;   // m[8] l[8] o[8][256]
constexpr int kMaxSplits = 256;
constexpr int kMaxItems = 2048;                   // per launch (sched entries)
constexpr int kMaxCtas = 160;
constexpr int kOStride = 260;                     // padded head stride of the merge buffer
constexpr float kLog2e = 1.4426950408889634f;

struct DJob {
    const float *q, *gate;
    const float *k_new, *v_new, *q_norm, *k_norm;
    __half *k_cache, *v_cache;
    float *out;
    float *pdst;        // push mode: this job's merged records [2][kPF] (any GPU's memory), else null
    unsigned *ptag;     // push mode: the 2 tag words set to `epoch` once the records are visible
    long long qg_stride, length, position, chunk;
    int item_base, nsplit, append, pad;
};

struct DParams {
    DJob jobs[kMaxJobs];
    unsigned short sched[kMaxItems];    // (job << 9) | (split << 1) | kv head, grouped by CTA
    unsigned short cta_off[kMaxCtas + 1];
    float inv_freq[32];
    float *part;        // [nitems][kPF]
    float *newpart;     // [njobs][2][kPF]
    float *pout;        // partial mode: [njobs][2][kPF], else null
    unsigned *err;
    int njobs, nitems;
    unsigned epoch;     // push mode: tag value of this step
};

struct Smem {
    unsigned char stage[kStages][kStageBytes];   // [K|V][4 chunks][32 pos][128 B], swizzled
    float qf[2][8][kHD];                  // prepped q (fp32), double-buffered by item parity
    float kf[kHD];                        // prepped new k
    union {
        float ow[kCons][8][kOStride];     // per-warp O (merge of the 4 warps)
    } u;
    float mw[kCons][8], lw[kCons][8];
    float red[8];
    alignas(8) unsigned long long full[kStages], empty[kStages];
    alignas(8) unsigned long long qready[2], qfree[2];   // qf hand-off: producers -> consumers
    int abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 128;   // + alignment slack
static_assert(kSmemBytes <= 232448, "decode kernel shared memory exceeds a CTA's");

__device__ __forceinline__ void item_decode(const DParams &p, int idx, int &j, int &kvh, int &split, int &item)
{
    const unsigned e = p.sched[idx];
    j = (int)(e >> 9);
    split = (int)((e >> 1) & 255u);
    kvh = (int)(e & 1u);
    item = p.jobs[j].item_base + 2 * split + kvh;
}

__device__ __forceinline__ void item_range(const DJob &J, int split, long long &t0, long long &t1)
{
    t0 = (long long)split * J.chunk;
    t1 = t0 + J.chunk < J.length ? t0 + J.chunk : J.length;
    if (t1 < t0)
        t1 = t0;
}

__device__ __forceinline__ void set_error(const DParams &p, unsigned bits, Smem &sm)
{
    atomicOr(p.err, bits);
    *reinterpret_cast<volatile int *>(&sm.abort) = 1;
}

__device__ __forceinline__ bool aborted(Smem &sm)
{
    return *reinterpret_cast<volatile int *>(&sm.abort) != 0;
}

// RMSNorm * w then RoPE (dims 0..63) of query heads 2*pw and 2*pw + 1 of kv head `kvh` into qf,
// by one warp with shuffles only: lane l holds elements l + 32 i of a head, so the RoPE pair
// (d, d + 32) of d = lane sits in one lane. The four producer warps together prepare the 8 heads.
// `after_loads` runs once every load is issued (before any of them is used).
template <typename AfterLoads>
__device__ void prep_q_warp(const DParams &p, const DJob &J, int kvh, float (*qf)[kHD], int pw, int lane,
                            AfterLoads after_loads)
{
    // every load first (both heads' rows and the norm weights: one memory round trip)
    float x[2][8], w[8];
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
        const float *src = J.q + (long long)(kvh * 8 + 2 * pw + hh) * J.qg_stride;
#pragma unroll
        for (int i = 0; i < 8; i++)
            x[hh][i] = __ldg(src + lane + 32 * i);
    }
#pragma unroll
    for (int i = 0; i < 8; i++)
        w[i] = __ldg(J.q_norm + lane + 32 * i);
    after_loads();
    float sn, cs;
    sincosf((float)J.position * p.inv_freq[lane], &sn, &cs);
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
        const int h = 2 * pw + hh;
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++)
            ss = fmaf(x[hh][i], x[hh][i], ss);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = 1.0f / sqrtf(ss / (float)kHD + 1e-6f);
        float y[8];
#pragma unroll
        for (int i = 0; i < 8; i++)
            y[i] = x[hh][i] * inv * w[i];
        const float a = y[0], b = y[1];
        y[0] = a * cs - b * sn;
        y[1] = b * cs + a * sn;
#pragma unroll
        for (int i = 0; i < 8; i++)
            qf[h][lane + 32 * i] = y[i];
    }
}

// New token of (job, kvh): normalise + rotate k, append K/V (f16) at index `length`, and write
// its fp32 softmax partial (m = q.k/16 in log2 units, l = 1, o = v).
__device__ void new_token(const DParams &p, const DJob &J, int jidx, int kvh, const float (*qf)[kHD], Smem &sm,
                          int t)
{
    const float *kn = J.k_new + kvh * kHD;
    const float x0 = __ldg(kn + t), x1 = __ldg(kn + t + 128);
    float ss = x0 * x0 + x1 * x1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((t & 31) == 0)
        sm.red[t >> 5] = ss;
    named_bar_sync(1, 128);
    ss = sm.red[0] + sm.red[1] + sm.red[2] + sm.red[3];
    const float inv = 1.0f / sqrtf(ss / (float)kHD + 1e-6f);
    sm.kf[t] = x0 * inv * __ldg(J.k_norm + t);
    sm.kf[t + 128] = x1 * inv * __ldg(J.k_norm + t + 128);
    named_bar_sync(1, 128);
    if (t < 32) {
        float sn, cs;
        sincosf((float)J.position * p.inv_freq[t], &sn, &cs);
        const float a = sm.kf[t], b = sm.kf[t + 32];
        sm.kf[t] = a * cs - b * sn;
        sm.kf[t + 32] = b * cs + a * sn;
    }
    named_bar_sync(1, 128);
    // append (cached K is normed + rotated, V raw; model.c:815-819)
    const long long row = (J.length * 2 + kvh) * kHD;
    const float *vn = J.v_new + kvh * kHD;
    J.k_cache[row + t] = __float2half_rn(sm.kf[t]);
    J.k_cache[row + t + 128] = __float2half_rn(sm.kf[t + 128]);
    J.v_cache[row + t] = __float2half_rn(__ldg(vn + t));
    J.v_cache[row + t + 128] = __float2half_rn(__ldg(vn + t + 128));
    // scores of the 8 heads against the new key, fp32
    const int h = t >> 4, g = t & 15;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 16; i++)
        s = fmaf(qf[h][g + 16 * i], sm.kf[g + 16 * i], s);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1)
        s += __shfl_xor_sync(0xffffffffu, s, o);
    float *rec = p.newpart + ((long long)jidx * 2 + kvh) * kPF;
    if (g == 0) {
        rec[h] = s * (kLog2e / 16.0f);
        rec[8 + h] = 1.0f;
    }
    for (int e = t; e < 8 * kHD; e += 128)
        rec[16 + e] = __ldg(vn + (e & (kHD - 1)));
}

// Combine of one launch's partial records. Grid: (n jobs x 2 kv heads x 8 query heads);
// 256 threads = 4 part groups x 64 threads of 4 output dims. Each (job, kv head) merges
// its nsplit split records plus the new token's record: M = max m_i, w_i = l_i 2^(m_i - M),
// o = sum w_i o_i / sum w_i. Part group g takes parts g, g + 4, ... (up to 8 per batch, every
// load of a batch issued before its arithmetic) and the four groups' sums are added in group
// order, so a block costs about two memory round trips and the result does not depend on
// timing. Output: the gated result (o * sigmoid(gate)), or in partial / push mode the head's
// part of one merged record (m = M, l = sum w_i, o) to p.pout / the job's push address, then in
// push mode the head's tag.
__global__ void __launch_bounds__(256) attn_combine_kernel(const __grid_constant__ DParams p)
{
    __shared__ float red[8];
    __shared__ float4 gacc[4][64];
    __shared__ float gl[4];
    const int j = blockIdx.x >> 4, kvh = (blockIdx.x >> 3) & 1, h = blockIdx.x & 7;
    const DJob &J = p.jobs[j];
    const int t = threadIdx.x, grp = t >> 6, d = (t & 63) * 4;
    // The gates are inputs, not the decode kernel's output: this grid starts only once every
    // decode CTA has passed its own griddepcontrol.wait (the kernels that wrote the inputs have
    // completed), so they are read before the wait, off the merge's critical path.
    float gv[4] = {0.f, 0.f, 0.f, 0.f};
    if (grp == 0 && !J.pdst && !p.pout) {
        const float *g = J.gate + (long long)(kvh * 8 + h) * J.qg_stride + d;
#pragma unroll
        for (int x = 0; x < 4; x++)
            gv[x] = __ldg(g + x);
    }
    griddep_wait();
    griddep_launch_dependents();
    const int ns = J.nsplit, np = ns + (J.append ? 1 : 0);
    const float *part0 = p.part + (long long)(J.item_base + kvh) * kPF;
    const float *newp = p.newpart + ((long long)j * 2 + kvh) * kPF;
    auto rec = [&](int i) { return i < ns ? part0 + (long long)i * 2 * kPF : newp; };
    float *dst = J.pdst ? J.pdst + kvh * kPF : (p.pout ? p.pout + ((long long)j * 2 + kvh) * kPF : nullptr);
    {
        // One pass over the records: part group g merges parts g, g + 4, ... with a running
        // maximum (every load of a batch issued before its arithmetic), then group 0 rescales the
        // four groups' sums to the overall maximum. One memory round trip per batch instead of a
        // first pass for the maximum.
        constexpr int B = 8;
        float Mg = -INFINITY, L = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int i0 = grp; i0 < np; i0 += 4 * B) {
            float mv[B], lv[B];
            float4 vv[B];
#pragma unroll
            for (int u = 0; u < B; u++) {
                const int i = i0 + 4 * u;
                if (i < np) {
                    const float *r = rec(i);
                    mv[u] = __ldcg(r + h);
                    lv[u] = __ldcg(r + 8 + h);
                    vv[u] = __ldcg(reinterpret_cast<const float4 *>(r + 16 + h * kHD + d));
                } else {
                    mv[u] = -INFINITY;
                    lv[u] = 0.f;
                    vv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
            float mb = Mg;
#pragma unroll
            for (int u = 0; u < B; u++)
                mb = fmaxf(mb, mv[u]);
            if (mb == -INFINITY)
                continue;
            const float sc = Mg == -INFINITY ? 0.f : exp2f(Mg - mb);
            L *= sc;
            acc.x *= sc;
            acc.y *= sc;
            acc.z *= sc;
            acc.w *= sc;
#pragma unroll
            for (int u = 0; u < B; u++) {
                const float w = (mv[u] == -INFINITY) ? 0.f : lv[u] * exp2f(mv[u] - mb);
                L += w;
                acc.x = fmaf(w, vv[u].x, acc.x);
                acc.y = fmaf(w, vv[u].y, acc.y);
                acc.z = fmaf(w, vv[u].z, acc.z);
                acc.w = fmaf(w, vv[u].w, acc.w);
            }
            Mg = mb;
        }
        gacc[grp][t & 63] = acc;
        if ((t & 63) == 0) {
            gl[grp] = L;
            red[grp] = Mg;
        }
        __syncthreads();
        if (grp == 0) {
            const float M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
            float Lt = 0.f;
#pragma unroll
            for (int g2 = 0; g2 < 4; g2++) {
                if (red[g2] == -INFINITY)
                    continue;
                const float f = exp2f(red[g2] - M);
                const float4 b = gacc[g2][t];
                a.x = fmaf(f, b.x, a.x);
                a.y = fmaf(f, b.y, a.y);
                a.z = fmaf(f, b.z, a.z);
                a.w = fmaf(f, b.w, a.w);
                Lt = fmaf(f, gl[g2], Lt);
            }
            const float inv = Lt > 0.f ? 1.0f / Lt : 0.f;
            const float o[4] = {a.x * inv, a.y * inv, a.z * inv, a.w * inv};
            if (dst) {
                if (t == 0) {
                    dst[h] = M;
                    dst[8 + h] = Lt;
                }
                *reinterpret_cast<float4 *>(dst + 16 + h * kHD + d) = make_float4(o[0], o[1], o[2], o[3]);
            } else {
                float *out = J.out + (kvh * 8 + h) * kHD + d;
#pragma unroll
                for (int x = 0; x < 4; x++)
                    out[x] = o[x] * (1.0f / (1.0f + expf(-gv[x])));
            }
        }
    }
    if (J.ptag) {
        // Every writer makes its record stores visible system-wide before the tag goes out:
        // the home GPU reads the head's record part as soon as it sees the tag.
        __threadfence_system();
        __syncthreads();
        if (t == 0)
            st_release_sys(J.ptag + kvh * 8 + h, p.epoch);
    }
}

__global__ void __launch_bounds__(kThreads, 1) attn_decode_kernel(const __grid_constant__ DParams p)
{
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    Smem &sm = *reinterpret_cast<Smem *>(smem_raw + ((128u - (raw & 127u)) & 127u));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(smem_addr(&sm.full[s]), kProd * 32);   // one cp.async arrival per producer thread
            mbar_init(smem_addr(&sm.empty[s]), 1);           // the consuming warp
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(smem_addr(&sm.qready[b]), kProd);      // one arrival per producer warp
            mbar_init(smem_addr(&sm.qfree[b]), kCons);       // one arrival per consumer warp
        }
        sm.abort = 0;
        mbar_init_fence();
    }
    __syncthreads();
    griddep_wait();                  // inputs are written by the kernels before this one
    griddep_launch_dependents();     // the combine's blocks wait (griddep_wait) for this grid's end

    if (warp >= kCons) {
        // ------------------------------------------------------------ producers (128 threads)
        // Warp pw copies rows pos = pw + 4k (k < 8) of both K and V each stage; lane -> dims
        // lane*8 .. lane*8+7 = chunk lane >> 3, 16-byte unit lane & 7, stored at unit
        // (lane & 7) ^ (pos & 7) of the chunk's row.
        const int pw = warp - kCons;
        const uint32_t ldst = (uint32_t)(lane >> 3) * kChunkBytes;
        unsigned seq = 0;
        const int i0 = p.cta_off[blockIdx.x], i1 = p.cta_off[blockIdx.x + 1];
        // Prepare the q of this CTA's k-th item into qf[k & 1] once the consumers released that
        // buffer (its use two items earlier).
        auto prep = [&](int k) -> bool {
            const int b = k & 1;
            const unsigned u = (unsigned)k >> 1;
            if (u > 0 && !mbar_wait(smem_addr(&sm.qfree[b]), (u - 1) & 1)) {
                if (lane == 0)
                    set_error(p, kErrWaitTimeout, sm);
                return false;
            }
            int jj, kh, sp, it;
            item_decode(p, i0 + k, jj, kh, sp, it);
            prep_q_warp(p, p.jobs[jj], kh, sm.qf[b], pw, lane, [] {});
            __syncwarp();
            if (lane == 0)
                mbar_arrive(smem_addr(&sm.qready[b]));
            return true;
        };
        bool ok = true;
        // the consumers' loads of the first item's q go out before the first stages' copies,
        // ahead of them in the memory system (named barrier 2: 128 arrivals, 128 waits)
        if (i0 < i1)
            named_bar_sync(2, 2 * 128);
        for (int k = 0; i0 + k < i1 && ok && !aborted(sm); k++) {
            int j, kvh, split, item;
            item_decode(p, i0 + k, j, kvh, split, item);
            const DJob &J = p.jobs[j];
            long long t0, t1;
            item_range(J, split, t0, t1);
            const int ntiles = (int)((t1 - t0 + kTile - 1) / kTile);
            const long long avail = J.length - t0;          // rows that exist from t0 on
            const __half *kg = J.k_cache + (t0 * 2 + kvh) * kHD + lane * 8;
            const __half *vg = J.v_cache + (t0 * 2 + kvh) * kHD + lane * 8;
            // (the first item's q is the consumers' to prepare: they are idle until it is ready)
            for (int i = 0; i < ntiles && ok; i++, seq++) {
                const int s = seq % kStages;
                const unsigned f = seq / kStages;
                if (f > 0 && !mbar_wait(smem_addr(&sm.empty[s]), (f - 1) & 1)) {
                    if (lane == 0)
                        set_error(p, kErrWaitTimeout, sm);
                    ok = false;
                    break;
                }
                const uint32_t st = smem_addr(&sm.stage[s][0]) + ldst;
#pragma unroll
                for (int kk = 0; kk < kTile / kProd; kk++) {
                    const int pos = pw + kProd * kk;
                    const long long row = (long long)i * kTile + pos;
                    if (row < avail) {
                        const uint32_t d = st + pos * 128 + (((lane & 7) ^ (pos & 7)) << 4);
                        cp_async16(d, kg + row * 2 * kHD);
                        cp_async16(d + kHalfBytes, vg + row * 2 * kHD);
                    }
                }
                cp_async_arrive(smem_addr(&sm.full[s]));
            }
            // the next item's q, ready while the consumers finish this item from the ring
            if (ok && i0 + k + 1 < i1)
                ok = prep(k + 1);
        }
        cp_async_wait_all();     // nothing of ours may still be landing when the CTA retires
        return;
    }

    // ---------------------------------------------------------------- consumers (128 threads)
    const int t = tid;
    unsigned seq = 0;
    const float sc = kLog2e / 16.0f;
    const int r = lane >> 2, cpair = (lane & 3) * 2;
    // Swizzled ldmatrix addressing. Row p of a [chunk][32 pos][128 B] tile holds 16-byte unit u at
    // unit u ^ (p & 7). K (A operand) rows: position (lane & 15) (+16 for the second half), units
    // ((ks & 3) * 2 + (lane >> 4)); V^T (A via .trans) rows: position (lane & 7) + 8 * (lane >> 4),
    // units ((mt & 3) * 2 + ((lane >> 3) & 1)). For both, p & 7 == lane & 7.
    const uint32_t kx = (uint32_t)((lane >> 4) ^ (lane & 7));
    const uint32_t vx = (uint32_t)(((lane >> 3) & 1) ^ (lane & 7));
    const uint32_t krow = (uint32_t)(lane & 15) * 128;
    const uint32_t vrow = (uint32_t)((lane & 7) + ((lane >> 4) << 3)) * 128;

    // The first item's q: the four consumer warps prepare it (two heads each) while the producers'
    // first stages are in flight, and arrive on its hand-off barrier in the producers' place
    // (same count), so the later items' phases are unchanged. The producers start their copies
    // once these loads are issued (named barrier 2), so the loads do not queue behind them.
    if (p.cta_off[blockIdx.x] < p.cta_off[blockIdx.x + 1]) {
        int j, kvh, split, item;
        item_decode(p, p.cta_off[blockIdx.x], j, kvh, split, item);
        prep_q_warp(p, p.jobs[j], kvh, sm.qf[0], warp, lane, [] { named_bar_arrive(2, 2 * 128); });
        __syncwarp();
        if (lane == 0)
            mbar_arrive(smem_addr(&sm.qready[0]));
    }

    int kq = 0;                                  // this CTA's item counter
    for (int idx = p.cta_off[blockIdx.x]; idx < p.cta_off[blockIdx.x + 1]; idx++, kq++) {
        int j, kvh, split, item;
        item_decode(p, idx, j, kvh, split, item);
        const DJob &J = p.jobs[j];
        long long t0, t1;
        item_range(J, split, t0, t1);
        const int ntiles = (int)((t1 - t0 + kTile - 1) / kTile);

        // the producers prepared this item's q into qf[kq & 1]; a wait that runs out records the
        // error and goes on, so every consumer warp still meets the barriers below
        const int qbuf = kq & 1;
        if (!mbar_wait(smem_addr(&sm.qready[qbuf]), ((unsigned)kq >> 1) & 1) && lane == 0)
            set_error(p, kErrWaitTimeout, sm);
        if (split == 0 && J.append)
            new_token(p, J, j, kvh, sm.qf[qbuf], sm, t);

        uint32_t qb[16][2];
#pragma unroll
        for (int ks = 0; ks < 16; ks++) {
            const float *qr = &sm.qf[qbuf][r][ks * 16 + cpair];
            qb[ks][0] = pack_f16x2(qr[0], qr[1]);
            qb[ks][1] = pack_f16x2(qr[8], qr[9]);
        }
        __syncwarp();
        if (lane == 0)
            mbar_arrive(smem_addr(&sm.qfree[qbuf]));
        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
        float o[16][4];
#pragma unroll
        for (int mt = 0; mt < 16; mt++)
            o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

        for (int i = 0; i < ntiles; i++) {
            const unsigned q = seq + i;
            if ((int)(q % kCons) != warp)
                continue;
            const int s = q % kStages;
            if (!mbar_wait(smem_addr(&sm.full[s]), (q / kStages) & 1)) {
                if (lane == 0)
                    set_error(p, kErrWaitTimeout, sm);
                break;
            }
            const uint32_t kb = smem_addr(&sm.stage[s][0]), vb = kb + kHalfBytes;
            const long long tile0 = t0 + (long long)i * kTile;
            // Rows past the window end are not loaded and hold stale data (possibly NaN bit
            // patterns): zero their V so P = 0 contributes exactly nothing. K rows there are
            // masked below.
            const long long live = J.length - tile0;
            const bool ragged = live < kTile;
            if (ragged) {
                for (int row = (int)(live > 0 ? live : 0); row < kTile; row++)
                    sts_zero16(vb + (lane >> 3) * kChunkBytes + row * 128 + (lane & 7) * 16);
                __syncwarp();
            }
            float x[2][4];
#pragma unroll
            for (int hf = 0; hf < 2; hf++) {
                float acc[2][4];
#pragma unroll
                for (int c = 0; c < 2; c++)
                    acc[c][0] = acc[c][1] = acc[c][2] = acc[c][3] = 0.f;
#pragma unroll
                for (int ks = 0; ks < 16; ks++) {
                    uint32_t a[4];
                    ldsm_x4(kb + (ks >> 2) * kChunkBytes + hf * 16 * 128 + krow +
                                ((((uint32_t)(ks & 3) << 1) ^ kx) << 4), a);
                    mma_f16(acc[ks & 1], a, qb[ks][0], qb[ks][1]);
                }
                const long long p0 = tile0 + hf * 16 + r;
                const bool v0 = p0 < t1, v1 = p0 + 8 < t1;
                x[hf][0] = v0 ? (acc[0][0] + acc[1][0]) * sc : -INFINITY;
                x[hf][1] = v0 ? (acc[0][1] + acc[1][1]) * sc : -INFINITY;
                x[hf][2] = v1 ? (acc[0][2] + acc[1][2]) * sc : -INFINITY;
                x[hf][3] = v1 ? (acc[0][3] + acc[1][3]) * sc : -INFINITY;
            }
            float mx0 = fmaxf(fmaxf(x[0][0], x[0][2]), fmaxf(x[1][0], x[1][2]));
            float mx1 = fmaxf(fmaxf(x[0][1], x[0][3]), fmaxf(x[1][1], x[1][3]));
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
            }
            const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);   // finite: row 0 is valid
            const float c0 = exp2f(m0 - n0), c1 = exp2f(m1 - n1);
            uint32_t pb[2][2];
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int hf = 0; hf < 2; hf++) {
                const float e0 = exp2f(x[hf][0] - n0), e1 = exp2f(x[hf][1] - n1);
                const float e2 = exp2f(x[hf][2] - n0), e3 = exp2f(x[hf][3] - n1);
                s0 += e0 + e2;
                s1 += e1 + e3;
                pb[hf][0] = movmatrix_t(pack_f16x2(e0, e1));
                pb[hf][1] = movmatrix_t(pack_f16x2(e2, e3));
            }
            l0 = fmaf(l0, c0, s0);
            l1 = fmaf(l1, c1, s1);
            m0 = n0;
            m1 = n1;
#pragma unroll
            for (int mt = 0; mt < 16; mt++) {
                o[mt][0] *= c0;
                o[mt][1] *= c1;
                o[mt][2] *= c0;
                o[mt][3] *= c1;
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
                    uint32_t a[4];
                    ldsm_x4_t(vb + (mt >> 2) * kChunkBytes + hf * 16 * 128 + vrow +
                                  ((((uint32_t)(mt & 3) << 1) ^ vx) << 4), a);
                    mma_f16(o[mt], a, pb[hf][0], pb[hf][1]);
                }
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(smem_addr(&sm.empty[s]));
        }
        seq += ntiles;

        // ------------------------------------------------ merge the 4 warps into one record
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            l0 += __shfl_xor_sync(0xffffffffu, l0, off);
            l1 += __shfl_xor_sync(0xffffffffu, l1, off);
        }
        if (lane < 4) {
            sm.mw[warp][cpair] = m0;
            sm.mw[warp][cpair + 1] = m1;
            sm.lw[warp][cpair] = l0;
            sm.lw[warp][cpair + 1] = l1;
        }
#pragma unroll
        for (int mt = 0; mt < 16; mt++) {
            const int d = mt * 16 + r;
            sm.u.ow[warp][cpair][d] = o[mt][0];
            sm.u.ow[warp][cpair + 1][d] = o[mt][1];
            sm.u.ow[warp][cpair][d + 8] = o[mt][2];
            sm.u.ow[warp][cpair + 1][d + 8] = o[mt][3];
        }
        named_bar_sync(1, 128);
        float *rec = p.part + (long long)item * kPF;
        for (int e = t; e < 8 * kHD; e += 128) {
            const int h = e >> 8, d = e & (kHD - 1);
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kCons; w++)
                M = fmaxf(M, sm.mw[w][h]);
            float L = 0.f, acc = 0.f;
#pragma unroll
            for (int w = 0; w < kCons; w++) {
                const float f = sm.mw[w][h] == -INFINITY ? 0.f : exp2f(sm.mw[w][h] - M);
                L = fmaf(f, sm.lw[w][h], L);
                acc = fmaf(f, sm.u.ow[w][h][d], acc);
            }
            rec[16 + e] = L > 0.f ? acc / L : 0.f;
            if (d == 0) {
                rec[h] = M;
                rec[8 + h] = L;
            }
        }
        named_bar_sync(1, 128);
        if (aborted(sm))
            break;
    }
}

// Merge of per-GPU partial records: grid (n jobs x 2 kv heads), 256 threads.
struct MParams {
    const float *partials;
    const float *gates[kMaxJobs];
    float *outs[kMaxJobs];
    long long qg_stride;
    int nparts, n, job0;
};

__global__ void __launch_bounds__(256) attn_merge_kernel(const __grid_constant__ MParams p)
{
    __shared__ float w[64][8], Ls[8];
    const int j = blockIdx.x >> 1, kvh = blockIdx.x & 1, t = threadIdx.x;
    const long long stride = (long long)p.n * 2 * kPF;
    const float *rec0 = p.partials + ((long long)(p.job0 + j) * 2 + kvh) * kPF;
    if (t < 8) {
        float M = -INFINITY, L = 0.f;
        for (int i = 0; i < p.nparts; i++)
            M = fmaxf(M, rec0[i * stride + t]);
        for (int i = 0; i < p.nparts; i++) {
            const float m = rec0[i * stride + t];
            const float x = m == -INFINITY ? 0.f : rec0[i * stride + 8 + t] * exp2f(m - M);
            w[i][t] = x;
            L += x;
        }
        Ls[t] = L;
    }
    __syncthreads();
    for (int e = t; e < 8 * kHD; e += 256) {
        const int h = e >> 8, d = e & (kHD - 1);
        float acc = 0.f;
        for (int i = 0; i < p.nparts; i++)
            acc = fmaf(w[i][h], rec0[i * stride + 16 + e], acc);
        const float o = Ls[h] > 0.f ? acc / Ls[h] : 0.f;
        const float g = p.gates[j][(long long)(kvh * 8 + h) * p.qg_stride + d];
        p.outs[j][(kvh * 8 + h) * kHD + d] = o * (1.0f / (1.0f + expf(-g)));
    }
}

// Merge on the home GPU of the records every GPU pushed into its memory (push mode): grid
// (n jobs x 2 kv heads x 8 query heads), 256 threads. The first warp waits (bounded) until each
// of the nparts records carries this step's tag for the block's head, then the merge of
// attn_combine_kernel over the parts (4 part groups x 64 threads of 4 dims). recv:
// [nparts][n][2][kPF]; tags: [nparts][n][2][8].
struct MWParams {
    const float *recv;
    const unsigned *tags;
    const float *gates[kMaxJobs];
    float *outs[kMaxJobs];
    long long qg_stride, budget;
    unsigned *err;
    int nparts, n, job0;
    unsigned epoch;
};

__global__ void __launch_bounds__(256) attn_merge_wait_kernel(const __grid_constant__ MWParams p)
{
    __shared__ float red[8];
    __shared__ float4 gacc[4][64];
    __shared__ float gl[4];
    __shared__ int ready;
    griddep_wait();
    const int j = blockIdx.x >> 4, kvh = (blockIdx.x >> 3) & 1, h = blockIdx.x & 7;
    const int t = threadIdx.x, grp = t >> 6, d = (t & 63) * 4;
    if (t < 32) {
        bool ok = true;
        for (int i = t; i < p.nparts; i += 32) {
            const unsigned *tag = p.tags + (((long long)i * p.n + p.job0 + j) * 2 + kvh) * 8 + h;
            const long long t0 = clock64();
            while (ld_acquire_sys(tag) != p.epoch) {
                if (clock64() - t0 > p.budget) {
                    ok = false;
                    break;
                }
                __nanosleep(32);
            }
        }
        ok = __all_sync(0xffffffffu, ok);
        if (t == 0)
            ready = ok ? 1 : 0;
    }
    __syncthreads();
    if (!ready) {
        if (t == 0)
            atomicOr(p.err, kErrWaitTimeout);
        return;
    }
    const long long stride = (long long)p.n * 2 * kPF;
    const float *rec0 = p.recv + ((long long)(p.job0 + j) * 2 + kvh) * kPF;
    float m = -INFINITY;
    for (int i = t; i < p.nparts; i += 256)
        m = fmaxf(m, __ldcg(rec0 + i * stride + h));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((t & 31) == 0)
        red[t >> 5] = m;
    __syncthreads();
    float M = red[0];
#pragma unroll
    for (int w = 1; w < 8; w++)
        M = fmaxf(M, red[w]);
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = grp; i < p.nparts; i += 4) {
        const float *r = rec0 + i * stride;
        const float mi = __ldcg(r + h), li = __ldcg(r + 8 + h);
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(r + 16 + h * kHD + d));
        const float w = (mi == -INFINITY) ? 0.f : li * exp2f(mi - M);
        L += w;
        acc.x = fmaf(w, v.x, acc.x);
        acc.y = fmaf(w, v.y, acc.y);
        acc.z = fmaf(w, v.z, acc.z);
        acc.w = fmaf(w, v.w, acc.w);
    }
    gacc[grp][t & 63] = acc;
    if ((t & 63) == 0)
        gl[grp] = L;
    __syncthreads();
    if (grp == 0) {
        float4 a = gacc[0][t];
        float Lt = gl[0];
#pragma unroll
        for (int g2 = 1; g2 < 4; g2++) {
            const float4 b = gacc[g2][t];
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
            Lt += gl[g2];
        }
        const float inv = Lt > 0.f ? 1.0f / Lt : 0.f;
        const float o[4] = {a.x * inv, a.y * inv, a.z * inv, a.w * inv};
        const float *g = p.gates[j] + (long long)(kvh * 8 + h) * p.qg_stride + d;
        float *out = p.outs[j] + (kvh * 8 + h) * kHD + d;
#pragma unroll
        for (int x = 0; x < 4; x++)
            out[x] = o[x] * (1.0f / (1.0f + expf(-__ldg(g + x))));
    }
}

int validate(const KernelAttnDecodeJob &j, int i, bool partial)
{
    if (!j.q || !j.q_norm || !j.k_cache || !j.v_cache)
        return fail("attn decode: job %d has a null pointer", i);
    if (!aligned16(j.k_cache) || !aligned16(j.v_cache))
        return fail("attn decode: job %d cache not 16-byte aligned", i);
    if (j.qg_stride < 256)
        return fail("attn decode: job %d qg_stride %zu < 256", i, j.qg_stride);
    if (j.append) {
        if (!j.k_new || !j.v_new || !j.k_norm)
            return fail("attn decode: job %d has a null new-token pointer", i);
        if (j.length >= j.capacity)
            return fail("attn decode: job %d window full (length %zu, capacity %zu)", i, j.length,
                        j.capacity);
    } else if (j.length > j.capacity) {
        return fail("attn decode: job %d length %zu > capacity %zu", i, j.length, j.capacity);
    }
    if (!partial && (!j.gate || !j.out))
        return fail("attn decode: job %d has a null gate/out pointer", i);
    return 0;
}

bool g_attr_set = false;

// The decode kernel, then the combine kernel, each as a programmatic dependent of the kernel
// before it (the combine's blocks are scheduled as decode CTAs retire and wait in griddep_wait
// for the whole decode grid).
// `before_combine`, when set, is an event the combine waits for (the gates' input copy, which
// the decode kernel does not read, overlaps the decode kernel).
int launch_pair(const DParams &p, int grid, cudaStream_t st, cudaEvent_t before_combine = nullptr)
{
    if (launch_dependent(attn_decode_kernel, dim3(grid), dim3(kThreads), kSmemBytes, st, "attn_decode_kernel", p) != 0)
        return -1;
    if (before_combine && check(cudaStreamWaitEvent(st, before_combine, 0), "cudaStreamWaitEvent") != 0)
        return -1;
    return launch_dependent(attn_combine_kernel, dim3((unsigned)p.njobs * 16), dim3(256), 0, st,
                            "attn_combine_kernel", p);
}

// Items per SM the planner aims for (per kv head pair). ROASTER_DECODE_ITEMS_PER_SM overrides.
double decode_items_per_sm()
{
    static double v = [] {
        const char *e = getenv("ROASTER_DECODE_ITEMS_PER_SM");
        const double x = e ? atof(e) : 1.0;
        return x > 0.05 && x < 64.0 ? x : 1.0;
    }();
    return v;
}

struct PlanItem {
    long long cost;
    unsigned short code;      // (job << 9) | (split << 1) | kv head
    short cta;
};

// Split plan and CTA assignment of one launch, shared by every entry point. Each slot's window
// is cut into equal splits of about `target` positions, target = total / (SMs x items per SM),
// doubled until the (slot, kv head, split) items fit `cap_items`; the items then go longest
// first (ties in item order) onto the least-loaded of the grid's CTAs (ties to the lower id),
// an item costing its positions plus a fixed 256 for its set-up and record. Fills
// p.jobs[i].chunk / nsplit / item_base, p.sched, p.cta_off and p.nitems; returns the grid size,
// or -1 when the batch cannot be planned. Allocates no heap memory.
int plan(const KernelAttnDecodeJob *jobs, int n, int num_sms, int cap_items, DParams &p)
{
    long long total = 0;
    for (int i = 0; i < n; i++)
        total += (long long)jobs[i].length;
    long long target = (long long)((double)total / ((double)num_sms * decode_items_per_sm())) + 1;
    if (target < 2 * kTile)
        target = 2 * kTile;
    int items = 0;
    for (int attempt = 0;; attempt++) {
        items = 0;
        for (int i = 0; i < n; i++) {
            const long long L = (long long)jobs[i].length;
            long long ns = (L + target / 2) / target;
            ns = ns < 1 ? 1 : (ns > kMaxSplits ? kMaxSplits : ns);
            long long ch = (L + ns - 1) / ns;
            ch = (ch + kTile - 1) / kTile * kTile;
            if (ch < kTile)
                ch = kTile;
            ns = (L + ch - 1) / ch;
            if (ns < 1)
                ns = 1;
            p.jobs[i].chunk = ch;
            p.jobs[i].nsplit = (int)ns;
            p.jobs[i].item_base = items;
            items += 2 * (int)ns;
        }
        if (items <= cap_items)
            break;
        if (attempt > 40) {
            fail("attn decode: cannot plan %d slots within %d items", n, cap_items);
            return -1;
        }
        target *= 2;
    }
    const int ctas = num_sms < kMaxCtas ? num_sms : kMaxCtas;
    const int grid = items < ctas ? items : ctas;
    PlanItem order[kMaxItems];
    int k = 0;
    for (int i = 0; i < n; i++) {
        const DJob &d = p.jobs[i];
        for (int sp = 0; sp < d.nsplit; sp++) {
            const long long t0 = (long long)sp * d.chunk;
            const long long t1 = std::min<long long>(t0 + d.chunk, (long long)jobs[i].length);
            for (int kvh = 0; kvh < 2; kvh++)
                order[k++] = PlanItem{(t1 > t0 ? t1 - t0 : 0) + 256, (unsigned short)((i << 9) | (sp << 1) | kvh), 0};
        }
    }
    std::sort(order, order + items, [](const PlanItem &a, const PlanItem &b) {
        return a.cost != b.cost ? a.cost > b.cost : a.code < b.code;
    });
    long long load[kMaxCtas] = {0};
    int heap[kMaxCtas];                      // binary min-heap of CTA ids by (load, id)
    auto less = [&](int a, int b) { return load[a] != load[b] ? load[a] < load[b] : a < b; };
    for (int c = 0; c < grid; c++) {
        load[c] = 0;
        heap[c] = c;
    }
    for (int it = 0; it < items; it++) {
        const int c = heap[0];
        order[it].cta = (short)c;
        load[c] += order[it].cost;
        int pos = 0;                          // sift the grown root down
        for (;;) {
            const int l = 2 * pos + 1, r = l + 1;
            int m = pos;
            if (l < grid && less(heap[l], heap[m]))
                m = l;
            if (r < grid && less(heap[r], heap[m]))
                m = r;
            if (m == pos)
                break;
            std::swap(heap[pos], heap[m]);
            pos = m;
        }
    }
    int count[kMaxCtas + 1];
    for (int c = 0; c <= grid; c++)
        count[c] = 0;
    for (int it = 0; it < items; it++)
        count[order[it].cta + 1]++;
    for (int c = 0; c < grid; c++)
        count[c + 1] += count[c];
    for (int c = 0; c <= grid; c++)
        p.cta_off[c] = (unsigned short)count[c];
    for (int it = 0; it < items; it++)
        p.sched[count[order[it].cta]++] = order[it].code;
    p.nitems = items;
    return grid;
}

// The jobs' pointers and scalars into the kernel's job table.
void fill_jobs(const KernelAttnDecodeJob *jobs, int n, DParams &p, float *const *dst, unsigned *const *tags)
{
    for (int i = 0; i < n; i++) {
        const KernelAttnDecodeJob &s = jobs[i];
        DJob &d = p.jobs[i];
        d.q = s.q;
        d.gate = s.gate;
        d.k_new = s.k_new;
        d.v_new = s.v_new;
        d.q_norm = s.q_norm;
        d.k_norm = s.k_norm;
        d.k_cache = reinterpret_cast<__half *>(s.k_cache);
        d.v_cache = reinterpret_cast<__half *>(s.v_cache);
        d.out = s.out;
        d.qg_stride = (long long)s.qg_stride;
        d.length = (long long)s.length;
        d.position = (long long)s.position;
        d.append = s.append ? 1 : 0;
        d.pdst = dst ? dst[i] : nullptr;
        d.ptag = dst ? tags[i] : nullptr;
    }
    p.njobs = n;
}

// One launch over jobs[0..n), n <= kMaxJobs. `pout` selects partial mode; `dst` + `tags`
// select push mode (job i's merged records to dst[i], then tags[i][kvh] = epoch).
int launch(const KernelAttnDecodeJob *jobs, int n, float *pout, float *const *dst = nullptr,
           unsigned *const *tags = nullptr, unsigned epoch = 0, cudaEvent_t before_combine = nullptr)
{
    if (dst) {
        for (int i = 0; i < n; i++)
            if (!dst[i] || !tags || !tags[i] || !aligned16(dst[i]))
                return fail("attn decode push: job %d needs a 16-byte aligned record address and tags", i);
        pout = nullptr;
    }
    const bool partial = pout != nullptr || dst != nullptr;
    Runtime &R = rt();
    for (int i = 0; i < n; i++)
        if (validate(jobs[i], i, partial) != 0)
            return -1;
    DParams p;
    memset(static_cast<void *>(&p), 0, sizeof(p));
    const int grid = plan(jobs, n, R.num_sms, kMaxItems, p);
    if (grid < 0)
        return -1;
    const int items = p.nitems;
    fill_jobs(jobs, n, p, dst, tags);
    p.epoch = epoch;
    memcpy(p.inv_freq, R.inv_freq, sizeof(p.inv_freq));
    const size_t part_floats = (size_t)items * kPF, new_floats = (size_t)n * 2 * kPF;
    float *ws = static_cast<float *>(scratch((part_floats + new_floats) * sizeof(float)));
    if (!ws)
        return -1;
    p.part = ws;
    p.newpart = ws + part_floats;
    p.pout = pout;
    p.err = R.err_word;
    if (!g_attr_set) {
        if (check(cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBytes), "attn decode smem attribute") != 0)
            return -1;
        g_attr_set = true;
    }
    return launch_pair(p, grid, R.stream, before_combine);
}

// ---------------------------------------------------------------- allocation-free variant
//
// Some callers cannot allocate device memory while they decode: a host that runs under a fixed
// device-memory budget handed out up front, code that must not enter the CUDA allocator (or any
// allocating library, torch's caching allocator included) once serving has started, or a
// process where allocation would serialise against other streams. For them,
// kernel_attn_decode_batch_noalloc runs the same decode and combine kernels with their scratch
// (the split softmax partial records) in this statically sized device array instead of
// library-allocated memory. Every GPU that loads the library
// holds the array until the process exits. Kernel-recorded failures go to the library's error
// word, which kernel_cuda_init allocates once at start-up, so kernel_cuda_synchronize reports
// them exactly as for the allocating entry point.
constexpr size_t kNoAllocBytes = 8u << 20;                     // 8 MiB per device
constexpr size_t kNoAllocNewFloats = (size_t)kMaxJobs * 2 * kPF;
constexpr int kNoAllocMaxItems =
    (int)((kNoAllocBytes - kNoAllocNewFloats * sizeof(float)) / (kPF * sizeof(float)));
static_assert(kNoAllocMaxItems >= 4 * kMaxJobs, "static scratch too small for a full batch");

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

namespace {

struct NoAllocDevice {
    bool ready;
    unsigned char *base;       // device address of g_noalloc_scratch on that device
    int num_sms;
};
NoAllocDevice g_noalloc_dev[64];

// Per-device set-up, once, with `device` current: resolve the array's device address (host code
// must not use the symbol itself, which on the host is only a stand-in) and the SM count; set the
// kernel's shared-memory limit. Nothing here allocates.
int noalloc_setup(int device)
{
    NoAllocDevice &d = g_noalloc_dev[device];
    if (d.ready)
        return 0;
    void *ptr = nullptr;
    if (check(cudaGetSymbolAddress(&ptr, g_noalloc_scratch), "cudaGetSymbolAddress(noalloc scratch)") != 0)
        return -1;
    int sms = 0;
    if (check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "SM count") != 0)
        return -1;
    if (check(cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)kSmemBytes), "attn decode smem attribute") != 0)
        return -1;
    d.base = static_cast<unsigned char *>(ptr);
    d.num_sms = sms < kMaxCtas ? sms : kMaxCtas;
    d.ready = true;
    return 0;
}

}  // namespace

int attn_decode_batch_noalloc(const KernelAttnDecodeJob *jobs, int n)
{
    if (n < 0 || (n > 0 && !jobs))
        return fail("kernel_attn_decode_batch_noalloc: bad job array");
    if (n > kMaxJobs)
        return fail("kernel_attn_decode_batch_noalloc: %d slots in one call; the static scratch "
                    "serves at most %d (split the batch into several calls)", n, kMaxJobs);
    if (n == 0)
        return 0;
    int device = 0;
    if (check(cudaGetDevice(&device), "cudaGetDevice") != 0)
        return -1;
    if (device < 0 || device >= 64)
        return fail("kernel_attn_decode_batch_noalloc: device %d out of range", device);
    // The call runs on the current device, which must be the one kernel_cuda_init chose: the
    // library's stream and error word belong to that device.
    if (rt().device != device)
        return fail("kernel_attn_decode_batch_noalloc: the current device is %d but the library is "
                    "initialised on %d; call kernel_cuda_init(%d) once at start-up (the only step "
                    "that allocates) and keep that device current", device, rt().device, device);
    if (noalloc_setup(device) != 0)
        return -1;
    const NoAllocDevice &dev = g_noalloc_dev[device];
    for (int i = 0; i < n; i++)
        if (validate(jobs[i], i, false) != 0)
            return -1;
    DParams p;
    memset(static_cast<void *>(&p), 0, sizeof(p));
    // Same plan as the allocating path, capped at the items the static array holds.
    const int grid = plan(jobs, n, dev.num_sms, kNoAllocMaxItems < kMaxItems ? kNoAllocMaxItems : kMaxItems, p);
    if (grid < 0)
        return -1;
    fill_jobs(jobs, n, p, nullptr, nullptr);
    for (int j = 0; j < 32; j++)           // same host libm powf the reference uses
        p.inv_freq[j] = powf(10000000.0f, -2.0f * (float)j / 64.0f);
    // Every record the kernels read is written earlier in the same call, so nothing left in the
    // array by a previous call is read and nothing needs clearing.
    float *ws = reinterpret_cast<float *>(dev.base);
    p.newpart = ws;
    p.part = ws + kNoAllocNewFloats;
    p.pout = nullptr;
    p.err = rt().err_word;          // reported by kernel_cuda_synchronize
    return launch_pair(p, grid, rt().stream);
}

}  // namespace

int attn_decode_batch(const KernelAttnDecodeJob *jobs, int n, float *pout, cudaEvent_t before_combine = nullptr)
{
    if (n < 0 || (n > 0 && !jobs))
        return fail("attn decode: bad job array");
    for (int i = 0; i < n; i += kMaxJobs) {
        const int m = n - i < kMaxJobs ? n - i : kMaxJobs;
        if (launch(jobs + i, m, pout ? pout + (size_t)i * 2 * kPF : nullptr, nullptr, nullptr, 0,
                   i == 0 ? before_combine : nullptr) != 0)
            return -1;
    }
    return 0;
}

int attn_decode_push(const KernelAttnDecodeJob *jobs, int n, float *const *dst, unsigned *const *tags,
                     unsigned epoch)
{
    if (n < 0 || (n > 0 && (!jobs || !dst || !tags)))
        return fail("kernel_attn_decode_partial_push: bad arguments");
    for (int i = 0; i < n; i += kMaxJobs) {
        const int m = n - i < kMaxJobs ? n - i : kMaxJobs;
        if (launch(jobs + i, m, nullptr, dst + i, tags + i, epoch) != 0)
            return -1;
    }
    return 0;
}

int attn_merge_wait(const float *recv, const unsigned *tags, int nparts, int n, const float *const *gates,
                    size_t qg_stride, float *const *outs, unsigned epoch)
{
    if (nparts < 1 || nparts > 64 || n < 0 || !recv || !tags || (n && (!gates || !outs)))
        return fail("attn merge wait: bad arguments (nparts %d, n %d)", nparts, n);
    for (int i = 0; i < n; i += kMaxJobs) {
        MWParams p;
        memset(&p, 0, sizeof(p));
        const int m = n - i < kMaxJobs ? n - i : kMaxJobs;
        for (int k = 0; k < m; k++) {
            p.gates[k] = gates[i + k];
            p.outs[k] = outs[i + k];
            if (!p.gates[k] || !p.outs[k])
                return fail("attn merge wait: null gate/out for job %d", i + k);
        }
        p.recv = recv;
        p.tags = tags;
        p.qg_stride = (long long)qg_stride;
        p.budget = 2000000000ll;
        p.err = rt().err_word;
        p.nparts = nparts;
        p.n = n;
        p.job0 = i;
        p.epoch = epoch;
        if (launch_dependent(attn_merge_wait_kernel, dim3(m * 16), dim3(256), 0, rt().stream,
                             "attn_merge_wait_kernel", p) != 0)
            return -1;
    }
    return 0;
}

int attn_merge(const float *partials, int nparts, int n, const float *const *gates, size_t qg_stride,
               float *const *outs)
{
    if (nparts < 1 || nparts > 64 || n < 0 || !partials || (n && (!gates || !outs)))
        return fail("attn merge: bad arguments (nparts %d, n %d)", nparts, n);
    for (int i = 0; i < n; i += kMaxJobs) {
        MParams p;
        memset(&p, 0, sizeof(p));
        const int m = n - i < kMaxJobs ? n - i : kMaxJobs;
        for (int k = 0; k < m; k++) {
            p.gates[k] = gates[i + k];
            p.outs[k] = outs[i + k];
            if (!p.gates[k] || !p.outs[k])
                return fail("attn merge: null gate/out for job %d", i + k);
        }
        p.partials = partials;
        p.qg_stride = (long long)qg_stride;
        p.nparts = nparts;
        p.n = n;
        p.job0 = i;
        attn_merge_kernel<<<m * 2, 256, 0, rt().stream>>>(p);
        if (launched("attn_merge_kernel") != 0)
            return -1;
    }
    return 0;
}

}  // namespace rb

using namespace rb;

extern "C" int kernel_attn_decode_batch(const KernelAttnDecodeJob *jobs, int n)
{
    if (ensure() != 0)
        return -1;
    return attn_decode_batch(jobs, n, nullptr);
}

extern "C" int kernel_attn_decode_batch_noalloc(const KernelAttnDecodeJob *jobs, int n)
{
    return attn_decode_batch_noalloc(jobs, n);
}

extern "C" int kernel_attn_decode_partial_batch(const KernelAttnDecodeJob *jobs, int n, float *partials)
{
    if (ensure() != 0)
        return -1;
    if (!partials)
        return fail("kernel_attn_decode_partial_batch: null partials");
    return attn_decode_batch(jobs, n, partials);
}

extern "C" int kernel_attn_merge_partials(const float *partials, int nparts, int n,
                                          const float *const *gates, size_t qg_stride,
                                          float *const *outs)
{
    if (ensure() != 0)
        return -1;
    return attn_merge(partials, nparts, n, gates, qg_stride, outs);
}

extern "C" int kernel_attn_decode_partial_push(const KernelAttnDecodeJob *jobs, int n, float *const *dst,
                                               unsigned *const *tags, unsigned epoch)
{
    if (ensure() != 0)
        return -1;
    return attn_decode_push(jobs, n, dst, tags, epoch);
}

extern "C" int kernel_attn_merge_wait(const float *recv, const unsigned *tags, int nparts, int n,
                                      const float *const *gates, size_t qg_stride, float *const *outs,
                                      unsigned epoch)
{
    if (ensure() != 0)
        return -1;
    return attn_merge_wait(recv, tags, nparts, n, gates, qg_stride, outs, epoch);
}

// Host-buffer batch: pack every job's q/gate rows, new K/V, norms into one pinned block, one
// H2D copy, the device batch, one D2H copy of the outputs.
extern "C" int kernel_attn_decode_batch_host(const KernelAttnDecodeJob *jobs, int n)
{
    if (ensure() != 0)
        return -1;
    if (n < 0 || (n > 0 && !jobs))
        return fail("kernel_attn_decode_batch_host: bad job array");
    if (n == 0)
        return 0;
    // per job: q 4096, gate 4096, k 512, v 512, qnorm 256, knorm 256 in; out 4096
    const size_t in_f = 4096 * 2 + 512 * 2 + 256 * 2, out_f = 4096;
    const size_t total = (size_t)n * (in_f + out_f);
    float *h = static_cast<float *>(pinned(total * sizeof(float)));
    if (!h)
        return -1;
    std::vector<KernelAttnDecodeJob> dj(jobs, jobs + n);
    for (int i = 0; i < n; i++) {
        const KernelAttnDecodeJob &s = jobs[i];
        if (!s.q || !s.gate || !s.out || !s.q_norm || (s.append && (!s.k_new || !s.v_new || !s.k_norm)))
            return fail("kernel_attn_decode_batch_host: job %d has a null pointer", i);
    }
    // Registered buffers: when every host buffer of every job lies in memory registered with
    // kernel_cuda_host_register, the copy engine moves the buffers' contiguous runs straight
    // between host and device (a few large copies per call, no staging memcpy on the host). The
    // gates are read only by the combine kernel: when their runs are apart from the other inputs'
    // (separate q and gate buffers), they copy in on the copy stream while the decode kernel
    // runs, and the combine waits for them. Interleaved q|gate rows form one run set.
    {
        HostRuns in, late, out;
        bool reg = true;
        for (int i = 0; i < n && reg; i++) {
            const KernelAttnDecodeJob &s = jobs[i];
            const size_t rows = (15 * s.qg_stride + 256) * sizeof(float);
            reg = host_registered(s.q, rows) && host_registered(s.gate, rows) &&
                  host_registered(s.q_norm, 1024) && host_registered(s.out, 4096 * sizeof(float)) &&
                  (!s.append || (host_registered(s.k_new, 2048) && host_registered(s.v_new, 2048) &&
                                 host_registered(s.k_norm, 1024)));
            in.add(s.q, rows);
            late.add(s.gate, rows);
            in.add(s.q_norm, 1024);
            if (s.append) {
                in.add(s.k_new, 2048);
                in.add(s.v_new, 2048);
                in.add(s.k_norm, 1024);
            }
            out.add(s.out, 4096 * sizeof(float));
        }
        if (reg) {
            in.build(kRunGap);
            late.build(kRunGap);
            cudaStream_t cs = nullptr;
            static cudaEvent_t ev[2];               // decode inputs queued, gates landed
            static int made = -1;
            bool split = !runs_overlap(in, late);
            if (split && made != rt().device) {
                for (auto &e : ev)
                    if (check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate") != 0)
                        return -1;
                made = rt().device;
            }
            if (split && !(cs = copy_stream()))
                return -1;
            if (!split) {
                for (const auto &g : late.segs)
                    in.segs.push_back(g);
                in.build(kRunGap);
                late = HostRuns();
            }
            out.build(0);
            const size_t in_bytes = (in.bytes + 15) & ~(size_t)15, late_bytes = (late.bytes + 15) & ~(size_t)15;
            char *d = static_cast<char *>(dstage(in_bytes + late_bytes + out.bytes + 32));
            if (!d)
                return -1;
            char *dlate = d + in_bytes, *dout = dlate + late_bytes + 16;
            // the gates follow the decode kernel's inputs on the host link, not beside them
            if (runs_h2d(in, d) != 0)
                return -1;
            if (split && (check(cudaEventRecord(ev[0], rt().stream), "cudaEventRecord") != 0 ||
                          check(cudaStreamWaitEvent(cs, ev[0], 0), "cudaStreamWaitEvent") != 0 ||
                          runs_copy(late, dlate, cudaMemcpyHostToDevice, cs) != 0 ||
                          check(cudaEventRecord(ev[1], cs), "cudaEventRecord") != 0))
                return -1;
            for (int i = 0; i < n; i++) {
                const KernelAttnDecodeJob &s = jobs[i];
                KernelAttnDecodeJob &t = dj[i];
                auto at = [&](const float *p) { return reinterpret_cast<const float *>(d + in.offset(p)); };
                t.q = at(s.q);
                t.gate = split ? reinterpret_cast<const float *>(dlate + late.offset(s.gate)) : at(s.gate);
                t.q_norm = at(s.q_norm);
                if (s.append) {
                    t.k_new = at(s.k_new);
                    t.v_new = at(s.v_new);
                    t.k_norm = at(s.k_norm);
                }
                t.out = reinterpret_cast<float *>(dout + out.offset(s.out));
            }
            if (attn_decode_batch(dj.data(), n, nullptr, split ? ev[1] : nullptr) != 0 || runs_d2h(out, dout) != 0)
                return -1;
            return kernel_cuda_synchronize() != 0 ? -1 : 0;
        }
    }
    dj.assign(jobs, jobs + n);
    float *dev_in = static_cast<float *>(dstage(total * sizeof(float)));
    if (!dev_in)
        return -1;
    const int in_ok = stage_in(h, dev_in, n, in_f, [&](int i, float *b) {
        const KernelAttnDecodeJob &s = jobs[i];
        for (int r = 0; r < 16; r++) {
            memcpy(b + r * 256, s.q + r * s.qg_stride, 256 * 4);
            memcpy(b + 4096 + r * 256, s.gate + r * s.qg_stride, 256 * 4);
        }
        if (s.append) {
            memcpy(b + 8192, s.k_new, 512 * 4);
            memcpy(b + 8704, s.v_new, 512 * 4);
            memcpy(b + 9472, s.k_norm, 256 * 4);
        }
        memcpy(b + 9216, s.q_norm, 256 * 4);
    });
    if (in_ok != 0)
        return -1;
    float *dout = dev_in + (size_t)n * in_f;
    for (int i = 0; i < n; i++) {
        float *b = dev_in + (size_t)i * in_f;
        dj[i].q = b;
        dj[i].gate = b + 4096;
        dj[i].qg_stride = 256;
        dj[i].k_new = b + 8192;
        dj[i].v_new = b + 8704;
        dj[i].q_norm = b + 9216;
        dj[i].k_norm = b + 9472;
        dj[i].out = dout + (size_t)i * out_f;
    }
    if (attn_decode_batch(dj.data(), n, nullptr) != 0)
        return -1;
    if (stage_out(h + (size_t)n * in_f, dout, n, out_f,
                  [&](int i, const float *b) { memcpy(jobs[i].out, b, out_f * 4); }) != 0)
        return -1;
    return kernel_cuda_synchronize() != 0 ? -1 : 0;
}

extern "C" int kernel_attn_decode(const float *q_gate, const float *k_new, const float *v_new,
                                  const float *q_norm, const float *k_norm, uint16_t *k_cache,
                                  uint16_t *v_cache, size_t capacity, size_t length, size_t position,
                                  float *out)
{
    if (!q_gate)
        return fail("kernel_attn_decode: null q_gate");
    KernelAttnDecodeJob j;
    memset(&j, 0, sizeof(j));
    j.q = q_gate;
    j.gate = q_gate + 256;
    j.qg_stride = 512;
    j.k_new = k_new;
    j.v_new = v_new;
    j.q_norm = q_norm;
    j.k_norm = k_norm;
    j.k_cache = k_cache;
    j.v_cache = v_cache;
    j.capacity = capacity;
    j.length = length;
    j.position = position;
    j.out = out;
    j.append = 1;
    return kernel_attn_decode_batch_host(&j, 1);
}
