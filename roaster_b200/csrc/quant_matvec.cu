// k-quant matrix-vector products for the layer projections of a decode step: the batched
// kernel_matvec_quant_batch of the reference (src/kernels.h:30-44; CPU path kernels.c:150-578)
// with the weights resident in device memory.
//
//   y[r] = sum_c W[r][c] x[c],  W rows of 256-weight blocks:
//   Q4_K (144 B): f16 d, f16 dmin, 12 bytes of packed 6-bit scales/mins, 128 bytes of nibbles;
//        group g (64 weights): qs[32g + i] low nibble -> weight 64g + i (scale/min j = 2g), high
//        nibble -> 64g + 32 + i (j = 2g + 1); weight = d sc_j q - dmin m_j
//        (q4_k_get_scales, kernels.c:155-174).
//   Q6_K (210 B): ql[128], qh[64], int8 scales[16], f16 d; half n, l < 32: the low nibbles of
//        ql[64n + l], ql[64n + 32 + l] and the high ones, with the bit pairs of qh[32n + l],
//        are weights 128n + l, +32, +64, +96 with scales sc[8n + l/16 + 0, 2, 4, 6];
//        weight = d sc (q - 32) (kernels.c:437-488).
//
// The op streams the weights once (0.5625 B per weight for Q4_K, 0.8203 for Q6_K); at HBM rate
// an SM has about 6 cycles per 144-byte block, so the per-weight work has to stay at a few
// instructions per 8 weights. The staged kernel does the products on the tensor cores (warp MMA
// m16n8k16, f16 inputs, fp32 accumulation):
//
//  * Sixteen warps per CTA, each streaming its own tiles of 16 rows one block at a time through a
//    private ring of shared memory, one tensor-map box copy per block (16 rows x the block's
//    16-byte-aligned window; Q4_K: 5 stages of 16 x 144 B; Q6_K: 3 stages of 16 x 240 B; rows
//    past the matrix arrive as zeros). Warps never wait on one another inside a job, and each
//    keeps about 8 KB in flight.
//  * Lane (g, t) holds rows g and g + 8 of the tile. Weights enter the A fragment as exact f16
//    subnormals: a Q4_K nibble field ANDed in place is q 2^-24 (low) or q 2^-20 (high), a Q6_K
//    6-bit field q 2^-24 - one AND per two weights, no conversion.
//  * The activation, scaled by a power of two so its largest element sits near 2^14, is split
//    into f16 hi + lo (about 22 bits) and enters B as two columns. In each window of four scale
//    groups (Q4_K: four 32-weight sub-blocks; Q6_K: four 16-weight groups) lane t's k-slots hold
//    only group t and only lanes 2t, 2t+1 of the B fragment are non-zero, so accumulator columns
//    2t, 2t+1 of lane t are exactly group t's dot product: one fp32 scale per lane per window.
//  * The B fragments of a job (1 KB per block) and its activation sums per scale group (for the
//    Q4_K min and the Q6_K -32 terms) are built in shared memory at the start of each job a CTA
//    works on (the only CTA-wide syncs, on a bounded mbarrier). CTAs take contiguous tile ranges
//    of about equal cost. When a call has fewer than two tiles per warp, tiles split into 2-16 parts
//    along the blocks; parts leave fp32 partials and the last one of a tile sums them in order.
//
// Matrices the staged kernel does not take (not 16-byte aligned, rows longer than 4096 weights,
// Q6_K rows that are not a multiple of 16 bytes) run in the row kernel: one warp per row reading
// global memory directly.
//
// Multi-token products (kernel_matmul_quant_batch, kernels.h:51-64) of 8 or more tokens run in
// quant_matmul_kernel: a CTA multiplies 256 rows by 32 tokens, so each weight block is read and
// decoded once per 32 tokens, with the scales folded into the A fragments (exact f16 products)
// and each token's activation split hi + lo in B; described where the kernel is defined.
#include "ptx.cuh"
#include "runtime.h"
#include "tcgen05.cuh"
#include "../../include/roaster_cuda.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstring>
#include <unordered_map>
#include <vector>

namespace rb {
namespace {

constexpr int kMaxJobs = 64;
// Per-token row pointers a tensor-core call may carry in each parameter block (the activations'
// rows, the results' rows): a job with a table reads or writes token t's row through entry
// `first + t` instead of one contiguous [T][cols] / [T][rows] block.
constexpr int kRowTab = 320;

// ---------------------------------------------------------------- staged kernel geometry

constexpr int kCWarps = 16;
constexpr int kCThreads = kCWarps * 32;
constexpr int kThreads = kCThreads;
constexpr int kRingBytes = 12 * 1024;            // per warp
constexpr int kQ4Slot = 144, kQ6Slot = 240;      // staged bytes per row of one block
constexpr int kQ4Stages = kRingBytes / (16 * kQ4Slot);   // 5
constexpr int kQ6Stages = kRingBytes / (16 * kQ6Slot);   // 3
constexpr int kMaxNb = 16;                       // staged path: up to 16 blocks (4096 weights) a row
constexpr int kOffBtab = kCWarps * kRingBytes;   // B fragments: 1 KB per block
constexpr int kOffXsum = kOffBtab + kMaxNb * 1024;   // activation sums: 16 a block (Q6_K), 8 (Q4_K)
constexpr int kOffMisc = kOffXsum + kMaxNb * 16 * 4; // max reduction (one float per warp)
constexpr int kOffJobs = kOffMisc + kCWarps * 4;     // the job table, copied from the parameters
constexpr int kOffZero = kOffJobs + kMaxJobs * 80;   // 1 KB of zeros: B fragments of the zero lanes
constexpr int kOffWBar = kOffZero + 1024;            // per warp: 8 stage barriers
constexpr int kOffBar = kOffWBar + kCWarps * 64;     // job barrier
constexpr int kSmemBytes = kOffBar + 8;
constexpr int kMaxCtas = 160;
static_assert(kSmemBytes <= 232448, "staged matvec exceeds the shared memory of a CTA");
static_assert(kQ4Stages >= 3 && kQ6Stages >= 3, "rings too small");
static_assert(kOffJobs % 16 == 0, "job table alignment");

struct SJob {
    const CUtensorMap *map;      // the matrix as rows x (row bytes) uint8, box one slot x 16 rows
    const unsigned char *w;      // rows x nb blocks, 16-byte aligned
    const float *x;
    float *y;
    float *part;                 // split tiles: partial sums [tile][part][16]
    int *cnt;                    // split tiles: arrivals per tile (zero between calls)
    long long item0;             // first global item (a tile of 16 rows, or a part of one) of the job
    long long rows;              // rows in tiles (the last Q6_K row may go to the row kernel)
    int nb, is_q6, plog;         // blocks per row; format; log2 of the parts per tile
};

static_assert(sizeof(SJob) <= 80, "job table slot");

struct SParams {
    SJob jobs[kMaxJobs];
    int njobs;
    long long items;
    long long cta_item[kMaxCtas + 1];   // CTA c takes items [cta_item[c], cta_item[c + 1])
    unsigned *err;
};

struct DJob {
    const unsigned char *w;
    const float *x;
    float *y;
    long long drow0;             // first global row of the job in the row kernel
    long long rows;
    int nb, is_q6;
};

struct DParams {
    DJob jobs[kMaxJobs];
    int njobs;
    long long drows;
};

// ---------------------------------------------------------------- staged kernel


// One box of a 2-D tensor map (in global memory) into shared memory, completion as transaction
// bytes on `bar`. x (bytes) is a multiple of 16.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Device-scope acquire-release increment; returns the old value.
__device__ __forceinline__ int arrive_acq_rel(int *p)
{
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(p) : "memory");
    return old;
}


// D += A * B, m16n8k16, f16 inputs, fp32 accumulation (not volatile: free to schedule).
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 lds128(const unsigned char *p)
{
    return *reinterpret_cast<const uint4 *>(p);
}

__device__ __forceinline__ uint32_t lds32(const unsigned char *p)
{
    return *reinterpret_cast<const uint32_t *>(p);
}

__device__ __forceinline__ uint32_t word_of(const uint4 &v, int i)
{
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Byte `sel` of each word as 2^23 + byte, less 2^23 (exact small integers as floats).
__device__ __forceinline__ float2 bytes_as_float2(uint32_t a, uint32_t b, uint32_t sel)
{
    const float2 f = make_float2(__uint_as_float(__byte_perm(a, 0x4B000000u, sel)),
                                 __uint_as_float(__byte_perm(b, 0x4B000000u, sel)));
    return __fadd2_rn(f, make_float2(-8388608.f, -8388608.f));
}

// Two int8 values (bytes 0, 1 of u) times d: (u ^ 0x80 bytes as 2^23 + 128 + v) - (2^23 + 128).
__device__ __forceinline__ float2 int8_pair_times(uint32_t u, float d)
{
    u ^= 0x8080u;
    const float2 f = make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650u)),
                                 __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651u)));
    return __fmul2_rn(__fadd2_rn(f, make_float2(-8388736.f, -8388736.f)), make_float2(d, d));
}

// Per-lane constants of the staged kernel.
struct Lane {
    int g, t;
    bool bnz;            // this lane's B fragment is non-zero (g >> 1 == t)
    int l8;              // its index among the eight non-zero lanes
    uint32_t sel;        // byte t of a word
};

// One Q4_K block of rows (g, g + 8) of a tile: window W covers sub-blocks 4W..4W+3, lane t's
// k-slots hold sub-block 4W + t (byte group 2W + t/2, nibble t&1), eight MMAs per window. `bt` is
// this lane's B column: its entries of the block's table, or the zero area for a zero lane.
__device__ __forceinline__ void q4_mma_block(const unsigned char *pa, const unsigned char *pb, const uint4 *bt,
                                             const float *xs, float f4, const Lane &L, float &acc_a, float &acc_b)
{
    const uint4 ha = lds128(pa), hb = lds128(pb);
    // scales and mins of sub-blocks t and 4 + t (q4_k_get_scales, four bytes at a time)
    float2 sa, ma, sb, mb;
    {
        const uint32_t scl = ha.y & 0x3F3F3F3Fu, mnl = ha.z & 0x3F3F3F3Fu;
        const uint32_t sch = (ha.w & 0x0F0F0F0Fu) | ((ha.y >> 2) & 0x30303030u);
        const uint32_t mnh = ((ha.w >> 4) & 0x0F0F0F0Fu) | ((ha.z >> 2) & 0x30303030u);
        const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&ha.x));
        const float ds = dd.x * f4;
        sa = __fmul2_rn(bytes_as_float2(scl, sch, L.sel), make_float2(ds, ds));
        ma = __fmul2_rn(bytes_as_float2(mnl, mnh, L.sel), make_float2(dd.y, dd.y));
    }
    {
        const uint32_t scl = hb.y & 0x3F3F3F3Fu, mnl = hb.z & 0x3F3F3F3Fu;
        const uint32_t sch = (hb.w & 0x0F0F0F0Fu) | ((hb.y >> 2) & 0x30303030u);
        const uint32_t mnh = ((hb.w >> 4) & 0x0F0F0F0Fu) | ((hb.z >> 2) & 0x30303030u);
        const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&hb.x));
        const float ds = dd.x * f4;
        sb = __fmul2_rn(bytes_as_float2(scl, sch, L.sel), make_float2(ds, ds));
        mb = __fmul2_rn(bytes_as_float2(mnl, mnh, L.sel), make_float2(dd.y, dd.y));
    }
    const uint32_t mask = (L.t & 1) ? 0x00F000F0u : 0x000F000Fu;
#pragma unroll
    for (int W = 0; W < 2; W++) {
        const int G = 2 * W + (L.t >> 1);
        const uint4 qa0 = lds128(pa + 16 + 32 * G), qa1 = lds128(pa + 32 + 32 * G);
        const uint4 qb0 = lds128(pb + 16 + 32 * G), qb1 = lds128(pb + 32 + 32 * G);
        uint4 bf[4];
#pragma unroll
        for (int i = 0; i < 4; i++)
            bf[i] = bt[(W * 4 + i) * 8];
        float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 8; s++) {
            const uint32_t wa = word_of(s < 4 ? qa0 : qa1, s & 3), wb = word_of(s < 4 ? qb0 : qb1, s & 3);
            const uint32_t b0 = (s & 1) ? bf[s >> 1].z : bf[s >> 1].x;
            const uint32_t b1 = (s & 1) ? bf[s >> 1].w : bf[s >> 1].y;
            mma16816(c, wa & mask, wb & mask, (wa >> 8) & mask, (wb >> 8) & mask, b0, b1);
        }
        const float xw = xs[4 * W + L.t];
        const float2 s2 = W ? make_float2(sa.y, sb.y) : make_float2(sa.x, sb.x);
        const float2 m2 = W ? make_float2(ma.y, mb.y) : make_float2(ma.x, mb.x);
        acc_a = fmaf(s2.x, c[0] + c[1], fmaf(-m2.x, xw, acc_a));
        acc_b = fmaf(s2.y, c[2] + c[3], fmaf(-m2.y, xw, acc_b));
    }
}

// Four consecutive logical words at byte offset `off` of a Q6_K block starting at `bp` (any even
// address): aligned loads, shifted by 16 bits when the words straddle.
template <bool kAligned>
__device__ __forceinline__ void q6_words(const unsigned char *bp, int off, uint32_t (&w)[4])
{
    const unsigned char *a = bp + off;
    if (kAligned) {                  // the block starts on a 4-byte boundary: plain word loads
#pragma unroll
        for (int i = 0; i < 4; i++)
            w[i] = lds32(a + 4 * i);
        return;
    }
    const unsigned char *al = reinterpret_cast<const unsigned char *>(reinterpret_cast<uintptr_t>(a) & ~(uintptr_t)3);
    const uint32_t sh = 8u * (uint32_t)(reinterpret_cast<uintptr_t>(a) & 3);
    uint32_t prev = lds32(al);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t nxt = lds32(al + 4 * i + 4);
        w[i] = __funnelshift_r(prev, nxt, sh);
        prev = nxt;
    }
}

// One Q6_K block of rows (g, g + 8): window (n, h) covers scale groups 8n + 2q + h, q = 0..3;
// lane t's k-slots hold group q = t (16 weights 128n + 32t + 16h + l), four MMAs per window.
template <bool kAligned>
__device__ __forceinline__ void q6_mma_block(const unsigned char *pa, const unsigned char *pb, const uint4 *bt,
                                             const float *xs, float f6, const Lane &L, float &acc_a, float &acc_b)
{
    const int sl = 4 * (L.t >> 1);                   // nibble: low for groups q = 0, 1
    const int rot = (2 * L.t - 4) & 31;              // qh bits 2t, 2t+1 of each byte to bits 4, 5
    // scales 8n + 2t + h for (n, h) = (0,0), (0,1) [s01] and (1,0), (1,1) [s23], times d
    const float da = __half2float(*reinterpret_cast<const __half *>(pa + 208));
    const float db = __half2float(*reinterpret_cast<const __half *>(pb + 208));
    const float2 sa01 = int8_pair_times(*reinterpret_cast<const unsigned short *>(pa + 192 + 2 * L.t), da);
    const float2 sa23 = int8_pair_times(*reinterpret_cast<const unsigned short *>(pa + 200 + 2 * L.t), da);
    const float2 sb01 = int8_pair_times(*reinterpret_cast<const unsigned short *>(pb + 192 + 2 * L.t), db);
    const float2 sb23 = int8_pair_times(*reinterpret_cast<const unsigned short *>(pb + 200 + 2 * L.t), db);
#pragma unroll
    for (int win = 0; win < 4; win++) {
        const int n = win >> 1, h = win & 1;
        uint32_t la[4], lb[4], ha[4], hb[4];
        q6_words<kAligned>(pa, 64 * n + 32 * (L.t & 1) + 16 * h, la);
        q6_words<kAligned>(pb, 64 * n + 32 * (L.t & 1) + 16 * h, lb);
        q6_words<kAligned>(pa, 128 + 32 * n + 16 * h, ha);
        q6_words<kAligned>(pb, 128 + 32 * n + 16 * h, hb);
        const uint4 bf[2] = {bt[(win * 2 + 0) * 8], bt[(win * 2 + 1) * 8]};
        float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const uint32_t qa = ((la[s] >> sl) & 0x0F0F0F0Fu) | (__funnelshift_r(ha[s], ha[s], rot) & 0xF0F0F0F0u);
            const uint32_t qb = ((lb[s] >> sl) & 0x0F0F0F0Fu) | (__funnelshift_r(hb[s], hb[s], rot) & 0xF0F0F0F0u);
            const uint32_t b0 = (s & 1) ? bf[s >> 1].z : bf[s >> 1].x;
            const uint32_t b1 = (s & 1) ? bf[s >> 1].w : bf[s >> 1].y;
            mma16816(c, qa & 0x003F003Fu, qb & 0x003F003Fu, (qa >> 8) & 0x003F003Fu, (qb >> 8) & 0x003F003Fu,
                     b0, b1);
        }
        // group k = 8n + 2t + h: d sc_k (sum q x - 32 sum x)
        const float xk = xs[8 * n + 2 * L.t + h];
        const float sa = n ? (h ? sa23.y : sa23.x) : (h ? sa01.y : sa01.x);
        const float sb = n ? (h ? sb23.y : sb23.x) : (h ? sb01.y : sb01.x);
        acc_a = fmaf(sa, fmaf(c[0] + c[1], f6, -32.f * xk), acc_a);
        acc_b = fmaf(sb, fmaf(c[2] + c[3], f6, -32.f * xk), acc_b);
    }
}

// CTA-wide sync on the job barrier (one arrival per warp, bounded wait). False on timeout.
__device__ __forceinline__ bool jb_sync(uint32_t jb, uint32_t &jph, int lane)
{
    __syncwarp();
    if (lane == 0)
        mbar_arrive(jb);
    const bool ok = mbar_wait(jb, jph & 1u);
    jph++;
    return __all_sync(0xffffffffu, ok);
}

// Build the shared-memory tables of job J: B fragments (x scaled by 2^e, split f16 hi/lo) and the
// activation sums per scale group. Called by every thread; one round of global loads, two syncs on
// the job barrier. Sets e (the activation scale exponent); false if a sync timed out.
//
// B entry (b, window, MMA pair, lane8) = 16 bytes = (b0, b1) of two MMAs for one of the eight
// non-zero lanes (lane8 = 2t + hi/lo). k-slots 2t, 2t+1 <- activations u = 0, 2 and 2t+8, 2t+9
// <- u = 1, 3 of the four weights of MMA s in lane t's group. Q4_K: index (W * 4 + pair) * 8 +
// lane8 within a block, group = sub-block 4W + t; Q6_K: (window (n, h) * 2 + pair) * 8 + lane8,
// group 8n + 2t + h.
__device__ bool build_tables(const SJob &J, unsigned char *sm, int tid, uint32_t jb, uint32_t &jph, int &e)
{
    const int cols = J.nb * 256, nent = J.nb * 64;
    float v[2][8];
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const int en = tid + i * kCThreads;
        if (en < nent) {
            const int l8 = en & 7, blk = en >> 6, t = l8 >> 1;
            int base;
            if (J.is_q6) {
                const int pr = (en >> 3) & 1, win = (en >> 4) & 3;
                base = blk * 256 + 128 * (win >> 1) + 32 * t + 16 * (win & 1) + 8 * pr;
            } else {
                const int pr = (en >> 3) & 3, W = (en >> 5) & 1;
                base = blk * 256 + 32 * (4 * W + t) + 8 * pr;
            }
            const float4 a = __ldg(reinterpret_cast<const float4 *>(J.x + base));
            const float4 b = __ldg(reinterpret_cast<const float4 *>(J.x + base + 4));
            v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
            v[i][4] = b.x; v[i][5] = b.y; v[i][6] = b.z; v[i][7] = b.w;
#pragma unroll
            for (int k = 0; k < 8; k++)
                mx = fmaxf(mx, fabsf(v[i][k]));
        }
    }
    // activation sums per scale group: Q4_K 32 weights (8 a block), Q6_K 16 weights indexed
    // 8n + 2q + h like the scales (16 a block)
    const int per = J.is_q6 ? 16 : 32, ngr = cols / per;
    float xsum = 0.f;
    if (tid < ngr) {
        int start;
        if (J.is_q6) {
            const int blk = tid >> 4, k = tid & 15;
            start = blk * 256 + 128 * (k >> 3) + 32 * ((k >> 1) & 3) + 16 * (k & 1);
        } else {
            start = tid * 32;
        }
        const float4 *xp = reinterpret_cast<const float4 *>(J.x + start);
        float4 xv[8];
#pragma unroll
        for (int i = 0; i < 8; i++)
            xv[i] = (i < per / 4) ? __ldg(xp + i) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int i = 0; i < 8; i++)
            xsum += (xv[i].x + xv[i].y) + (xv[i].z + xv[i].w);
    }
    float *red = reinterpret_cast<float *>(sm + kOffMisc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0)
        red[tid >> 5] = mx;
    if (!jb_sync(jb, jph, tid & 31))
        return false;
    mx = red[0];
#pragma unroll
    for (int i = 1; i < kCWarps; i++)
        mx = fmaxf(mx, red[i]);
    int E = 0;
    if (mx > 0.f && mx < 3.0e38f)
        frexpf(mx, &E);
    e = max(-100, min(100, 14 - E));
    const float scale = ldexpf(1.f, e);
    uint4 *bt = reinterpret_cast<uint4 *>(sm + kOffBtab);
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const int en = tid + i * kCThreads;
        if (en < nent) {
            const bool lo = en & 1;
            uint32_t hw[8];
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const float s = v[i][k] * scale;
                const __half hh = __float2half_rn(s);
                hw[k] = (uint32_t)__half_as_ushort(lo ? __float2half_rn(s - __half2float(hh)) : hh);
            }
            bt[en] = make_uint4(hw[0] | (hw[2] << 16), hw[1] | (hw[3] << 16), hw[4] | (hw[6] << 16),
                                hw[5] | (hw[7] << 16));
        }
    }
    if (tid < ngr)
        reinterpret_cast<float *>(sm + kOffXsum)[tid] = xsum;
    return jb_sync(jb, jph, tid & 31);
}

__device__ __forceinline__ int item_job(const SJob *jobs, int njobs, long long t)
{
    int lo = 0, hi = njobs - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (jobs[mid].item0 <= t)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

// One warp's share of a CTA segment of job J: its items it0 + warp, it0 + warp + 16, ... < it1
// (job-relative). Item i is part i & (P-1) of tile i >> plog: blocks [part * nb/P, +nb/P) of 16
// rows. Items advance by 16, a multiple of P, so a warp keeps its part and moves 16/P tiles per
// item. Each block of an item is one tensor-map box (16 rows x one slot; rows past the matrix
// read as zeros) landing in the warp's S-stage ring; lane 0 issues the box S - 1 blocks ahead
// before a block is multiplied. `ph` holds the parity each of the warp's stage barriers completes
// next (kept across segments). A whole tile (P = 1) stores y directly; the parts of a split tile
// store fp32 partials, and the last part to arrive (a counter per tile, returned to zero) sums
// them in part order into y.
template <int S, bool Q6>
__device__ __forceinline__ bool run_segment(const SJob &Jsm, long long it0, long long it1, unsigned char *sm,
                                            unsigned char *ring, uint32_t wbar, uint32_t &ph, uint32_t jb,
                                            uint32_t &jph, const Lane &L, int warp, int lane)
{
    constexpr int kSlot = Q6 ? kQ6Slot : kQ4Slot;
    constexpr int kStage = 16 * kSlot;
    // the job's fields in registers (the table in shared memory would be re-read every block)
    const CUtensorMap *const map = Jsm.map;
    const long long rows = Jsm.rows;
    const int nb = Jsm.nb, plog = Jsm.plog, P = 1 << plog, nbp = nb >> plog;
    const long long first = it0 + warp;
    const int nitems = first < it1 ? (int)((it1 - first + kCWarps - 1) / kCWarps) : 0;
    const int part = (int)(first & (P - 1));
    const int b0 = part * nbp;                             // first block of every item of this warp
    const int trow = (kCWarps >> plog) * 16;               // rows from one item to the next
    const uint32_t ring_s = smem_addr(ring);
    // issue state: item count, block within the item, stage, the item's first row
    int is_n = 0, is_b = 0, is_s = 0, issued = 0;
    int is_row0 = (int)((first >> plog) * 16);
    auto issue = [&]() {
        if (is_n < nitems) {
            if (lane == 0) {
                const int bx = b0 + is_b;
                const int x = Q6 ? (210 * bx) & ~15 : 144 * bx;
                // the stage was last read through the generic proxy; the box writes it through the async one
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive_expect_tx(wbar + 8u * is_s, (uint32_t)kStage);
                tma_load_2d(ring_s + is_s * kStage, map, x, is_row0, wbar + 8u * is_s);
            }
            issued++;
            if (++is_b == nbp) {
                is_b = 0;
                is_n++;
                is_row0 += trow;
            }
            is_s = is_s + 1 == S ? 0 : is_s + 1;
        }
    };
#pragma unroll
    for (int q = 0; q < S - 1; q++)
        issue();
    int cs = 0, consumed = 0;
    // give up: the boxes already issued must land before the CTA exits
    auto drain = [&]() {
        if (lane == 0)
            for (int k = consumed, s = cs; k < issued; k++, s = s + 1 == S ? 0 : s + 1) {
                mbar_wait(wbar + 8u * s, (ph >> s) & 1u, 20000000ll);
                ph ^= 1u << s;
            }
        __syncwarp();
    };
    // the first boxes are in flight: every warp past the previous segment, then the tables
    int e = 0;
    if (!jb_sync(jb, jph, lane) || !build_tables(Jsm, sm, threadIdx.x, jb, jph, e)) {
        drain();
        return false;
    }
    float *const y = Jsm.y;
    float *const partials = Jsm.part;
    int *const cnt = Jsm.cnt;
    // this lane's B column: its entries of each block's table, or the zero area
    const uint4 *bcol = L.bnz ? reinterpret_cast<const uint4 *>(sm + kOffBtab) + L.l8
                              : reinterpret_cast<const uint4 *>(sm + kOffZero);
    const int bstep = L.bnz ? 64 : 0;
    const float *xsum = reinterpret_cast<const float *>(sm + kOffXsum);
    const float f = ldexpf(1.f, Q6 ? 24 - e : 24 - 4 * (L.t & 1) - e);
    float acc_a = 0.f, acc_b = 0.f;
    int bi = 0;
    long long row0 = (first >> plog) * 16;
    for (int left = nitems; left > 0;) {
        const bool got = mbar_wait(wbar + 8u * cs, (ph >> cs) & 1u);
        if (!__all_sync(0xffffffffu, got)) {
            drain();
            return false;
        }
        ph ^= 1u << cs;
        consumed++;
        __syncwarp();        // every lane is past the previous block: its stage may be refilled
        issue();
        const unsigned char *st = ring + cs * kStage;
        const int b = b0 + bi;
        if (!Q6) {
            q4_mma_block(st + L.g * kSlot, st + (L.g + 8) * kSlot, bcol + b * bstep, xsum + b * 8, f, L, acc_a,
                         acc_b);
        } else {
            const int mis = (210 * b) & 15;                // the block's offset in its box (same every row)
            if ((mis & 3) == 0)                            // half the blocks: word-aligned, no shifts
                q6_mma_block<true>(st + L.g * kSlot + mis, st + (L.g + 8) * kSlot + mis, bcol + b * bstep,
                                   xsum + b * 16, f, L, acc_a, acc_b);
            else
                q6_mma_block<false>(st + L.g * kSlot + mis, st + (L.g + 8) * kSlot + mis, bcol + b * bstep,
                                    xsum + b * 16, f, L, acc_a, acc_b);
        }
        cs = cs + 1 == S ? 0 : cs + 1;
        if (++bi == nbp) {
            acc_a += __shfl_xor_sync(0xffffffffu, acc_a, 1);
            acc_a += __shfl_xor_sync(0xffffffffu, acc_a, 2);
            acc_b += __shfl_xor_sync(0xffffffffu, acc_b, 1);
            acc_b += __shfl_xor_sync(0xffffffffu, acc_b, 2);
            if (L.t == 0) {
                if (P == 1) {
                    if (row0 + L.g < rows)
                        y[row0 + L.g] = acc_a;
                    if (row0 + L.g + 8 < rows)
                        y[row0 + L.g + 8] = acc_b;
                } else {
                    float *pp = partials + (row0 * P + 16 * part);
                    __stcg(pp + L.g, acc_a);
                    __stcg(pp + L.g + 8, acc_b);
                }
            }
            acc_a = acc_b = 0.f;
            bi = 0;
            row0 += trow;
            left--;
        }
    }
    // split tiles: arrive once the warp's partial stores are issued; the last part of a tile sums
    // the partials in order
    if (P > 1) {
        __syncwarp();        // the partial stores of every lane precede lane 0's release
        long long r0 = (first >> plog) * 16;
        for (int n = 0; n < nitems; n++, r0 += trow) {
            const long long tile = r0 >> 4;
            int last = 0;
            if (lane == 0)
                last = arrive_acq_rel(cnt + tile) == P - 1;
            if (__shfl_sync(0xffffffffu, last, 0)) {   // lane 0's acquire covers the other parts
                if (lane < 16 && r0 + lane < rows) {
                    const float *tp = partials + r0 * P + lane;
                    float v = 0.f;
                    for (int q = 0; q < P; q++)
                        v += __ldcg(tp + 16 * q);
                    y[r0 + lane] = v;
                }
                if (lane == 0)
                    cnt[tile] = 0;
            }
        }
    }
    return true;
}

__global__ void __launch_bounds__(kThreads, 1) quant_matvec_staged_kernel(const __grid_constant__ SParams p)
{
    extern __shared__ __align__(128) unsigned char sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const uint32_t jb = smem_addr(sm + kOffBar);
    SJob *jobs = reinterpret_cast<SJob *>(sm + kOffJobs);
    // the job table into shared memory: one job per warp, uniform parameter reads
    for (int q = warp; q < p.njobs; q += kCWarps) {
        const SJob src = p.jobs[q];
        if (lane == 0)
            jobs[q] = src;
    }
    if (tid < 64)
        reinterpret_cast<uint4 *>(sm + kOffZero)[tid] = make_uint4(0, 0, 0, 0);
    const uint32_t wbar = smem_addr(sm + kOffWBar) + 64u * warp;   // this warp's stage barriers
    if (lane < 8)
        mbar_init(wbar + 8u * lane, 1);
    if (tid == 0)
        mbar_init(jb, kCWarps);
    __syncwarp();
    if (lane == 0)
        mbar_init_fence();
    __syncthreads();
    Lane L;
    L.g = lane >> 2;
    L.t = lane & 3;
    L.bnz = (L.g >> 1) == L.t;
    L.l8 = 2 * L.t + (L.g & 1);
    L.sel = 0x7650u | (uint32_t)L.t;
    unsigned char *ring = sm + warp * kRingBytes;
    uint32_t jph = 0, ph = 0;
    long long t = p.cta_item[blockIdx.x];
    const long long t1 = p.cta_item[blockIdx.x + 1];
    while (t < t1) {
        const int j = item_job(jobs, p.njobs, t);
        const SJob &J = jobs[j];
        const long long jend = j + 1 < p.njobs ? jobs[j + 1].item0 : p.items;
        const long long send = min(t1, jend);
        const bool ok = J.is_q6
            ? run_segment<kQ6Stages, true>(J, t - J.item0, send - J.item0, sm, ring, wbar, ph, jb, jph, L, warp, lane)
            : run_segment<kQ4Stages, false>(J, t - J.item0, send - J.item0, sm, ring, wbar, ph, jb, jph, L, warp,
                                            lane);
        if (!ok) {
            if (tid == 0)
                atomicOr(p.err, kErrWaitTimeout);
            return;
        }
        t = send;
    }
}

// ---------------------------------------------------------------- row kernel (global memory)

// Scale and min j (0..7) of a Q4_K block from its 12 scale bytes held as three words.
__device__ __forceinline__ void q4_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j, float &sc, float &mn)
{
    const int k = (j & 3) * 8;
    const uint32_t a = (s0 >> k) & 0xFFu, b = (s1 >> k) & 0xFFu, c = (s2 >> k) & 0xFFu;
    if (j < 4) {
        sc = (float)(a & 63u);
        mn = (float)(b & 63u);
    } else {
        sc = (float)((c & 0x0Fu) | ((a >> 6) << 4));
        mn = (float)((c >> 4) | ((b >> 6) << 4));
    }
}

__device__ __forceinline__ float q4_row(const unsigned char *w, const float *x, int nb, int lane)
{
    const int g = lane >> 3, i0 = (lane & 7) * 4;
    float acc = 0.f;
#pragma unroll 4
    for (int b = 0; b < nb; b++) {
        const unsigned char *blk = w + (size_t)b * 144;
        const uint4 hdr = __ldg(reinterpret_cast<const uint4 *>(blk));
        const uint32_t qw = __ldg(reinterpret_cast<const uint32_t *>(blk + 16) + lane);
        const float4 xl = __ldg(reinterpret_cast<const float4 *>(x + b * 256 + 64 * g + i0));
        const float4 xh = __ldg(reinterpret_cast<const float4 *>(x + b * 256 + 64 * g + 32 + i0));
        const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFF)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
        float sc0, m0, sc1, m1;
        q4_scale_min(hdr.y, hdr.z, hdr.w, 2 * g, sc0, m0);
        q4_scale_min(hdr.y, hdr.z, hdr.w, 2 * g + 1, sc1, m1);
        const float ql0 = (float)(qw & 15), ql1 = (float)((qw >> 8) & 15);
        const float ql2 = (float)((qw >> 16) & 15), ql3 = (float)((qw >> 24) & 15);
        const float qh0 = (float)((qw >> 4) & 15), qh1 = (float)((qw >> 12) & 15);
        const float qh2 = (float)((qw >> 20) & 15), qh3 = (float)(qw >> 28);
        const float dl = fmaf(ql3, xl.w, fmaf(ql2, xl.z, fmaf(ql1, xl.y, ql0 * xl.x)));
        const float dh = fmaf(qh3, xh.w, fmaf(qh2, xh.z, fmaf(qh1, xh.y, qh0 * xh.x)));
        const float sl = (xl.x + xl.y) + (xl.z + xl.w), sh = (xh.x + xh.y) + (xh.z + xh.w);
        acc = fmaf(d * sc0, dl, acc);
        acc = fmaf(-dmin * m0, sl, acc);
        acc = fmaf(d * sc1, dh, acc);
        acc = fmaf(-dmin * m1, sh, acc);
    }
    return acc;
}

__device__ __forceinline__ float q6_row(const unsigned char *w, const float *x, int nb, int lane)
{
    const int hs = lane >> 4;
    float acc = 0.f;
#pragma unroll 2
    for (int b = 0; b < nb; b++) {
        const unsigned char *blk = w + (size_t)b * 210;
        const float d = __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short *>(blk + 208))));
        const signed char *sc = reinterpret_cast<const signed char *>(blk + 192);
        const float *xb = x + b * 256;
        float part = 0.f;
#pragma unroll
        for (int n = 0; n < 2; n++) {
            const int a = __ldg(blk + 64 * n + lane), c = __ldg(blk + 64 * n + 32 + lane);
            const int h = __ldg(blk + 128 + 32 * n + lane);
            const int q1 = ((a & 15) | ((h & 3) << 4)) - 32;
            const int q2 = ((c & 15) | (((h >> 2) & 3) << 4)) - 32;
            const int q3 = ((a >> 4) | (((h >> 4) & 3) << 4)) - 32;
            const int q4 = ((c >> 4) | (((h >> 6) & 3) << 4)) - 32;
            const int is = 8 * n + hs;
            const float x1 = __ldg(xb + 128 * n + lane), x2 = __ldg(xb + 128 * n + 32 + lane);
            const float x3 = __ldg(xb + 128 * n + 64 + lane), x4 = __ldg(xb + 128 * n + 96 + lane);
            part = fmaf((float)(__ldg(sc + is) * q1), x1, part);
            part = fmaf((float)(__ldg(sc + is + 2) * q2), x2, part);
            part = fmaf((float)(__ldg(sc + is + 4) * q3), x3, part);
            part = fmaf((float)(__ldg(sc + is + 6) * q4), x4, part);
        }
        acc = fmaf(d, part, acc);
    }
    return acc;
}

constexpr int kRowWarps = 8;
constexpr int kRowsPerWarp = 2;

__global__ void __launch_bounds__(kRowWarps * 32) quant_matvec_row_kernel(const __grid_constant__ DParams p)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long base = ((long long)blockIdx.x * kRowWarps + warp) * kRowsPerWarp;
#pragma unroll 1
    for (int rr = 0; rr < kRowsPerWarp; rr++) {
        const long long grow = base + rr;
        if (grow >= p.drows)
            return;
        int lo = 0, hi = p.njobs - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (p.jobs[mid].drow0 <= grow)
                lo = mid;
            else
                hi = mid - 1;
        }
        const DJob &J = p.jobs[lo];
        const long long r = grow - J.drow0;
        float acc;
        if (J.is_q6)
            acc = q6_row(J.w + (size_t)r * J.nb * 210, J.x, J.nb, lane);
        else
            acc = q4_row(J.w + (size_t)r * J.nb * 144, J.x, J.nb, lane);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0)
            J.y[r] = acc;
    }
}

// ---------------------------------------------------------------- multi-token (prefill) kernel
//
// Y[t][r] = W[r] . X[t] for T tokens. The products run on the warp MMA with the scales folded
// into A, so B carries four tokens x (hi, lo) in its eight columns:
//   Q4_K: A = sc_j q 2^-24 (exact f16 subnormals: sc q <= 945; a high nibble, ANDed in place, is
//         q 2^-20 and is multiplied by sc / 16), one fp32 accumulator per block and token scaled
//         by d; the min term runs as one more MMA per block, A = m_j (f16 integers) against the
//         tokens' sub-block sums.
//   Q6_K: A = (q - 32) sc 2^-24 as two exact MMAs per 16 weights, sc = 2 s' + r: A1 = (q-32) 2s'
//         2^-24 (even integers up to 4096) and A2 = (q-32) r 2^-24.
// A CTA takes 256 rows (16 warps x a 16-row tile) and 32 tokens; all warps walk the blocks
// together through two shared-memory stages, each holding the block's 16 weight boxes (the
// matrix's tensor map) and its B fragments (prepared once per call by quant_mm_prep_kernel:
// each token's activation scaled by its own 2^e and split f16 hi + lo, in fragment order).

constexpr int kMmRows = 256;                     // rows per CTA
constexpr int kMmMaxNb = 128;                    // up to 32768 weights a row
constexpr int kMmTok = 32;                       // tokens per CTA (8 groups of 4)
constexpr int kMmBfBytes = 8 * 16 * 32 * 8;      // B fragments of one block: [group][mma][lane] uint2
constexpr int kMmBmBytes = 8 * 32 * 8;           // min-term B fragments: [group][lane] uint2
constexpr int kMmStageW = 16 * 16 * kQ6Slot;     // 16 boxes of 16 rows x slot (Q6_K size)
constexpr int kMmStage = kMmStageW + kMmBfBytes + kMmBmBytes;
constexpr int kMmSmem = 2 * kMmStage + 64;
static_assert(kMmSmem <= 232448, "matmul exceeds the shared memory of a CTA");
static_assert(kMmStage % 128 == 0 && kMmStageW % 128 == 0, "matmul stage alignment");

struct MJob {
    const CUtensorMap *map;      // the matrix (box slot x 16 rows)
    const uint2 *bf;             // B fragments of X: [chunk][block][group][mma][lane]
    const uint2 *bm;             // min-term fragments: [chunk][block][group][lane]
    const int *e;                // per token: activation scale exponent
    float *y;                    // [T][rows]
    float *part;                 // split jobs: unscaled partial products [P][T][rows]
    long long item0;             // first CTA item of the job
    int rows, nb, T, is_q6, rgroups, chunks, P;   // CTAs along the rows, token chunks, block parts
};

struct MParams {
    MJob jobs[kMaxJobs];
    int njobs;
    long long items;
    unsigned *err;
};

// The activations of one call: each distinct X with its fragment buffers.
struct PJob {
    const float *X;
    uint2 *bf, *bm;
    int *e;
    int T, cols, cta0;           // cta0: first CTA of this X (one CTA per padded token)
};

struct PParams {
    PJob jobs[kMaxJobs];
    int njobs;
};

// Per padded token (one CTA each): the activation's scale exponent and its B fragments.
__global__ void __launch_bounds__(256) quant_mm_prep_kernel(const __grid_constant__ PParams pp)
{
    __shared__ float red[8];
    __shared__ float xs[8 * kMmMaxNb];             // sub-block sums, scaled by 2^(e-5) to stay in f16 range
    int jx = 0;
    while (jx + 1 < pp.njobs && pp.jobs[jx + 1].cta0 <= (int)blockIdx.x)
        jx++;
    const PJob &P = pp.jobs[jx];
    const float *X = P.X;
    uint2 *bf = P.bf, *bm = P.bm;
    int *eout = P.e;
    const int T = P.T, cols = P.cols;
    const int tok = blockIdx.x - P.cta0, nb = cols / 256;
    const bool real = tok < T;
    const float *x = X + (size_t)(real ? tok : 0) * cols;
    float mx = 0.f;
    if (real)
        for (int i = threadIdx.x; i < cols / 4; i += 256) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(x) + i);
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0)
        red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int i = 1; i < 8; i++)
        mx = fmaxf(mx, red[i]);
    int E = 0;
    if (mx > 0.f && mx < 3.0e38f)
        frexpf(mx, &E);
    const int e = max(-100, min(100, 14 - E));
    const float scale = ldexpf(1.f, e);
    if (threadIdx.x == 0 && real)
        eout[tok] = e;
    for (int i = threadIdx.x; i < nb * 8; i += 256) {
        float acc = 0.f;
        if (real) {
            const float4 *xp = reinterpret_cast<const float4 *>(x + 32 * i);
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const float4 v = __ldg(xp + k);
                acc += (v.x + v.y) + (v.z + v.w);
            }
        }
        xs[i] = acc * scale * 0x1p-5f;
    }
    __syncthreads();
    const int c = tok / kMmTok, grp = (tok % kMmTok) / 4, tg = tok & 3;
    auto hl = [](float v, int lo) -> uint32_t {
        const __half h = __float2half_rn(v);
        return (uint32_t)__half_as_ushort(lo ? __float2half_rn(v - __half2float(h)) : h);
    };
    // B fragments: lane 8 tg + 4 hl + t holds, for MMA s of block b, weights 16 s + 4 t + {0,2} (b0)
    // and {1,3} (b1) of this token, hi or lo
    for (int q = threadIdx.x; q < nb * 16 * 8; q += 256) {
        const int b = q / 128, s = (q / 8) % 16, lo = (q / 4) & 1, t = q & 3;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (real) {
            const float4 a = __ldg(reinterpret_cast<const float4 *>(x + 256 * b + 16 * s + 4 * t));
            v[0] = a.x * scale; v[1] = a.y * scale; v[2] = a.z * scale; v[3] = a.w * scale;
        }
        const int lane = 8 * tg + 4 * lo + t;
        bf[((((size_t)c * nb + b) * 8 + grp) * 16 + s) * 32 + lane] =
            make_uint2(hl(v[0], lo) | (hl(v[2], lo) << 16), hl(v[1], lo) | (hl(v[3], lo) << 16));
    }
    // min-term fragments: k-slots 2t, 2t+1 hold sub-blocks 2t, 2t+1
    for (int q = threadIdx.x; q < nb * 8; q += 256) {
        const int b = q / 8, lo = (q / 4) & 1, t = q & 3;
        const int lane = 8 * tg + 4 * lo + t;
        bm[(((size_t)c * nb + b) * 8 + grp) * 32 + lane] =
            make_uint2(hl(xs[8 * b + 2 * t], lo) | (hl(xs[8 * b + 2 * t + 1], lo) << 16), 0u);
    }
}

__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b)
{
    const __half2 r = __hmul2(*reinterpret_cast<const __half2 *>(&a), *reinterpret_cast<const __half2 *>(&b));
    return *reinterpret_cast<const uint32_t *>(&r);
}

__device__ __forceinline__ uint32_t hsub2u(uint32_t a, uint32_t b)
{
    const __half2 r = __hsub2(*reinterpret_cast<const __half2 *>(&a), *reinterpret_cast<const __half2 *>(&b));
    return *reinterpret_cast<const uint32_t *>(&r);
}

// (v, v) as an f16 pair for the byte `sel` of a word (a small non-negative integer): the byte
// under the exponent of 1024, less 1024.
__device__ __forceinline__ uint32_t byte_pair_f16(uint32_t w, uint32_t k)
{
    const uint32_t sel = 0x4040u | (k << 8) | k;     // [b_k, 0x64, b_k, 0x64]
    return hsub2u(__byte_perm(w, 0x64646464u, sel), 0x64006400u);
}

// Multiply the warp's 16-row tile by one block for the CTA's 32 tokens. The 16 MMA slices of the
// block run in the outer loop and the 8 token groups in the inner one, each group on its own
// accumulator (d scales the whole block), so a warp keeps 8 independent MMA chains in flight.
// acc[grp][0/1]: rows g, g+8.
__device__ __forceinline__ void mm_q4_block(const unsigned char *pa, const unsigned char *pb, const uint2 *bf,
                                            const uint2 *bmn, const Lane &L, int lane, float (&acc)[8][2])
{
    const uint4 ha = lds128(pa), hb = lds128(pb);
    const float2 da = __half22float2(*reinterpret_cast<const __half2 *>(&ha.x));
    const float2 db = __half22float2(*reinterpret_cast<const __half2 *>(&hb.x));
    // 6-bit scales and mins as bytes: j 0..3 in *l, 4..7 in *h (q4_k_get_scales)
    const uint32_t scla = ha.y & 0x3F3F3F3Fu, scha = (ha.w & 0x0F0F0F0Fu) | ((ha.y >> 2) & 0x30303030u);
    const uint32_t mnla = ha.z & 0x3F3F3F3Fu, mnha = ((ha.w >> 4) & 0x0F0F0F0Fu) | ((ha.z >> 2) & 0x30303030u);
    const uint32_t sclb = hb.y & 0x3F3F3F3Fu, schb = (hb.w & 0x0F0F0F0Fu) | ((hb.y >> 2) & 0x30303030u);
    const uint32_t mnlb = hb.z & 0x3F3F3F3Fu, mnhb = ((hb.w >> 4) & 0x0F0F0F0Fu) | ((hb.z >> 2) & 0x30303030u);
    const uint32_t sixteenth = 0x2C002C00u;          // (1/16, 1/16)
    float c[8][4];
#pragma unroll
    for (int grp = 0; grp < 8; grp++)
        c[grp][0] = c[grp][1] = c[grp][2] = c[grp][3] = 0.f;
#pragma unroll
    for (int s = 0; s < 16; s++) {
        const int j = s >> 1, e = s & 1, G = j >> 1, H = j & 1;
        uint32_t sa = byte_pair_f16(j < 4 ? scla : scha, j & 3), sb = byte_pair_f16(j < 4 ? sclb : schb, j & 3);
        if (H) {
            sa = hmul2u(sa, sixteenth);
            sb = hmul2u(sb, sixteenth);
        }
        const uint32_t mask = H ? 0x00F000F0u : 0x000F000Fu;
        const uint32_t wa = lds32(pa + 16 + 32 * G + 16 * e + 4 * L.t), wb = lds32(pb + 16 + 32 * G + 16 * e + 4 * L.t);
        const uint32_t a0 = hmul2u(wa & mask, sa), a1 = hmul2u(wb & mask, sb);
        const uint32_t a2 = hmul2u((wa >> 8) & mask, sa), a3 = hmul2u((wb >> 8) & mask, sb);
        const uint2 *bs = bf + s * 32 + lane;
#pragma unroll
        for (int grp = 0; grp < 8; grp++) {
            const uint2 bb = bs[grp * 16 * 32];
            mma16816(c[grp], a0, a1, a2, a3, bb.x, bb.y);
        }
    }
    // min term: A = (m_2t, m_2t+1) of rows g and g + 8 against the sub-block sums (2^-5 of them)
    const uint32_t ka = 2 * (L.t & 1);
    const uint32_t mwa = L.t < 2 ? mnla : mnha, mwb = L.t < 2 ? mnlb : mnhb;
    const uint32_t sel_m = 0x4040u | ((ka + 1) << 8) | ka;
    const uint32_t ama = hsub2u(__byte_perm(mwa, 0x64646464u, sel_m), 0x64006400u);
    const uint32_t amb = hsub2u(__byte_perm(mwb, 0x64646464u, sel_m), 0x64006400u);
    const float das = da.x * 0x1p24f, dbs = db.x * 0x1p24f;
    const float dma = da.y * 32.f, dmb = db.y * 32.f;
#pragma unroll
    for (int grp = 0; grp < 8; grp++) {
        float m[4] = {0.f, 0.f, 0.f, 0.f};
        const uint2 bb = bmn[grp * 32 + lane];
        mma16816(m, ama, amb, 0u, 0u, bb.x, bb.y);
        acc[grp][0] += fmaf(das, c[grp][0] + c[grp][1], -dma * (m[0] + m[1]));
        acc[grp][1] += fmaf(dbs, c[grp][2] + c[grp][3], -dmb * (m[2] + m[3]));
    }
}

// One logical word at byte offset `off` of a Q6_K block starting at `bp` (any even address).
__device__ __forceinline__ uint32_t q6_word(const unsigned char *bp, int off)
{
    const unsigned char *a = bp + off;
    const unsigned char *al = reinterpret_cast<const unsigned char *>(reinterpret_cast<uintptr_t>(a) & ~(uintptr_t)3);
    return __funnelshift_r(lds32(al), lds32(al + 4), 8u * (uint32_t)(reinterpret_cast<uintptr_t>(a) & 3));
}

// Q6_K: `pa`, `pb` point at the block in its box (offset (210 b) & 15, the same on every row).
// Slices outer, token groups inner, as for Q4_K.
__device__ __forceinline__ void mm_q6_block(const unsigned char *pa, const unsigned char *pb, const uint2 *bf,
                                            const Lane &L, int lane, float (&acc)[8][2])
{
    const float da = __half2float(*reinterpret_cast<const __half *>(pa + 208)) * 0x1p24f;
    const float db = __half2float(*reinterpret_cast<const __half *>(pb + 208)) * 0x1p24f;
    const uint32_t off32 = 0x00200020u;              // (32 2^-24, 32 2^-24) as f16 subnormals
    float c[8][4];
#pragma unroll
    for (int grp = 0; grp < 8; grp++)
        c[grp][0] = c[grp][1] = c[grp][2] = c[grp][3] = 0.f;
#pragma unroll
    for (int s = 0; s < 16; s++) {
        const int n = s >> 3, q = (s >> 1) & 3, h = s & 1;
        // scale s: sc = 2 s' + r as f16 pairs (2 s', 2 s') and (r, r)
        const int sca = *reinterpret_cast<const signed char *>(pa + 192 + s);
        const int scb = *reinterpret_cast<const signed char *>(pb + 192 + s);
        const uint32_t ea = __half_as_ushort(__short2half_rn((short)(sca & ~1)));
        const uint32_t eb = __half_as_ushort(__short2half_rn((short)(scb & ~1)));
        const uint32_t ra = (sca & 1) ? 0x3C003C00u : 0u, rbq = (scb & 1) ? 0x3C003C00u : 0u;
        const uint32_t la = q6_word(pa, 64 * n + 32 * (q & 1) + 16 * h + 4 * L.t);
        const uint32_t lb = q6_word(pb, 64 * n + 32 * (q & 1) + 16 * h + 4 * L.t);
        const uint32_t qa = q6_word(pa, 128 + 32 * n + 16 * h + 4 * L.t);
        const uint32_t qb = q6_word(pb, 128 + 32 * n + 16 * h + 4 * L.t);
        const uint32_t Qa = ((la >> (4 * (q >> 1))) & 0x0F0F0F0Fu) | (((qa >> (2 * q)) << 4) & 0x30303030u);
        const uint32_t Qb = ((lb >> (4 * (q >> 1))) & 0x0F0F0F0Fu) | (((qb >> (2 * q)) << 4) & 0x30303030u);
        const uint32_t v0a = hsub2u(Qa & 0x003F003Fu, off32), v1a = hsub2u((Qa >> 8) & 0x003F003Fu, off32);
        const uint32_t v0b = hsub2u(Qb & 0x003F003Fu, off32), v1b = hsub2u((Qb >> 8) & 0x003F003Fu, off32);
        const uint32_t s2a = ea | (ea << 16), s2b = eb | (eb << 16);
        const uint32_t x0 = hmul2u(v0a, s2a), x1 = hmul2u(v0b, s2b), x2 = hmul2u(v1a, s2a), x3 = hmul2u(v1b, s2b);
        const uint32_t y0 = hmul2u(v0a, ra), y1 = hmul2u(v0b, rbq), y2 = hmul2u(v1a, ra), y3 = hmul2u(v1b, rbq);
        const uint2 *bs = bf + s * 32 + lane;
#pragma unroll
        for (int grp = 0; grp < 8; grp++) {
            const uint2 bb = bs[grp * 16 * 32];
            mma16816(c[grp], x0, x1, x2, x3, bb.x, bb.y);
            mma16816(c[grp], y0, y1, y2, y3, bb.x, bb.y);
        }
    }
#pragma unroll
    for (int grp = 0; grp < 8; grp++) {
        acc[grp][0] = fmaf(da, c[grp][0] + c[grp][1], acc[grp][0]);
        acc[grp][1] = fmaf(db, c[grp][2] + c[grp][3], acc[grp][1]);
    }
}

__device__ __forceinline__ int mm_item_job(const MParams &p, long long u)
{
    int lo = 0, hi = p.njobs - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (p.jobs[mid].item0 <= u)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

__global__ void __launch_bounds__(kThreads, 1) quant_matmul_kernel(const __grid_constant__ MParams p)
{
    extern __shared__ __align__(128) unsigned char sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const uint32_t full = smem_addr(sm + 2 * kMmStage);   // full[s] = full + 8 s
    const int j = mm_item_job(p, blockIdx.x);
    const MJob J = p.jobs[j];
    const long long it = blockIdx.x - J.item0;
    const int rg = (int)(it % J.rgroups), ch = (int)((it / J.rgroups) % J.chunks);
    const int part = (int)(it / ((long long)J.rgroups * J.chunks));
    const int slot = J.is_q6 ? kQ6Slot : kQ4Slot;
    // this CTA's blocks: b0 .. b0 + nb - 1, part `part` of P near-equal ranges
    const int b0 = (int)((long long)part * J.nb / J.P);
    const int nb = (int)((long long)(part + 1) * J.nb / J.P) - b0;
    if (tid < 2)
        mbar_init(full + 8u * tid, 1);
    __syncwarp();
    if (tid == 0)
        mbar_init_fence();
    __syncthreads();
    // stage s: 16 weight boxes, then the block's B fragments and min-term fragments
    auto issue = [&](int bi, int s) {
        const int b = b0 + bi;
        const uint32_t st = smem_addr(sm + s * kMmStage);
        if (lane == 0)
            mbar_arrive_expect_tx(full + 8u * s, (uint32_t)(16 * 16 * slot + kMmBfBytes + kMmBmBytes));
        __syncwarp();
        if (lane < 16) {
            const int x = J.is_q6 ? (210 * b) & ~15 : 144 * b;
            tma_load_2d(st + lane * 16 * slot, J.map, x, rg * kMmRows + 16 * lane, full + 8u * s);
        } else if (lane == 16) {
            const size_t f = (size_t)ch * J.nb + b;
            bulk_g2s(st + kMmStageW, J.bf + f * (kMmBfBytes / 8), kMmBfBytes, full + 8u * s);
            bulk_g2s(st + kMmStageW + kMmBfBytes, J.bm + f * (kMmBmBytes / 8), kMmBmBytes, full + 8u * s);
        }
    };
    if (warp == 0) {
        issue(0, 0);
        if (nb > 1)
            issue(1, 1);
    }
    Lane L;
    L.g = lane >> 2;
    L.t = lane & 3;
    float acc[8][2];
#pragma unroll
    for (int g = 0; g < 8; g++)
        acc[g][0] = acc[g][1] = 0.f;
    int bi = 0;
    for (; bi < nb; bi++) {
        const int s = bi & 1;
        const bool got = mbar_wait(full + 8u * s, (uint32_t)((bi >> 1) & 1));
        if (!bar_all(1, kThreads, got))
            break;
        const unsigned char *st = sm + s * kMmStage;
        const unsigned char *pa = st + (warp * 16 + L.g) * slot, *pb = pa + 8 * slot;
        const uint2 *bf = reinterpret_cast<const uint2 *>(st + kMmStageW);
        const uint2 *bmn = reinterpret_cast<const uint2 *>(st + kMmStageW + kMmBfBytes);
        if (J.is_q6) {
            const int mis = (210 * (b0 + bi)) & 15;
            mm_q6_block(pa + mis, pb + mis, bf, L, lane, acc);
        } else {
            mm_q4_block(pa, pb, bf, bmn, L, lane, acc);
        }
        named_bar_sync(2, kThreads);     // every warp is done with stage s
        if (warp == 0 && bi + 2 < nb) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(bi + 2, s);
        }
    }
    if (bi < nb) {
        // a wait ran out: record it and let the copies already issued land before exiting
        if (tid == 0) {
            atomicOr(p.err, kErrWaitTimeout);
            for (int k = bi; k < bi + 2 && k < nb; k++)
                mbar_wait(full + 8u * (k & 1), (uint32_t)((k >> 1) & 1), 20000000ll);
        }
        return;
    }
    // acc[grp] of lane (g, t): token 4 grp + t, rows g and g + 8 of the warp's tile
    const int r0 = rg * kMmRows + warp * 16 + L.g;
    float *out = J.P > 1 ? J.part + (size_t)part * J.T * J.rows : J.y;
#pragma unroll
    for (int grp = 0; grp < 8; grp++) {
        const int tok = ch * kMmTok + 4 * grp + L.t;
        if (tok < J.T) {
            const float f = J.P > 1 ? 1.f : ldexpf(1.f, -J.e[tok]);
            if (r0 < J.rows)
                out[(size_t)tok * J.rows + r0] = acc[grp][0] * f;
            if (r0 + 8 < J.rows)
                out[(size_t)tok * J.rows + r0 + 8] = acc[grp][1] * f;
        }
    }
}

// Split jobs: Y[t][r] = 2^-e_t (part 0 + part 1 + ... + part P-1), summed in part order.
struct RJob {
    const float *part;
    float *y;
    const int *e;
    long long n0;                // first element of the job in the launch
    int rows, T, P;
    int yr0;                     // >= 0: token t's result row is p.yr[yr0 + t]
};

struct RParams {
    RJob jobs[kMaxJobs];
    int njobs;
    long long n;
    float *yr[kRowTab];
};

__global__ void __launch_bounds__(256) quant_mm_reduce_kernel(const __grid_constant__ RParams p)
{
    griddep_wait();                 // launched as a dependent of the matmul that wrote the planes
    for (long long u = blockIdx.x * 256ll + threadIdx.x; u < p.n; u += (long long)gridDim.x * 256) {
        int lo = 0, hi = p.njobs - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (p.jobs[mid].n0 <= u)
                lo = mid;
            else
                hi = mid - 1;
        }
        const RJob &J = p.jobs[lo];
        const long long i = u - J.n0, plane = (long long)J.T * J.rows;
        float v = 0.f;
        for (int q = 0; q < J.P; q++)
            v += __ldcs(J.part + q * plane + i);
        const long long t = i / J.rows;
        float *y = J.yr0 >= 0 ? p.yr[J.yr0 + t] + (i - t * J.rows) : J.y + i;
        *y = v * ldexpf(1.f, -J.e[t]);
    }
}

// ---------------------------------------------------------------- multi-token kernel on tcgen05
//
// Y[t] = W X[t] for 64 or more tokens on the 5th-generation tensor cores. A CTA computes 128 rows
// x 64 tokens: D (128 x 128 fp32 in tensor memory) = A (128 rows x K, f16) B^T, B = the 64
// tokens' activations scaled by 2^e_t and split f16 hi (B rows 0-63) + lo (rows 64-127), one
// accumulator per 256-weight block (two in turn), so the block's d -- and the Q4_K min term --
// apply when the block is read back.
//  * 8 decode warps build A a quarter block (64 weights) at a time straight into tensor memory
//    (one row per TMEM lane, f16 pairs; A never touches shared memory, whose bandwidth the B
//    tiles need), with the scales folded in exactly: Q4_K sc q 2^-24; Q6_K two tiles (q - 32) 2s'
//    2^-24 and (q - 32) r 2^-24 (sc = 2s' + r). They also write each row's (d, dmin) and, for
//    Q4_K, an A operand of the mins m_j (f16 integers, K = 16).
//  * One warp issues the copies: the raw blocks of the 128 rows (tensor-map box), B quarter
//    tiles and the Q4_K sub-block sums (bulk copies of images quant_mm_tc_prep_kernel made).
//  * One thread issues the MMAs (M = N = 128, K = 16, A from tensor memory): 4 per quarter block
//    (Q6_K 8), and for Q4_K one more per block into a second accumulator, mins against the
//    sub-block sums (shared memory).
//  * 8 epilogue warps (two per TMEM lane quarter, 32 tokens each) keep
//    y += d (hi + lo) - dmin (min hi + min lo) in registers; 2^-e_t at the end.
// Every hand-off between the roles is an mbarrier with a bounded wait.

namespace tcm {
constexpr int kRows = 128, kTok = 64;
constexpr int kThreads = 576;           // 18 warps: copies, MMA, 8 epilogue, 8 decode
constexpr int kTile = 16384;            // 128 rows x 64 K f16, swizzled
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColMain = 0, kColMin = 256;   // accumulators: main 0 / 128 (by block parity), min 256
constexpr uint32_t kColA = 384;                   // A ring: Q4_K 4 x 32 columns; Q6_K (no min) 4 x 64 at 256
// barrier slots (A ring 4 stages, released through the B ring's barriers; B ring 8; 3 raw buffers)
constexpr int kAFull = 0, kBFull = 8, kBEmpty = 16, kRawFull = 24, kRawEmpty = 27, kMnFullA = 30, kMnFullB = 32,
              kMnEmpty = 34, kAccFull = 36, kAccEmpty = 38, kSclFull = 40, kSclEmpty = 42, kDrain = 44, kSlot = 45;
}  // namespace tcm

template <bool Q6>
struct TcCfg {
    static constexpr int kSlot = Q6 ? kQ6Slot : kQ4Slot;
    static constexpr int kStA = 4;                          // A ring (decoded quarters, in tensor memory): deep
                                                            // enough to cover the MMAs' completion latency
    static constexpr uint32_t kColA = Q6 ? 256u : tcm::kColA;
    static constexpr uint32_t kAcols = Q6 ? 64u : 32u;      // TMEM columns of a decoded quarter
    static constexpr int kStB = 8;                          // B ring (copied quarters: covers the copy latency)
    static constexpr int kOffB = 0;
    static constexpr int kRawN = 2;                         // raw block buffers
    static constexpr int kRaw = 128 * kSlot;
    static constexpr int kOffRaw = kOffB + kStB * tcm::kTile;
    static constexpr int kOffMin = kOffRaw + kRawN * kRaw;
    static constexpr int kMin = Q6 ? 0 : 8192;              // A of the mins 4 KB + sums tile 4 KB
    static constexpr int kOffScl = kOffMin + 2 * kMin;
    static constexpr int kOffBar = kOffScl + 2 * 128 * 8;
    static constexpr int kSmem = kOffBar + 512 + 1024;
    static_assert(kRaw % 1024 == 0, "tile alignment");
    static_assert(kColA + kStA * kAcols <= tcm::kTmemCols, "tensor memory");
    static_assert(kStA < kStB, "the A ring is released through the B ring's barriers");
    static_assert(kStA <= 4 && kStB <= 8 && kRawN <= 3, "barrier slots");
    static_assert(kSmem <= 232448, "shared memory");
};

struct TJob {
    const CUtensorMap *map;     // the matrix, boxes of slot x 128 rows
    const uint4 *bq;            // B quarter tiles [token tile][quarter][16 KB]
    const uint4 *bsum;          // Q4_K sums tiles [token tile][block][4 KB]
    const int *e;               // per token: activation scale exponent
    float *y;                   // [T][rows]: the result, or (raw) this part's unscaled partial plane
    long long item0;
    int rows, nb, T, rtiles, ctiles;
    int kb0, nbt, raw;          // first block of this part, blocks per row, 1 = partial plane
    int yr0;                    // >= 0 (results only): token t's result row is p.yr[yr0 + t]
};

struct TParams {
    TJob jobs[kMaxJobs];
    int njobs;
    long long items;
    unsigned *err;
    float *yr[kRowTab];
};

// The activations of a call for the tensor-core kernel: each distinct X with its images.
struct PJobTc {
    const float *X;
    uint4 *bq, *bsum;
    int *e;
    int T, cols, cta0;
    int xr0;                    // >= 0: token t's activations are pp.xr[xr0 + t]
};

struct PParamsTc {
    PJobTc jobs[kMaxJobs];
    int njobs;
    const float *xr[kRowTab];
};

__device__ __forceinline__ void sts128u(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w)
{
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

// (byte k0, byte k1) of w as an f16 pair of small integers (the byte under the exponent of 1024,
// less 1024).
__device__ __forceinline__ uint32_t f16pair_bytes(uint32_t w, uint32_t k0, uint32_t k1)
{
    return hsub2u(__byte_perm(w, 0x64646464u, 0x4040u | (k1 << 8) | k0), 0x64006400u);
}

__device__ __forceinline__ uint32_t hi_lo_f16(float v, bool lo)
{
    const __half h = __float2half_rn(v);
    return (uint32_t)__half_as_ushort(lo ? __float2half_rn(v - __half2float(h)) : h);
}

// Per padded token (one CTA each): its scale 2^e; its rows of the B quarter tiles (hi at row t,
// lo at row 64 + t of its token tile, 128-byte swizzle); its rows of the Q4_K sums tiles
// (sub-block sums x 2^(e-5), hi / lo, K = 16 with 8 zeros, core matrices of 8 rows x 16 bytes).
__global__ void __launch_bounds__(256) quant_mm_tc_prep_kernel(const __grid_constant__ PParamsTc pp)
{
    __shared__ float red[8];
    // the matmul launch that follows may start now: only its activation copies and its epilogue
    // read what this kernel writes, and they wait for it (griddepcontrol.wait)
    griddep_launch_dependents();
    int jx = 0;
    while (jx + 1 < pp.njobs && pp.jobs[jx + 1].cta0 <= (int)blockIdx.x)
        jx++;
    const PJobTc &P = pp.jobs[jx];
    const int tok = blockIdx.x - P.cta0, T = P.T, cols = P.cols, nq = cols / 64, nb = cols / 256;
    const bool real = tok < T;
    const float *x = P.xr0 >= 0 ? pp.xr[P.xr0 + (real ? tok : 0)] : P.X + (size_t)(real ? tok : 0) * cols;
    float mx = 0.f;
    if (real)
        for (int i = threadIdx.x; i < cols / 4; i += 256) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(x) + i);
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0)
        red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int i = 1; i < 8; i++)
        mx = fmaxf(mx, red[i]);
    int E = 0;
    if (mx > 0.f && mx < 3.0e38f)
        frexpf(mx, &E);
    const int e = max(-100, min(100, 14 - E));
    const float scale = ldexpf(1.f, e);
    if (threadIdx.x == 0 && real)
        P.e[tok] = e;
    const int ct = tok >> 6, tl = tok & 63;
    for (int idx = threadIdx.x; idx < nq * 8; idx += 256) {
        const int g = idx >> 3, u = idx & 7;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (real) {
            const float4 a = __ldg(reinterpret_cast<const float4 *>(x + 64 * g + 8 * u));
            const float4 b = __ldg(reinterpret_cast<const float4 *>(x + 64 * g + 8 * u + 4));
            v[0] = a.x * scale; v[1] = a.y * scale; v[2] = a.z * scale; v[3] = a.w * scale;
            v[4] = b.x * scale; v[5] = b.y * scale; v[6] = b.z * scale; v[7] = b.w * scale;
        }
        uint4 *tile = P.bq + ((size_t)ct * nq + g) * (tcm::kTile / 16);
        const int pos = u ^ (tl & 7);
#pragma unroll
        for (int lo = 0; lo < 2; lo++) {
            uint4 w;
            w.x = hi_lo_f16(v[0], lo) | (hi_lo_f16(v[1], lo) << 16);
            w.y = hi_lo_f16(v[2], lo) | (hi_lo_f16(v[3], lo) << 16);
            w.z = hi_lo_f16(v[4], lo) | (hi_lo_f16(v[5], lo) << 16);
            w.w = hi_lo_f16(v[6], lo) | (hi_lo_f16(v[7], lo) << 16);
            tile[(64 * lo + tl) * 8 + pos] = w;
        }
    }
    if (P.bsum) {
        const float sscale = scale * 0x1p-5f;        // the sums stay inside the f16 range
        for (int b = threadIdx.x; b < nb; b += 256) {
            float sv[8];
#pragma unroll
            for (int jj = 0; jj < 8; jj++) {
                float acc = 0.f;
                if (real) {
                    const float4 *xp = reinterpret_cast<const float4 *>(x + 256 * b + 32 * jj);
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        const float4 q = __ldg(xp + k);
                        acc += (q.x + q.y) + (q.z + q.w);
                    }
                }
                sv[jj] = acc * sscale;
            }
            uint4 *tile = P.bsum + ((size_t)ct * nb + b) * 256;
#pragma unroll
            for (int lo = 0; lo < 2; lo++) {
                const int row = 64 * lo + tl;
                uint4 w;
                w.x = hi_lo_f16(sv[0], lo) | (hi_lo_f16(sv[1], lo) << 16);
                w.y = hi_lo_f16(sv[2], lo) | (hi_lo_f16(sv[3], lo) << 16);
                w.z = hi_lo_f16(sv[4], lo) | (hi_lo_f16(sv[5], lo) << 16);
                w.w = hi_lo_f16(sv[6], lo) | (hi_lo_f16(sv[7], lo) << 16);
                tile[(row >> 3) * 16 + (row & 7)] = w;                       // K 0-7
                tile[(row >> 3) * 16 + 8 + (row & 7)] = make_uint4(0u, 0u, 0u, 0u);   // K 8-15
            }
        }
    }
}

// One CTA's work: tile `item` of the format's job table.
template <bool Q6>
__device__ __forceinline__ void tc_tile(const TParams &p, long long item)
{
    using Cfg = TcCfg<Q6>;
    using namespace tcm;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;
    unsigned char *gb = smem_raw + (base - smem_addr(smem_raw));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int j = 0;
    {
        int lo = 0, hi = p.njobs - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (p.jobs[mid].item0 <= item)
                lo = mid;
            else
                hi = mid - 1;
        }
        j = lo;
    }
    const TJob &J = p.jobs[j];
    const long long it = item - J.item0;
    const int rt = (int)(it % J.rtiles), ct = (int)(it / J.rtiles);
    const int nb = J.nb, nq = 4 * nb, kb0 = J.kb0, nqt = 4 * J.nbt;   // this part's blocks kb0 .. kb0 + nb - 1
    unsigned long long *bars = reinterpret_cast<unsigned long long *>(gb + Cfg::kOffBar);
    auto BAR = [&](int i) -> uint32_t { return smem_addr(&bars[i]); };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(&bars[kSlot]);
    if (tid == 0) {
        for (int s = 0; s < Cfg::kStA; s++)
            mbar_init(BAR(kAFull + s), 8);
        for (int s = 0; s < Cfg::kStB; s++) {
            mbar_init(BAR(kBFull + s), 1);
            mbar_init(BAR(kBEmpty + s), 1);
        }
        for (int r = 0; r < 3; r++) {
            mbar_init(BAR(kRawFull + r), 1);
            mbar_init(BAR(kRawEmpty + r), 8);
        }
        for (int x = 0; x < 2; x++) {
            mbar_init(BAR(kMnFullA + x), 8);
            mbar_init(BAR(kMnFullB + x), 1);
            mbar_init(BAR(kMnEmpty + x), 1);
            mbar_init(BAR(kAccFull + x), 1);
            mbar_init(BAR(kAccEmpty + x), 8);
            mbar_init(BAR(kSclFull + x), 8);
            mbar_init(BAR(kSclEmpty + x), 8);
        }
        mbar_init(BAR(kDrain), 1);
        mbar_init_fence();
    }
    if (warp == 1) {
        tc::tmem_alloc(smem_addr(tmem_slot), kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tb = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        // ============================================================ copies
        // three independent streams, one lane each, so none waits behind another's buffer:
        // lane 0 the B quarter tiles, lane 1 the raw blocks, lane 2 (Q4_K) the sums tiles
        if (lane == 0) {
            griddep_wait();                               // the activation tiles are the prep kernel's
            int nst[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int g = 0; g < nq; g++) {
                const int s = g % Cfg::kStB;
                if (g >= Cfg::kStB && !mbar_wait(BAR(kBEmpty + s), (uint32_t)(g / Cfg::kStB - 1) & 1u)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(BAR(kBFull + s), (uint32_t)kTile);
                bulk_g2s(base + Cfg::kOffB + s * kTile, J.bq + ((size_t)ct * nqt + 4 * kb0 + g) * (kTile / 16),
                         (uint32_t)kTile, BAR(kBFull + s));
                nst[s]++;
            }
            if (!ok)
                atomicOr(p.err, kErrWaitTimeout);
            // every copy issued lands before the CTA ends (a wait on its buffer's last phase)
            for (int s = 0; s < Cfg::kStB; s++)
                if (nst[s])
                    mbar_wait(BAR(kBFull + s), (uint32_t)(nst[s] - 1) & 1u, 20000000ll);
        } else if (lane == 1) {
            const int row0 = rt * kRows;
            int nraw[3] = {0, 0, 0};
            for (int b = 0; b < nb; b++) {
                const int r = b % Cfg::kRawN;
                if (b >= Cfg::kRawN && !mbar_wait(BAR(kRawEmpty + r), (uint32_t)(b / Cfg::kRawN - 1) & 1u)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(BAR(kRawFull + r), (uint32_t)Cfg::kRaw);
                const int x = Q6 ? (210 * (kb0 + b)) & ~15 : 144 * (kb0 + b);
                tma_load_2d(base + Cfg::kOffRaw + r * Cfg::kRaw, J.map, x, row0, BAR(kRawFull + r));
                nraw[r]++;
            }
            if (!ok)
                atomicOr(p.err, kErrWaitTimeout);
            for (int r = 0; r < Cfg::kRawN; r++)
                if (nraw[r])
                    mbar_wait(BAR(kRawFull + r), (uint32_t)(nraw[r] - 1) & 1u, 20000000ll);
        } else if (lane == 2 && !Q6) {
            griddep_wait();                               // so are the sums tiles
            int nsum[2] = {0, 0};
            for (int b = 0; b < nb; b++) {
                if (b >= 2 && !mbar_wait(BAR(kMnEmpty + (b & 1)), (uint32_t)((b >> 1) - 1) & 1u)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(BAR(kMnFullB + (b & 1)), 4096u);
                bulk_g2s(base + Cfg::kOffMin + (b & 1) * Cfg::kMin + 4096, J.bsum + ((size_t)ct * J.nbt + kb0 + b) * 256,
                         4096u, BAR(kMnFullB + (b & 1)));
                nsum[b & 1]++;
            }
            if (!ok)
                atomicOr(p.err, kErrWaitTimeout);
            for (int x = 0; x < 2; x++)
                if (nsum[x])
                    mbar_wait(BAR(kMnFullB + x), (uint32_t)(nsum[x] - 1) & 1u, 20000000ll);
        }
    } else if (warp == 1) {
        // ============================================================ MMA issue
        // One thread; the issue path is kept short (the tensor pipe idles whenever the thread spends
        // longer between quarters than a quarter's MMAs take): with a 4-deep A ring and an 8-deep B
        // ring every slot and parity in a block is a constant or one AND of the block index, and
        // the descriptors are built once.
        static_assert(Cfg::kStA == 4 && Cfg::kStB == 8, "the issue loop's slot arithmetic");
        if (lane == 0) {
            const uint32_t id = tc::idesc_f16(128, 128, 0, 0);
            const uint64_t dB0 = tc::smem_desc(base + Cfg::kOffB, 16, 1024);
            const uint32_t ta0 = tb + Cfg::kColA;
            const uint32_t mb0 = base + Cfg::kOffMin;
            const uint64_t dAm0 = tc::smem_desc_plain(mb0, 128, 256), dBm0 = tc::smem_desc_plain(mb0 + 4096, 128, 256);
            for (int b = 0; b < nb && ok; b++) {
                const uint32_t odd = (uint32_t)(b & 1);
                const uint32_t dmain = tb + kColMain + odd * 128u;
                if (b >= 2 && !mbar_wait(BAR(kAccEmpty + odd), (uint32_t)((b >> 1) - 1) & 1u)) {
                    ok = false;
                    break;
                }
                const uint32_t pa = odd, pb = (uint32_t)(b >> 1) & 1u;   // A / B ring phases of this block
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const uint32_t sb = 4u * odd + (uint32_t)q;          // B slot; the A slot is q
                    if (!mbar_wait(BAR(kAFull + q), pa) || !mbar_wait(BAR(kBFull + sb), pb)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t ta = ta0 + (uint32_t)q * Cfg::kAcols;
                    const uint64_t dB = tc::desc_adv(dB0, sb * (uint32_t)kTile);
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {
                        tc::mma_ts_f16(dmain, ta + 8u * kk, tc::desc_adv(dB, kk * 32u), id, (q | kk) ? 1u : 0u);
                        if (Q6)
                            tc::mma_ts_f16(dmain, ta + 32u + 8u * kk, tc::desc_adv(dB, kk * 32u), id, 1u);
                    }
                    // one commit per quarter frees both its B slot and (quarters complete in order)
                    // its A slot: the decode warps wait on the B-slot barrier of quarter g - kStA
                    tc::commit(BAR(kBEmpty + sb));
                }
                if (!ok)
                    break;
                if (!Q6) {
                    // the min accumulator is single: the epilogue has read block b - 1's
                    if (!mbar_wait(BAR(kMnFullA + odd), pb) || !mbar_wait(BAR(kMnFullB + odd), pb) ||
                        (b >= 1 && !mbar_wait(BAR(kAccEmpty + (odd ^ 1u)), (uint32_t)((b - 1) >> 1) & 1u))) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    tc::mma_ss_f16(tb + kColMin, tc::desc_adv(dAm0, odd * (uint32_t)Cfg::kMin),
                                   tc::desc_adv(dBm0, odd * (uint32_t)Cfg::kMin), id, 0u);
                    tc::commit(BAR(kMnEmpty + odd));
                }
                tc::commit(BAR(kAccFull + odd));
            }
            if (!ok)
                atomicOr(p.err, kErrWaitTimeout);
            // every MMA issued finishes before tensor memory is released
            tc::commit(BAR(kDrain));
            mbar_wait(BAR(kDrain), 0, 20000000ll);
        }
    } else if (warp < 10) {
        // ============================================================ epilogue
        const int qd = warp & 3, half = (warp - 2) >> 2;
        const int r = 32 * qd + lane;
        const uint32_t lq = (uint32_t)(32 * qd) << 16;
        const float2 *scl = reinterpret_cast<const float2 *>(gb + Cfg::kOffScl);
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; i++)
            acc[i] = 0.f;
        for (int b = 0; b < nb && ok; b++) {
            const uint32_t ph = (uint32_t)(b >> 1) & 1u;
            if (!mbar_wait_sleep(BAR(kAccFull + (b & 1)), ph, 32) || !mbar_wait(BAR(kSclFull + (b & 1)), ph)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const float2 sd = scl[(b & 1) * 128 + r];           // (d 2^24, 32 dmin)
            const uint32_t cm = tb + lq + kColMain + (uint32_t)(b & 1) * 128u + 32u * half;
            const uint32_t cn = tb + lq + kColMin + 32u * half;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                float h[8], l[8];
                tc::tmem_ld8(cm + 8 * c, h);
                tc::tmem_ld8(cm + 64 + 8 * c, l);
                if (Q6) {
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 8; i++)
                        acc[8 * c + i] = fmaf(sd.x, h[i] + l[i], acc[8 * c + i]);
                } else {
                    float mh[8], ml[8];
                    tc::tmem_ld8(cn + 8 * c, mh);
                    tc::tmem_ld8(cn + 64 + 8 * c, ml);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 8; i++)
                        acc[8 * c + i] = fmaf(sd.x, h[i] + l[i], fmaf(-sd.y, mh[i] + ml[i], acc[8 * c + i]));
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(BAR(kAccEmpty + (b & 1)));
                mbar_arrive(BAR(kSclEmpty + (b & 1)));
            }
        }
        griddep_wait();                                   // the token exponents are the prep kernel's
        if (ok) {
            const int row = rt * kRows + r;
            if (row < J.rows) {
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const int t = ct * kTok + 32 * half + i;
                    if (t < J.T)
                        (J.yr0 >= 0 ? p.yr[J.yr0 + t] : J.y + (size_t)t * J.rows)[row] =
                            J.raw ? acc[i] : acc[i] * ldexpf(1.f, -J.e[t]);
                }
            }
        } else if (lane == 0) {
            atomicOr(p.err, kErrWaitTimeout);
        }
    } else {
        // ============================================================ decode
        const int dq = tid - 320;                             // 0..255
        float2 *scl = reinterpret_cast<float2 *>(gb + Cfg::kOffScl);
        for (int b = 0; b < nb && ok; b++) {
            const int rr = b % Cfg::kRawN;
            if (!mbar_wait(BAR(kRawFull + rr), (uint32_t)(b / Cfg::kRawN) & 1u)) {
                ok = false;
                break;
            }
            const unsigned char *raw = gb + Cfg::kOffRaw + rr * Cfg::kRaw;
            const int mis = Q6 ? (210 * (kb0 + b)) & 15 : 0;
            // per-row tables of the block
            if (b >= 2) {
                const uint32_t ph = (uint32_t)((b >> 1) - 1) & 1u;
                if (!mbar_wait(BAR(kSclEmpty + (b & 1)), ph) || (!Q6 && !mbar_wait(BAR(kMnEmpty + (b & 1)), ph))) {
                    ok = false;
                    break;
                }
            }
            if (dq < kRows) {
                const unsigned char *blk = raw + dq * Cfg::kSlot + mis;
                if (Q6) {
                    const float d = __half2float(*reinterpret_cast<const __half *>(blk + 208));
                    scl[(b & 1) * 128 + dq] = make_float2(d * 0x1p24f, 0.f);
                } else {
                    const uint4 hd = lds128(blk);
                    const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&hd.x));
                    scl[(b & 1) * 128 + dq] = make_float2(dd.x * 0x1p24f, dd.y * 32.f);
                    // the row's mins m_0..m_7 (q4_k_get_scales) and 8 zeros, K = 16
                    const uint32_t mnl = hd.z & 0x3F3F3F3Fu;
                    const uint32_t mnh = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
                    const uint32_t am = base + Cfg::kOffMin + (uint32_t)(b & 1) * Cfg::kMin + (uint32_t)(dq >> 3) * 256u +
                                        (uint32_t)(dq & 7) * 16u;
                    sts128u(am, f16pair_bytes(mnl, 0, 1), f16pair_bytes(mnl, 2, 3), f16pair_bytes(mnh, 0, 1),
                            f16pair_bytes(mnh, 2, 3));
                    sts128u(am + 128u, 0u, 0u, 0u, 0u);
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(BAR(kSclFull + (b & 1)));
                if (!Q6)
                    mbar_arrive(BAR(kMnFullA + (b & 1)));
            }
            // each thread: the row of its TMEM lane (warp quarter), units 4h .. 4h + 3 of every quarter
            // block (h = which of the quarter's two decode warps), i.e. TMEM columns 16h .. 16h + 15
            const int row = 32 * (warp & 3) + lane, h = (warp - 10) >> 2;
            const unsigned char *rblk = raw + row * Cfg::kSlot + mis;
            const uint32_t tl = tb + ((uint32_t)(32 * (warp & 3)) << 16) + 16u * (uint32_t)h;
            uint32_t s4[4];                                   // Q4_K: the scale pair of each quarter
            if (!Q6) {
                const uint4 hd = lds128(rblk);
                const uint32_t scl4 = hd.y & 0x3F3F3F3Fu, sch4 = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int jj = 2 * q + h;
                    uint32_t s2 = f16pair_bytes(jj < 4 ? scl4 : sch4, (uint32_t)(jj & 3), (uint32_t)(jj & 3));
                    s4[q] = h ? hmul2u(s2, 0x2C002C00u) : s2;   // sc / 16 for the high nibbles
                }
            }
            for (int q = 0; q < 4; q++) {
                const int g = 4 * b + q, s = g % Cfg::kStA, gp = g - Cfg::kStA;   // gp: the slot's previous quarter
                if (g >= Cfg::kStA && !mbar_wait(BAR(kBEmpty + gp % Cfg::kStB), (uint32_t)(gp / Cfg::kStB) & 1u)) {
                    ok = false;
                    break;
                }
                const uint32_t ta = tl + Cfg::kColA + (uint32_t)s * Cfg::kAcols;
                uint32_t w1[16], w2[16];
                if (Q6) {
                    const int n = q >> 1, qq = 2 * (q & 1) + h;
                    // 32 bytes of ql (nibble qq / 2) and of qh (bits 2 qq), from a 2-byte-aligned start
                    uint32_t L[8], Hh[8];
                    {
                        const unsigned char *a = rblk + 64 * n + 32 * (qq & 1);
                        const unsigned char *al = reinterpret_cast<const unsigned char *>(reinterpret_cast<uintptr_t>(a) & ~(uintptr_t)3);
                        const uint32_t sh = 8u * (uint32_t)(reinterpret_cast<uintptr_t>(a) & 3);
                        uint32_t w[9];
#pragma unroll
                        for (int i = 0; i < 9; i++)
                            w[i] = lds32(al + 4 * i);
#pragma unroll
                        for (int i = 0; i < 8; i++)
                            L[i] = __funnelshift_r(w[i], w[i + 1], sh);
                    }
                    {
                        const unsigned char *a = rblk + 128 + 32 * n;
                        const unsigned char *al = reinterpret_cast<const unsigned char *>(reinterpret_cast<uintptr_t>(a) & ~(uintptr_t)3);
                        const uint32_t sh = 8u * (uint32_t)(reinterpret_cast<uintptr_t>(a) & 3);
                        uint32_t w[9];
#pragma unroll
                        for (int i = 0; i < 9; i++)
                            w[i] = lds32(al + 4 * i);
#pragma unroll
                        for (int i = 0; i < 8; i++)
                            Hh[i] = __funnelshift_r(w[i], w[i + 1], sh);
                    }
                    const int ls = 4 * (qq >> 1), hs = 2 * qq;
                    const int scA = *reinterpret_cast<const signed char *>(rblk + 192 + 8 * n + 2 * qq);
                    const int scB = *reinterpret_cast<const signed char *>(rblk + 192 + 8 * n + 2 * qq + 1);
                    const uint32_t off32 = 0x00200020u;          // (32 2^-24, 32 2^-24)
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const int sc = k < 2 ? scA : scB;        // weights 8k .. 8k + 7: scale group k / 2
                        const uint32_t e1 = __half_as_ushort(__short2half_rn((short)(sc & ~1)));
                        const uint32_t s2 = e1 | (e1 << 16), r2 = (sc & 1) ? 0x3C003C00u : 0u;
                        const uint32_t Qx = ((L[2 * k] >> ls) & 0x0F0F0F0Fu) | (((Hh[2 * k] >> hs) << 4) & 0x30303030u);
                        const uint32_t Qy =
                            ((L[2 * k + 1] >> ls) & 0x0F0F0F0Fu) | (((Hh[2 * k + 1] >> hs) << 4) & 0x30303030u);
                        const uint32_t p0 = hsub2u(__byte_perm(Qx, 0u, 0x4140u) & 0x003F003Fu, off32);
                        const uint32_t p1 = hsub2u(__byte_perm(Qx, 0u, 0x4342u) & 0x003F003Fu, off32);
                        const uint32_t p2 = hsub2u(__byte_perm(Qy, 0u, 0x4140u) & 0x003F003Fu, off32);
                        const uint32_t p3 = hsub2u(__byte_perm(Qy, 0u, 0x4342u) & 0x003F003Fu, off32);
                        w1[4 * k] = hmul2u(p0, s2);
                        w1[4 * k + 1] = hmul2u(p1, s2);
                        w1[4 * k + 2] = hmul2u(p2, s2);
                        w1[4 * k + 3] = hmul2u(p3, s2);
                        w2[4 * k] = hmul2u(p0, r2);
                        w2[4 * k + 1] = hmul2u(p1, r2);
                        w2[4 * k + 2] = hmul2u(p2, r2);
                        w2[4 * k + 3] = hmul2u(p3, r2);
                    }
                    tc::tmem_st16(ta, w1);
                    tc::tmem_st16(ta + 32u, w2);
                } else {
                    const uint4 qa = lds128(rblk + 16 + 32 * q), qb = lds128(rblk + 32 + 32 * q);
                    const uint32_t W[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                    const uint32_t mask = h ? 0x00F000F0u : 0x000F000Fu, s2 = s4[q];
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        w1[4 * k] = hmul2u(__byte_perm(W[2 * k], 0u, 0x4140u) & mask, s2);
                        w1[4 * k + 1] = hmul2u(__byte_perm(W[2 * k], 0u, 0x4342u) & mask, s2);
                        w1[4 * k + 2] = hmul2u(__byte_perm(W[2 * k + 1], 0u, 0x4140u) & mask, s2);
                        w1[4 * k + 3] = hmul2u(__byte_perm(W[2 * k + 1], 0u, 0x4342u) & mask, s2);
                    }
                    tc::tmem_st16(ta, w1);
                    (void)w2;
                }
                tc::tmem_wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(BAR(kAFull + s));
            }
            if (!ok)
                break;
            __syncwarp();
            if (lane == 0)
                mbar_arrive(BAR(kRawEmpty + rr));
        }
        if (!ok && lane == 0)
            atomicOr(p.err, kErrWaitTimeout);
    }
    griddep_launch_dependents();                          // this CTA's outputs are written
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 1)
        tc::tmem_dealloc(tb, kTmemCols);
}

// Both formats' tiles in one launch: the Q4_K items first, then the Q6_K items. A call's two
// formats then share the SMs instead of running one after the other, which matters when each
// has fewer tiles than SMs (one layer's projections for a round of slots).
struct TParams2 {
    TParams f[2];               // [0] Q4_K, [1] Q6_K
};

__global__ void __launch_bounds__(tcm::kThreads, 1) quant_mm_tc_kernel(const __grid_constant__ TParams2 p)
{
    const long long b = blockIdx.x;
    if (b < p.f[0].items)
        tc_tile<false>(p.f[0], b);
    else
        tc_tile<true>(p.f[1], b - p.f[0].items);
}

// ---------------------------------------------------------------- host

// Tensor maps of the matrices, cached per device: weights stay resident between calls, so a
// matrix's map is encoded and uploaded once. A map holds only the address and the shape.
constexpr int kMapCap = 4096;

struct MapKey {
    uintptr_t w;
    long long rows;
    int rb, slot, box;                   // box: rows per copy
    bool operator==(const MapKey &o) const
    {
        return w == o.w && rows == o.rows && rb == o.rb && slot == o.slot && box == o.box;
    }
};

struct MapKeyHash {
    size_t operator()(const MapKey &k) const
    {
        return std::hash<uintptr_t>()(k.w) ^ (std::hash<long long>()(k.rows) * 31u) ^ ((size_t)k.rb << 20) ^
               (size_t)k.slot ^ ((size_t)k.box << 12);
    }
};

struct MapCache {
    CUtensorMap *dev = nullptr;          // kMapCap maps in device memory
    std::vector<CUtensorMap> host;       // their host copies (sources of the uploads)
    int used = 0;
    std::unordered_map<MapKey, int, MapKeyHash> idx;
};

MapCache g_maps[64];

const CUtensorMap *job_map(const unsigned char *w, long long rows, int rb, int slot, int box = 16)
{
    Runtime &R = rt();
    if (R.device < 0 || R.device >= 64) {
        fail("kernel_cuda_matvec_quant_batch: device %d out of range", R.device);
        return nullptr;
    }
    MapCache &mc = g_maps[R.device];
    if (!mc.dev) {
        if (check(cudaMalloc(&mc.dev, kMapCap * sizeof(CUtensorMap)), "cudaMalloc(matvec tensor maps)") != 0)
            return nullptr;
        mc.host.resize(kMapCap);
    }
    const MapKey key{reinterpret_cast<uintptr_t>(w), rows, rb, slot, box};
    const auto it = mc.idx.find(key);
    if (it != mc.idx.end())
        return mc.dev + it->second;
    if (mc.used == kMapCap) {
        // full: start over once no queued kernel can still read the old maps
        if (check(cudaStreamSynchronize(R.stream), "cudaStreamSynchronize(matvec tensor maps)") != 0)
            return nullptr;
        mc.idx.clear();
        mc.used = 0;
        R.gen++;                         // recorded work may point to the reused map slots
    }
    const int i = mc.used;
    if (encode_tmap_u8_2d(&mc.host[i], w, (uint64_t)rb, (uint64_t)rows, (uint64_t)rb, (uint32_t)slot, (uint32_t)box) != 0)
        return nullptr;
    if (check(cudaMemcpyAsync(mc.dev + i, &mc.host[i], sizeof(CUtensorMap), cudaMemcpyHostToDevice, R.stream),
              "upload matvec tensor map") != 0)
        return nullptr;
    mc.used++;
    mc.idx.emplace(key, i);
    return mc.dev + i;
}

int matvec_chunk(const KernelCudaMatvecJob *jobs, int n)
{
    static bool attr_set = false;
    SParams sp;
    DParams dp;
    memset(static_cast<void *>(&sp), 0, sizeof(sp));
    memset(static_cast<void *>(&dp), 0, sizeof(dp));
    long long tiles[kMaxJobs];
    long long total_tiles = 0;
    for (int i = 0; i < n; i++) {
        const KernelCudaMatvecJob &j = jobs[i];
        if (!j.matrix || !j.vector || !j.output)
            return fail("kernel_cuda_matvec_quant_batch: job %d has a null pointer", i);
        if (j.cols == 0 || j.cols % 256 != 0 || j.cols > (1u << 24))
            return fail("kernel_cuda_matvec_quant_batch: job %d cols %zu must be a positive multiple of 256", i,
                        j.cols);
        if (!aligned16(j.vector) || (!j.is_q6 && !aligned16(j.matrix)) ||
            (j.is_q6 && (reinterpret_cast<uintptr_t>(j.matrix) & 1)))
            return fail("kernel_cuda_matvec_quant_batch: job %d misaligned (vector 16 B, Q4_K matrix 16 B, "
                        "Q6_K matrix 2 B)", i);
        if (j.rows == 0)
            continue;
        const int nb = (int)(j.cols / 256);
        const long long rb = (long long)nb * (j.is_q6 ? 210 : 144);
        const unsigned char *w = static_cast<const unsigned char *>(j.matrix);
        // staged rows: the matrix as a 2-D byte array needs 16-byte alignment and a row length that
        // is a multiple of 16 bytes (Q6_K: a multiple of 8 blocks)
        long long srows = 0;
        if (aligned16(j.matrix) && nb <= kMaxNb && rb % 16 == 0 && rb <= 0x7FFFFFFF / 16 &&
            (long long)j.rows < 0x7FFFFFFF)
            srows = (long long)j.rows;
        if (srows > 0) {
            tiles[sp.njobs] = (srows + 15) / 16;
            total_tiles += tiles[sp.njobs];
            const CUtensorMap *map = job_map(w, srows, (int)rb, j.is_q6 ? kQ6Slot : kQ4Slot);
            if (!map)
                return -1;
            sp.jobs[sp.njobs++] = SJob{map, w, j.vector, j.output, nullptr, nullptr, 0, srows, nb, j.is_q6 ? 1 : 0, 0};
        }
        if (srows < (long long)j.rows) {
            dp.jobs[dp.njobs++] = DJob{w + srows * rb, j.vector, j.output + srows, dp.drows,
                                       (long long)j.rows - srows, nb, j.is_q6 ? 1 : 0};
            dp.drows += (long long)j.rows - srows;
        }
    }
    Runtime &R = rt();
    if (sp.njobs > 0) {
        if (!attr_set) {
            if (check(cudaFuncSetAttribute(quant_matvec_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kSmemBytes), "matvec shared memory") != 0)
                return -1;
            attr_set = true;
        }
        // split tiles into parts (along the blocks) when there are fewer than two tiles per warp
        const long long warps = (long long)std::min(R.num_sms, kMaxCtas) * kCWarps;
        int want = 1;
        while (want < 16 && total_tiles * want < 2 * warps)
            want <<= 1;
        long long part_floats = 0, ncnt = 0;
        double total = 0.0, item_bytes[kMaxJobs];
        for (int q = 0; q < sp.njobs; q++) {
            SJob &J = sp.jobs[q];
            int plog = 0;
            while ((1 << (plog + 1)) <= want && J.nb % (1 << (plog + 1)) == 0)
                plog++;
            J.plog = plog;
            J.item0 = sp.items;
            sp.items += tiles[q] << plog;
            // cost of an item: its bytes, Q6_K weighted by its slower multiply (about 2x per byte)
            item_bytes[q] = 16.0 * J.nb * (J.is_q6 ? 210 * 2.0 : 144) / (1 << plog);
            total += item_bytes[q] * (double)(tiles[q] << plog);
            if (plog > 0) {
                part_floats += (tiles[q] << plog) * 16;
                ncnt += tiles[q];
            }
        }
        if (ncnt > 0) {
            float *part = static_cast<float *>(scratch((size_t)part_floats * sizeof(float)));
            int *cnt = counters((size_t)ncnt);
            if (!part || !cnt)
                return -1;
            for (int q = 0; q < sp.njobs; q++)
                if (sp.jobs[q].plog > 0) {
                    sp.jobs[q].part = part;
                    sp.jobs[q].cnt = cnt;
                    part += (tiles[q] << sp.jobs[q].plog) * 16;
                    cnt += tiles[q];
                }
        }
        // contiguous item ranges of about equal cost per CTA
        const int G = (int)std::min<long long>(std::min(R.num_sms, kMaxCtas), sp.items);
        for (int c = 0; c < G; c++) {
            const double target = total * c / G;
            long long idx = sp.items;
            double cum = 0.0;
            for (int q = 0; q < sp.njobs; q++) {
                const long long ni = (q + 1 < sp.njobs ? sp.jobs[q + 1].item0 : sp.items) - sp.jobs[q].item0;
                const double jb = item_bytes[q] * (double)ni;
                if (target < cum + jb) {
                    idx = sp.jobs[q].item0 + (long long)((target - cum) / item_bytes[q]);
                    break;
                }
                cum += jb;
            }
            sp.cta_item[c] = c == 0 ? 0 : std::max(idx, sp.cta_item[c - 1]);
        }
        sp.cta_item[G] = sp.items;
        sp.err = R.err_word;
        quant_matvec_staged_kernel<<<(unsigned)G, kThreads, kSmemBytes, R.stream>>>(sp);
        if (launched("quant_matvec_staged_kernel") != 0)
            return -1;
    }
    if (dp.drows > 0) {
        const long long per_cta = (long long)kRowWarps * kRowsPerWarp;
        quant_matvec_row_kernel<<<(unsigned)((dp.drows + per_cta - 1) / per_cta), kRowWarps * 32, 0, R.stream>>>(dp);
        if (launched("quant_matvec_row_kernel") != 0)
            return -1;
    }
    return 0;
}


// Multi-token jobs: the staged matmul kernel for the jobs it takes (8 or more tokens, a 16-byte
// aligned matrix whose rows are a multiple of 16 bytes, 16-byte aligned X), per-token matrix-vector
// products for the rest. Jobs with the same X share its prepared fragments.
int matmul_chunk(const KernelCudaMatmulJob *jobs, int n, std::vector<KernelCudaMatvecJob> &rest)
{
    static bool attr_set = false;
    Runtime &R = rt();
    MParams mp;
    memset(static_cast<void *>(&mp), 0, sizeof(mp));
    struct XEnt {
        const float *X;
        size_t cols, T;
        size_t off_bf, off_bm, off_e;
    };
    std::vector<XEnt> xe;
    std::vector<int> xidx;
    long long tiles = 0;
    for (int i = 0; i < n; i++) {
        const KernelCudaMatmulJob &j = jobs[i];
        const int nb = (int)(j.cols / 256);
        const long long rb = (long long)nb * (j.is_q6 ? 210 : 144);
        const bool staged = j.T >= 8 && aligned16(j.matrix) && aligned16(j.X) && rb % 16 == 0 && nb <= kMmMaxNb &&
                            j.rows < (1u << 30) && j.T < (1u << 30);
        if (!staged) {
            for (size_t t = 0; t < j.T; t++)
                rest.push_back(KernelCudaMatvecJob{j.is_q6, j.matrix, j.X + t * j.cols, j.Y + t * j.rows, j.rows, j.cols});
            continue;
        }
        int x = -1;
        for (size_t q = 0; q < xe.size(); q++)
            if (xe[q].X == j.X && xe[q].cols == j.cols && xe[q].T == j.T)
                x = (int)q;
        if (x < 0) {
            xe.push_back(XEnt{j.X, j.cols, j.T, 0, 0, 0});
            x = (int)xe.size() - 1;
        }
        const CUtensorMap *map = job_map(static_cast<const unsigned char *>(j.matrix), (long long)j.rows, (int)rb,
                                         j.is_q6 ? kQ6Slot : kQ4Slot);
        if (!map)
            return -1;
        const int rgroups = (int)((j.rows + kMmRows - 1) / kMmRows);
        const int chunks = (int)((j.T + kMmTok - 1) / kMmTok);
        mp.jobs[mp.njobs] = MJob{map, nullptr, nullptr, nullptr, j.Y, nullptr, 0, (int)j.rows, nb, (int)j.T,
                                 j.is_q6 ? 1 : 0, rgroups, chunks, 1};
        xidx.push_back(x);
        mp.njobs++;
        tiles += (long long)rgroups * chunks;
    }
    if (mp.njobs == 0)
        return 0;
    // Few tiles (small T, few rows): split each tile's blocks into P parts, summed afterwards by
    // quant_mm_reduce_kernel. P minimises an estimate of the call's time: waves of one CTA per SM
    // x blocks per part x the measured time of one block per CTA (about 4.5 us Q4_K, 9 us Q6_K),
    // plus, when split, the reduce launch and the partial products written and read at HBM speed.
    int nb_max = 1;
    double block_us = 4.5, out_elems = 0;
    for (int q = 0; q < mp.njobs; q++) {
        nb_max = std::max(nb_max, mp.jobs[q].nb);
        if (mp.jobs[q].is_q6)
            block_us = 9.0;
        out_elems += (double)mp.jobs[q].rows * mp.jobs[q].T;
    }
    int want_p = 1;
    double best = 1e300;
    for (int P = 1; P <= std::min(16, nb_max); P++) {
        const double waves = (double)((tiles * P + R.num_sms - 1) / R.num_sms);
        const double cost = waves * ((nb_max + P - 1) / P) * block_us + (P > 1 ? 3.0 + P * out_elems * 8.0 / 6.0e6 : 0.0);
        if (cost < best) {
            best = cost;
            want_p = P;
        }
    }
    RParams rp;
    memset(static_cast<void *>(&rp), 0, sizeof(rp));
    size_t part_bytes = 0;
    for (int q = 0; q < mp.njobs; q++) {
        MJob &J = mp.jobs[q];
        J.P = std::max(1, std::min(want_p, J.nb));
        J.item0 = mp.items;
        mp.items += (long long)J.rgroups * J.chunks * J.P;
        if (J.P > 1) {
            rp.jobs[rp.njobs] = RJob{nullptr, J.y, nullptr, rp.n, J.rows, J.T, J.P, -1};
            rp.n += (long long)J.rows * J.T;
            rp.njobs++;
            part_bytes += ((size_t)J.P * J.rows * J.T * sizeof(float) + 255) / 256 * 256;
        }
    }
    if (mp.items >= (1ll << 31))
        return fail("kernel_cuda_matmul_quant_batch: too many tiles in one call");
    // scratch: per distinct X, B fragments [chunk][block][group][mma][lane], min-term fragments
    // [chunk][block][group][lane], scale exponents [T]
    size_t total = 0;
    for (XEnt &e : xe) {
        const size_t chunks = (e.T + kMmTok - 1) / kMmTok, nb = e.cols / 256;
        e.off_bf = total;
        total += chunks * nb * kMmBfBytes;
        e.off_bm = total;
        total += chunks * nb * kMmBmBytes;
        e.off_e = total;
        total += (e.T * sizeof(int) + 255) / 256 * 256;
    }
    const size_t off_part = total;
    total += part_bytes;
    unsigned char *ws = static_cast<unsigned char *>(scratch(total));
    if (!ws)
        return -1;
    size_t pos = off_part;
    for (int q = 0, r = 0; q < mp.njobs; q++) {
        MJob &J = mp.jobs[q];
        const XEnt &e = xe[xidx[q]];
        J.bf = reinterpret_cast<const uint2 *>(ws + e.off_bf);
        J.bm = reinterpret_cast<const uint2 *>(ws + e.off_bm);
        J.e = reinterpret_cast<const int *>(ws + e.off_e);
        if (J.P > 1) {
            J.part = reinterpret_cast<float *>(ws + pos);
            rp.jobs[r].part = J.part;
            rp.jobs[r].e = J.e;
            r++;
            pos += ((size_t)J.P * J.rows * J.T * sizeof(float) + 255) / 256 * 256;
        }
    }
    PParams pp;
    memset(static_cast<void *>(&pp), 0, sizeof(pp));
    long long ctas = 0;
    for (const XEnt &e : xe) {
        pp.jobs[pp.njobs++] = PJob{e.X, reinterpret_cast<uint2 *>(ws + e.off_bf), reinterpret_cast<uint2 *>(ws + e.off_bm),
                                   reinterpret_cast<int *>(ws + e.off_e), (int)e.T, (int)e.cols, (int)ctas};
        ctas += (long long)((e.T + kMmTok - 1) / kMmTok * kMmTok);
    }
    if (ctas >= (1ll << 31))
        return fail("kernel_cuda_matmul_quant_batch: too many tokens in one call");
    quant_mm_prep_kernel<<<(unsigned)ctas, 256, 0, R.stream>>>(pp);
    if (launched("quant_mm_prep_kernel") != 0)
        return -1;
    if (!attr_set) {
        if (check(cudaFuncSetAttribute(quant_matmul_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMmSmem),
                  "matmul shared memory") != 0)
            return -1;
        attr_set = true;
    }
    mp.err = R.err_word;
    quant_matmul_kernel<<<(unsigned)mp.items, kThreads, kMmSmem, R.stream>>>(mp);
    if (launched("quant_matmul_kernel") != 0)
        return -1;
    if (rp.njobs == 0)
        return 0;
    const long long blocks = std::min<long long>((rp.n + 255) / 256, 8ll * R.num_sms);
    return launch_dependent(quant_mm_reduce_kernel, dim3((unsigned)blocks), dim3(256), 0, R.stream,
                            "quant_mm_reduce_kernel", rp);
}


// Jobs of 64 or more tokens on a 16-byte-aligned matrix whose rows are a multiple of 16 bytes (and
// 16-byte-aligned X), when together they make at least 64 tiles of 128 rows x 64 tokens (with
// fewer, most SMs would idle and the warp-MMA kernel, which splits tiles along the blocks, is
// faster): the tensor-core kernel, one launch for both formats after one prep launch for every
// distinct X (plus a reduce launch when tiles are split along the blocks). The others go to
// `others`.
// `rows` (optional, one entry per job): per-token row pointers of a job's activations and
// results. A job with them runs here or nowhere: when it cannot take the tensor-core path, or its
// rows do not fit the parameter tables, the call returns 1 before launching anything.
int matmul_tc_chunk(const KernelCudaMatmulJob *jobs, int n, std::vector<KernelCudaMatmulJob> &others,
                    const MmRows *rows = nullptr)
{
    static bool attr = false;
    Runtime &R = rt();
    TParams tp[2];
    memset(static_cast<void *>(tp), 0, sizeof(tp));
    struct XEnt {
        const float *X;
        const float *const *xr;          // per-token activation rows, or null
        size_t cols, T, off_bq, off_bsum, off_e;
    };
    std::vector<XEnt> xe;
    auto has_rows = [&](int i) { return rows && rows[i].x && rows[i].y; };
    auto eligible = [&](int i) {
        const KernelCudaMatmulJob &j = jobs[i];
        const long long rb = (long long)(j.cols / 256) * (j.is_q6 ? 210 : 144);
        bool ok = j.T >= 64 && aligned16(j.matrix) && rb % 16 == 0 && j.rows < (1u << 30) && j.T < (1u << 30);
        if (ok && has_rows(i)) {
            for (size_t t = 0; t < j.T && ok; t++)
                ok = rows[i].x[t] && aligned16(rows[i].x[t]) && rows[i].y[t];
        } else if (ok) {
            ok = aligned16(j.X);
        }
        return ok;
    };
    long long tiles = 0;
    for (int i = 0; i < n; i++)
        if (eligible(i))
            tiles += (long long)((jobs[i].rows + tcm::kRows - 1) / tcm::kRows) *
                     (long long)((jobs[i].T + tcm::kTok - 1) / tcm::kTok);
    const bool use_tc = tiles >= 64;
    struct Sel {
        const KernelCudaMatmulJob *j;
        const CUtensorMap *map;
        int x, nb, rtiles, ctiles;
        int parts;
        int idx;
    };
    std::vector<Sel> sel[2];
    long long ftiles[2] = {0, 0};
    for (int i = 0; i < n; i++)
        if (has_rows(i) && (!use_tc || !eligible(i)))
            return 1;                        // nothing launched: the caller takes another route
    for (int i = 0; i < n; i++) {
        const KernelCudaMatmulJob &j = jobs[i];
        const int nb = (int)(j.cols / 256);
        const long long rb = (long long)nb * (j.is_q6 ? 210 : 144);
        if (!use_tc || !eligible(i)) {
            others.push_back(j);
            continue;
        }
        const float *const *xr = has_rows(i) ? rows[i].x : nullptr;
        int x = -1;
        for (size_t q = 0; q < xe.size(); q++)
            if (xe[q].xr == xr && (xr || xe[q].X == j.X) && xe[q].cols == j.cols && xe[q].T == j.T)
                x = (int)q;
        if (x < 0) {
            xe.push_back(XEnt{j.X, xr, j.cols, j.T, 0, 0, 0});
            x = (int)xe.size() - 1;
        }
        const CUtensorMap *map = job_map(static_cast<const unsigned char *>(j.matrix), (long long)j.rows, (int)rb,
                                         j.is_q6 ? kQ6Slot : kQ4Slot, tcm::kRows);
        if (!map)
            return -1;
        const int rtiles = (int)((j.rows + tcm::kRows - 1) / tcm::kRows), ctiles = (int)((j.T + tcm::kTok - 1) / tcm::kTok);
        sel[j.is_q6 ? 1 : 0].push_back(Sel{&j, map, x, nb, rtiles, ctiles, 1, i});
        ftiles[j.is_q6 ? 1 : 0] += (long long)rtiles * ctiles;
    }
    if (xe.empty())
        return 0;
    // Split along the blocks when the call has fewer tiles than SMs (a few jobs of 64 tokens, e.g.
    // one layer's projections for a round of slots): part h of a job takes blocks
    // [h nb / P, (h + 1) nb / P), at least 2 of them, and writes an unscaled partial plane; the
    // reduce launch sums the planes in part order, so results repeat bit for bit. A CTA's time is
    // a fixed set-up and drain plus a cost per block of about the same size for both formats, so
    // with every CTA in one wave the call takes as long as its largest part: P_j is chosen per job
    // as the split that makes the largest part smallest while all CTAs still fit one wave.
    size_t part_floats = 0;
    if (ftiles[0] + ftiles[1] < R.num_sms) {
        std::vector<int> cand;
        for (int k = 0; k < 2; k++)
            for (const Sel &q : sel[k])
                for (int p = 1; p <= std::max(1, q.nb / 2); p++)
                    cand.push_back((q.nb + p - 1) / p);
        std::sort(cand.begin(), cand.end());
        cand.erase(std::unique(cand.begin(), cand.end()), cand.end());
        for (const int w : cand) {
            long long ctas = 0;
            int ent[2] = {0, 0};
            bool fits = true;
            for (int k = 0; k < 2 && fits; k++)
                for (const Sel &q : sel[k]) {
                    const int p = std::min(std::max(1, q.nb / 2), (q.nb + w - 1) / w);
                    if ((q.nb + p - 1) / p > w) {
                        fits = false;
                        break;
                    }
                    ctas += (long long)q.rtiles * q.ctiles * p;
                    ent[k] += p;
                }
            if (!fits || ctas > R.num_sms || ent[0] > kMaxJobs || ent[1] > kMaxJobs)
                continue;
            for (int k = 0; k < 2; k++)
                for (Sel &q : sel[k])
                    q.parts = std::min(std::max(1, q.nb / 2), (q.nb + w - 1) / w);
            break;
        }
        for (int k = 0; k < 2; k++)
            for (const Sel &q : sel[k])
                if (q.parts > 1)
                    part_floats += (size_t)q.parts * q.j->T * q.j->rows;
    }
    if (tp[0].items >= (1ll << 31) || tp[1].items >= (1ll << 31))
        return fail("kernel_cuda_matmul_quant_batch: too many tiles in one call");
    // scratch per distinct X: B quarter tiles [token tile][quarter][16 KB], sums tiles
    // [token tile][block][4 KB], scale exponents [T]
    size_t total = 0;
    for (XEnt &e : xe) {
        const size_t ct = (e.T + tcm::kTok - 1) / tcm::kTok;
        e.off_bq = total;
        total += ct * (e.cols / 64) * tcm::kTile;
        e.off_bsum = total;
        total += ct * (e.cols / 256) * 4096;
        e.off_e = total;
        total += (e.T * sizeof(int) + 255) / 256 * 256;
    }
    const size_t off_part = total;
    total += part_floats * sizeof(float);
    unsigned char *ws = static_cast<unsigned char *>(scratch(total));
    if (!ws)
        return -1;
    RParams rp;
    memset(static_cast<void *>(&rp), 0, sizeof(rp));
    int nyr[2] = {0, 0}, nry = 0, nxr = 0;  // row-table entries used: tp[k].yr, rp.yr, pp.xr
    // a row table of T entries at the end of `tab` (capacity kRowTab); -1 when it does not fit
    auto put_rows = [](auto *tab, int &used, auto *src, size_t T) -> int {
        if (used + (long long)T > kRowTab)
            return -1;
        const int at = used;
        for (size_t t = 0; t < T; t++)
            tab[at + t] = src[t];
        used += (int)T;
        return at;
    };
    {
        float *part = reinterpret_cast<float *>(ws + off_part);
        for (int k = 0; k < 2; k++) {
            TParams &P = tp[k];
            for (const Sel &q : sel[k]) {
                const int S = q.parts;
                const KernelCudaMatmulJob &j = *q.j;
                const XEnt &e = xe[q.x];
                const long long plane = (long long)j.T * j.rows;
                int yr0 = -1;
                if (has_rows(q.idx) && (yr0 = S > 1 ? put_rows(rp.yr, nry, rows[q.idx].y, j.T)
                                                    : put_rows(P.yr, nyr[k], rows[q.idx].y, j.T)) < 0)
                    return 1;                // tables full, nothing launched yet
                for (int h = 0; h < S; h++) {
                    const int b0 = h * q.nb / S, b1 = (h + 1) * q.nb / S;
                    P.jobs[P.njobs++] = TJob{q.map, reinterpret_cast<const uint4 *>(ws + e.off_bq),
                                             reinterpret_cast<const uint4 *>(ws + e.off_bsum),
                                             reinterpret_cast<const int *>(ws + e.off_e), S > 1 ? part + h * plane : j.Y,
                                             P.items, (int)j.rows, b1 - b0, (int)j.T, q.rtiles, q.ctiles, b0, q.nb,
                                             S > 1 ? 1 : 0, S > 1 ? -1 : yr0};
                    P.items += (long long)q.rtiles * q.ctiles;
                }
                if (S > 1) {
                    rp.jobs[rp.njobs++] = RJob{part, j.Y, reinterpret_cast<const int *>(ws + e.off_e), rp.n, (int)j.rows,
                                               (int)j.T, S, yr0};
                    rp.n += plane;
                    part += S * plane;
                }
            }
        }
    }
    PParamsTc pp;
    memset(static_cast<void *>(&pp), 0, sizeof(pp));
    long long ctas = 0;
    for (const XEnt &e : xe) {
        const int xr0 = e.xr ? put_rows(pp.xr, nxr, e.xr, e.T) : -1;
        if (e.xr && xr0 < 0)
            return 1;
        pp.jobs[pp.njobs++] = PJobTc{e.X, reinterpret_cast<uint4 *>(ws + e.off_bq), reinterpret_cast<uint4 *>(ws + e.off_bsum),
                                     reinterpret_cast<int *>(ws + e.off_e), (int)e.T, (int)e.cols, (int)ctas, xr0};
        ctas += (long long)((e.T + tcm::kTok - 1) / tcm::kTok * tcm::kTok);
    }
    if (ctas >= (1ll << 31))
        return fail("kernel_cuda_matmul_quant_batch: too many tokens in one call");
    quant_mm_tc_prep_kernel<<<(unsigned)ctas, 256, 0, R.stream>>>(pp);
    if (launched("quant_mm_tc_prep_kernel") != 0)
        return -1;
    {
        const int smem = std::max(TcCfg<true>::kSmem, TcCfg<false>::kSmem);
        if (!attr) {
            if (check(cudaFuncSetAttribute(quant_mm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                      "tensor-core matmul shared memory") != 0)
                return -1;
            attr = true;
        }
        tp[0].err = tp[1].err = R.err_word;
        const long long items = tp[0].items + tp[1].items;
        if (items >= (1ll << 31))
            return fail("kernel_cuda_matmul_quant_batch: too many tiles in one call");
        TParams2 p2;
        p2.f[0] = tp[0];
        p2.f[1] = tp[1];
        // a programmatic dependent of the prep kernel: set-up, the weight stream and the decode
        // start while the prep kernel finishes
        if (launch_dependent(quant_mm_tc_kernel, dim3((unsigned)items), dim3(tcm::kThreads), (size_t)smem, R.stream,
                             "quant_mm_tc_kernel", p2) != 0)
            return -1;
    }
    if (rp.njobs == 0)
        return 0;
    const long long blocks = std::min<long long>((rp.n + 255) / 256, 8ll * R.num_sms);
    return launch_dependent(quant_mm_reduce_kernel, dim3((unsigned)blocks), dim3(256), 0, R.stream,
                            "quant_mm_reduce_kernel", rp);
}

}  // namespace
}  // namespace rb

using namespace rb;

extern "C" int kernel_cuda_matvec_quant_batch(const KernelCudaMatvecJob *jobs, int n)
{
    if (ensure() != 0)
        return -1;
    if (n < 0 || (n > 0 && !jobs))
        return fail("kernel_cuda_matvec_quant_batch: bad job array");
    for (int i = 0; i < n; i += kMaxJobs)
        if (matvec_chunk(jobs + i, std::min(kMaxJobs, n - i)) != 0)
            return -1;
    return 0;
}

namespace rb {

int matmul_quant_rows(const KernelCudaMatmulJob *jobs, int n, const MmRows *rows)
{
    if (ensure() != 0)
        return -1;
    if (n < 0 || n > kMaxJobs || (n > 0 && (!jobs || !rows)))
        return 1;
    for (int i = 0; i < n; i++) {
        const KernelCudaMatmulJob &j = jobs[i];
        if (!j.matrix || !j.X || !j.Y || !j.rows || !j.cols || !j.T || j.cols % 256 != 0 ||
            j.rows > 0xFFFFFFFFull || j.cols > 0xFFFFFFFFull || j.T > 0xFFFFFFFFull)
            return fail("matmul with row tables: job %d invalid", i);
    }
    std::vector<KernelCudaMatmulJob> small;
    const int rc = matmul_tc_chunk(jobs, n, small, rows);
    if (rc != 0)
        return rc;
    std::vector<KernelCudaMatvecJob> rest;
    if (!small.empty() && matmul_chunk(small.data(), (int)small.size(), rest) != 0)
        return -1;
    return rest.empty() ? 0 : kernel_cuda_matvec_quant_batch(rest.data(), (int)rest.size());
}

}  // namespace rb

using namespace rb;

extern "C" int kernel_cuda_matmul_quant_batch(const KernelCudaMatmulJob *jobs, int n)
{
    if (ensure() != 0)
        return -1;
    if (n < 0 || (n > 0 && !jobs))
        return fail("kernel_cuda_matmul_quant_batch: bad job array");
    for (int i = 0; i < n; i++) {
        const KernelCudaMatmulJob &j = jobs[i];
        // the reference's mm_job_valid (kernels.c:1916-1920)
        if (!j.matrix || !j.X || !j.Y || !j.rows || !j.cols || !j.T || j.cols % 256 != 0 ||
            j.rows > 0xFFFFFFFFull || j.cols > 0xFFFFFFFFull || j.T > 0xFFFFFFFFull)
            return fail("kernel_cuda_matmul_quant_batch: job %d invalid (null pointer, zero size, or cols not "
                        "a multiple of 256)", i);
    }
    std::vector<KernelCudaMatvecJob> rest;
    for (int i = 0; i < n; i += kMaxJobs) {
        std::vector<KernelCudaMatmulJob> small;
        if (matmul_tc_chunk(jobs + i, std::min(kMaxJobs, n - i), small) != 0)
            return -1;
        if (!small.empty() && matmul_chunk(small.data(), (int)small.size(), rest) != 0)
            return -1;
    }
    return rest.empty() ? 0 : kernel_cuda_matvec_quant_batch(rest.data(), (int)rest.size());
}
