// Gated DeltaNet pre-ops and post-op on the GPU, and the fused recurrent-layer drop-ins.
//
// Pre-ops (reference src/model.c:1291-1328 for a decode token; the same per-token loop in
// pf_ssm, model.c:1619-1643), per channel c of the 8192-wide qkv projection:
//     cv[c] = sum_{j<3} x_{t-3+j}[c] w[c][j] + x_t[c] w[c][3]   (depthwise causal conv, k = 4,
//             x_s for s < 0 from the layer's 3-row history; kernels.c:693-719)
//     cv[c] = cv[c] sigmoid(cv[c])                              (SiLU, kernels.c:628-651)
//     q = cv[0:2048], k = cv[2048:4096] L2-normalised per 128 (eps 1e-6), v = cv[4096:8192]
//     beta' = sigmoid(beta), g = a softplus(alpha + dt), softplus(x) = x for x > 20
//     history <- raw inputs of the last 3 tokens                (model.c:1299-1306)
// Post-op (model.c:1333-1343, pf_ssm 1655-1658), per value head row of 128:
//     out = rmsnorm(out) * ssm_norm (eps 1e-6), then out *= z sigmoid(z).
//
// deltanet_preop_kernel: one CTA per (128-channel block, token), one thread per channel; the 16
// q and 16 k blocks are exactly one head each, so the L2 norm is a CTA reduction.
// deltanet_history_kernel: the history shift of prompts (T > 1), after every token has read the
// old history; a decode token's shift is done by the pre-op thread that read the rows.
// deltanet_postop_kernel: one warp per (token, value head) row.
// All three are HBM/latency-bound elementwise work; fp32 throughout. They launch as programmatic
// dependents, so a decode step's pre-op, recurrence and post-op launches overlap one another's
// ramp and drain.
#include "ptx.cuh"
#include "runtime.h"
#include "../../include/roaster_cuda.h"

#include <cuda_runtime.h>
#include <algorithm>
#include <cstring>
#include <vector>

namespace rb {

int deltanet_step_batch(const KernelDeltaStepJob *jobs, int n);
int deltanet_prefill_batch(const KernelDeltaPrefillJob *jobs, int n);

namespace {

constexpr int kQKV = 8192;
constexpr int kMaxJobs = 64;

struct PreJob {
    const float *qkv, *alpha, *beta;
    float *conv_state;                 // shifted here for a job of one token (T = 1)
    const float *conv_w, *dt, *a;
    float *q, *k, *v, *g, *b;
    long long T, tok0;
};

struct PreParams {
    PreJob jobs[kMaxJobs];
    int njobs;
};

__device__ __forceinline__ int find_job(const PreParams &p, long long gtok)
{
    int lo = 0, hi = p.njobs - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (p.jobs[mid].tok0 <= gtok)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

// sigmoid in the form that never overflows exp
__device__ __forceinline__ float sigmoid_stable(float x)
{
    if (x >= 0.0f)
        return 1.0f / (1.0f + expf(-x));
    const float e = expf(x);
    return e / (1.0f + e);
}

__global__ void __launch_bounds__(128) deltanet_preop_kernel(const __grid_constant__ PreParams p)
{
    __shared__ float red[4];
    // launched as a programmatic dependent (as are the history and post-op kernels): every input
    // may be the previous kernel's output, so nothing is read or written before the wait
    griddep_wait();
    griddep_launch_dependents();
    const long long gtok = blockIdx.y;
    const PreJob &J = p.jobs[find_job(p, gtok)];
    const long long t = gtok - J.tok0;
    const int blk = blockIdx.x, tid = threadIdx.x;
    const int c = blk * 128 + tid;
    // raw inputs of tokens t-3 .. t (negative tokens come from the history, oldest row first)
    float x[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const long long s = t - 3 + j;
        x[j] = s >= 0 ? __ldg(J.qkv + s * kQKV + c) : J.conv_state[(s + 3) * kQKV + c];
    }
    if (J.T == 1) {
        // a decode token: the new history is the old rows 1, 2 and this token's input. The thread
        // that read channel c's rows is the only one to touch them, so it shifts them itself
        // (prompts of several tokens leave it to deltanet_history_kernel, after every token's read).
#pragma unroll
        for (int j = 0; j < 3; j++)
            J.conv_state[j * kQKV + c] = x[j + 1];
    }
    const float4 w = __ldg(reinterpret_cast<const float4 *>(J.conv_w) + c);
    float sum = x[0] * w.x;
    sum = fmaf(x[1], w.y, sum);
    sum = fmaf(x[2], w.z, sum);
    sum = fmaf(x[3], w.w, sum);
    float y = sum * sigmoid_stable(sum);
    if (blk < 32) {
        // q (blocks 0-15) or k (16-31) head: L2 norm over the block
        float ss = y * y;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((tid & 31) == 0)
            red[tid >> 5] = ss;
        __syncthreads();
        const float tot = (red[0] + red[1]) + (red[2] + red[3]);
        y *= 1.0f / sqrtf(tot + 1e-6f);
        float *dst = blk < 16 ? J.q + (t * 16 + blk) * 128 : J.k + (t * 16 + (blk - 16)) * 128;
        dst[tid] = y;
    } else {
        J.v[(t * 32 + (blk - 32)) * 128 + tid] = y;
    }
    if (blk == 0 && tid < 32) {
        const long long i = t * 32 + tid;
        J.b[i] = 1.0f / (1.0f + expf(-__ldg(J.beta + i)));
        const float xs = __ldg(J.alpha + i) + __ldg(J.dt + tid);
        J.g[i] = __ldg(J.a + tid) * (xs > 20.0f ? xs : log1pf(expf(xs)));
    }
}

struct HistJob {
    const float *qkv;
    float *conv_state;
    long long T;
};

struct HistParams {
    HistJob jobs[kMaxJobs];
};

// New history rows = raw inputs of tokens T-3, T-2, T-1 (old rows where T < 3).
__global__ void __launch_bounds__(256) deltanet_history_kernel(const __grid_constant__ HistParams p)
{
    griddep_wait();                  // the pre-op kernel reads the rows this kernel replaces
    griddep_launch_dependents();
    const HistJob &J = p.jobs[blockIdx.y];
    const int c = blockIdx.x * 256 + threadIdx.x;
    float h[3];
#pragma unroll
    for (int j = 0; j < 3; j++) {
        const long long s = J.T - 3 + j;                 // token index of new row j
        h[j] = s >= 0 ? J.qkv[s * kQKV + c] : J.conv_state[(s + 3) * kQKV + c];
    }
#pragma unroll
    for (int j = 0; j < 3; j++)
        J.conv_state[j * kQKV + c] = h[j];
}

struct PostJob {
    float *out;
    const float *z, *w;
    long long rows, row0;
};

struct PostParams {
    PostJob jobs[kMaxJobs];
    int njobs;
};

__global__ void __launch_bounds__(256) deltanet_postop_kernel(const __grid_constant__ PostParams p,
                                                              long long total_rows)
{
    griddep_wait();                  // `out` is the recurrence's output
    griddep_launch_dependents();
    const long long grow = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (grow >= total_rows)
        return;
    int lo = 0, hi = p.njobs - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (p.jobs[mid].row0 <= grow)
            lo = mid;
        else
            hi = mid - 1;
    }
    const PostJob &J = p.jobs[lo];
    const long long r = grow - J.row0;
    const int lane = threadIdx.x & 31;
    float4 *xo = reinterpret_cast<float4 *>(J.out + r * 128) + lane;
    const float4 x = *xo;
    const float4 z = __ldg(reinterpret_cast<const float4 *>(J.z + r * 128) + lane);
    const float4 w = __ldg(reinterpret_cast<const float4 *>(J.w) + lane);
    float ss = x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf(ss / 128.0f + 1e-6f);
    float4 y;
    y.x = x.x * inv * w.x * (z.x * (1.0f / (1.0f + expf(-z.x))));
    y.y = x.y * inv * w.y * (z.y * (1.0f / (1.0f + expf(-z.y))));
    y.z = x.z * inv * w.z * (z.z * (1.0f / (1.0f + expf(-z.z))));
    y.w = x.w * inv * w.w * (z.w * (1.0f / (1.0f + expf(-z.w))));
    *xo = y;
}

int preop_chunk(const KernelDeltaPreopJob *jobs, int n)
{
    PreParams pp;
    HistParams hp;
    memset(static_cast<void *>(&pp), 0, sizeof(pp));
    memset(static_cast<void *>(&hp), 0, sizeof(hp));
    long long tok = 0;
    int m = 0, mh = 0;                  // jobs; jobs of several tokens (history shifted apart)
    for (int i = 0; i < n; i++) {
        const KernelDeltaPreopJob &j = jobs[i];
        if (!j.qkv || !j.alpha || !j.beta || !j.conv_state || !j.conv_w || !j.dt || !j.a || !j.q || !j.k ||
            !j.v || !j.g || !j.beta_out)
            return fail("kernel_deltanet_preop_batch: job %d has a null pointer", i);
        if (!aligned16(j.conv_w))
            return fail("kernel_deltanet_preop_batch: job %d conv_w not 16-byte aligned", i);
        if (j.T == 0)
            continue;
        pp.jobs[m] = PreJob{j.qkv, j.alpha, j.beta, j.conv_state, j.conv_w, j.dt, j.a,
                            j.q, j.k, j.v, j.g, j.beta_out, (long long)j.T, tok};
        if (j.T > 1)
            hp.jobs[mh++] = HistJob{j.qkv, j.conv_state, (long long)j.T};
        tok += (long long)j.T;
        m++;
    }
    if (m == 0)
        return 0;
    if (tok > 65535ll * 1024)
        return fail("kernel_deltanet_preop_batch: too many tokens in one call (%lld)", tok);
    pp.njobs = m;
    cudaStream_t st = rt().stream;
    for (long long t0 = 0; t0 < tok; t0 += 65535) {
        // grid.y is limited to 65535: walk the flattened tokens in slices
        PreParams ps = pp;
        for (int i = 0; i < m; i++)
            ps.jobs[i].tok0 -= t0;
        const unsigned ny = (unsigned)std::min<long long>(65535, tok - t0);
        // tokens before the slice map to negative indices in ps; find_job only sees
        // blockIdx.y >= 0, i.e. tokens t0 .. t0 + ny - 1
        if (launch_dependent(deltanet_preop_kernel, dim3(64, ny), dim3(128), 0, st, "deltanet_preop_kernel", ps) != 0)
            return -1;
    }
    if (mh == 0)
        return 0;
    return launch_dependent(deltanet_history_kernel, dim3(kQKV / 256, mh), dim3(256), 0, st, "deltanet_history_kernel",
                            hp);
}

int postop_chunk(const KernelDeltaPostopJob *jobs, int n)
{
    PostParams pp;
    memset(static_cast<void *>(&pp), 0, sizeof(pp));
    long long rows = 0;
    int m = 0;
    for (int i = 0; i < n; i++) {
        const KernelDeltaPostopJob &j = jobs[i];
        if (!j.out || !j.z || !j.norm_w)
            return fail("kernel_deltanet_postop_batch: job %d has a null pointer", i);
        if (!aligned16(j.out) || !aligned16(j.z) || !aligned16(j.norm_w))
            return fail("kernel_deltanet_postop_batch: job %d buffers not 16-byte aligned", i);
        if (j.T == 0)
            continue;
        pp.jobs[m++] = PostJob{j.out, j.z, j.norm_w, (long long)j.T * 32, rows};
        rows += (long long)j.T * 32;
    }
    if (m == 0)
        return 0;
    pp.njobs = m;
    return launch_dependent(deltanet_postop_kernel, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0, rt().stream,
                            "deltanet_postop_kernel", pp, rows);
}

}  // namespace

int deltanet_preop_batch(const KernelDeltaPreopJob *jobs, int n)
{
    if (n < 0 || (n > 0 && !jobs))
        return fail("kernel_deltanet_preop_batch: bad job array");
    for (int i = 0; i < n; i += kMaxJobs)
        if (preop_chunk(jobs + i, std::min(kMaxJobs, n - i)) != 0)
            return -1;
    return 0;
}

int deltanet_postop_batch(const KernelDeltaPostopJob *jobs, int n)
{
    if (n < 0 || (n > 0 && !jobs))
        return fail("kernel_deltanet_postop_batch: bad job array");
    for (int i = 0; i < n; i += kMaxJobs)
        if (postop_chunk(jobs + i, std::min(kMaxJobs, n - i)) != 0)
            return -1;
    return 0;
}

// One recurrent layer over T tokens with host inputs/outputs: stage, pre-ops, the recurrence
// (decode step kernel for T = 1, chunked prefill otherwise), gated RMSNorm, copy back.
static int layer_host(float *state, float *conv_state, const float *conv_w, const float *dt, const float *a,
                      const float *ssm_norm, size_t T, const float *qkv, const float *z, const float *alpha,
                      const float *beta, float *out)
{
    if (!state || !conv_state || !conv_w || !dt || !a || !ssm_norm || !qkv || !z || !alpha || !beta || !out)
        return fail("kernel_deltanet_layer: null pointer");
    if (T == 0)
        return 0;
    // host in: qkv [T][8192], z [T][4096], alpha, beta [T][32]; device work: q, k [T][2048],
    // v [T][4096], g, b [T][32]; out [T][4096]
    const size_t n_qkv = T * kQKV, n_z = T * 4096, n_h = T * 32;
    const size_t in_f = n_qkv + n_z + 2 * n_h;
    const size_t off_q = (in_f + 3) / 4 * 4, off_k = off_q + T * 2048, off_v = off_k + T * 2048;
    const size_t off_g = off_v + T * 4096, off_b = off_g + n_h, off_o = (off_b + n_h + 3) / 4 * 4;
    const size_t tot = off_o + T * 4096;
    float *h = static_cast<float *>(pinned(tot * sizeof(float)));
    float *d = static_cast<float *>(dstage(tot * sizeof(float)));
    if (!h || !d)
        return -1;
    memcpy(h, qkv, n_qkv * 4);
    memcpy(h + n_qkv, z, n_z * 4);
    memcpy(h + n_qkv + n_z, alpha, n_h * 4);
    memcpy(h + n_qkv + n_z + n_h, beta, n_h * 4);
    cudaStream_t st = rt().stream;
    if (check(cudaMemcpyAsync(d, h, in_f * 4, cudaMemcpyHostToDevice, st), "stage in") != 0)
        return -1;
    const float *dz = d + n_qkv;
    KernelDeltaPreopJob pj{d, d + n_qkv + n_z, d + n_qkv + n_z + n_h, conv_state, conv_w, dt, a,
                           d + off_q, d + off_k, d + off_v, d + off_g, d + off_b, T};
    if (deltanet_preop_batch(&pj, 1) != 0)
        return -1;
    if (T == 1) {
        KernelDeltaStepJob sj{state, d + off_q, d + off_k, d + off_v, d + off_g, d + off_b, d + off_o};
        if (deltanet_step_batch(&sj, 1) != 0)
            return -1;
    } else {
        KernelDeltaPrefillJob fj{state, d + off_q, d + off_k, d + off_v, d + off_g, d + off_b, d + off_o, T};
        if (deltanet_prefill_batch(&fj, 1) != 0)
            return -1;
    }
    KernelDeltaPostopJob oj{d + off_o, dz, ssm_norm, T};
    if (deltanet_postop_batch(&oj, 1) != 0)
        return -1;
    if (check(cudaMemcpyAsync(h + off_o, d + off_o, T * 4096 * 4, cudaMemcpyDeviceToHost, st), "stage out") != 0)
        return -1;
    if (kernel_cuda_synchronize() != 0)
        return -1;
    memcpy(out, h + off_o, T * 4096 * 4);
    return 0;
}

}  // namespace rb

using namespace rb;

extern "C" int kernel_deltanet_preop_batch(const KernelDeltaPreopJob *jobs, int n)
{
    if (ensure() != 0)
        return -1;
    return deltanet_preop_batch(jobs, n);
}

extern "C" int kernel_deltanet_postop_batch(const KernelDeltaPostopJob *jobs, int n)
{
    if (ensure() != 0)
        return -1;
    return deltanet_postop_batch(jobs, n);
}

extern "C" int kernel_deltanet_layer_step(float *state, float *conv_state, const float *conv_w, const float *dt,
                                          const float *a, const float *ssm_norm, const float *qkv, const float *z,
                                          const float *alpha, const float *beta, float *out)
{
    if (ensure() != 0)
        return -1;
    return layer_host(state, conv_state, conv_w, dt, a, ssm_norm, 1, qkv, z, alpha, beta, out);
}

extern "C" int kernel_deltanet_layer_prefill(float *state, float *conv_state, const float *conv_w, const float *dt,
                                             const float *a, const float *ssm_norm, size_t T, const float *qkv,
                                             const float *z, const float *alpha, const float *beta, float *out)
{
    if (ensure() != 0)
        return -1;
    return layer_host(state, conv_state, conv_w, dt, a, ssm_norm, T, qkv, z, alpha, beta, out);
}
