// Gated DeltaNet decode step on B200: one read and one write of each 64 KB head state.
//
// Replaces recurrent_delta_step (reference src/model.c:272-323). For value head vh (key head
// vh % 16, model.c:285), with d = exp(g):
//     A = S^T k,  B = S^T q,  kq = k.q            (old state)
//     delta = (v - d A) beta
//     out   = (d B + kq delta) / sqrt(128)
//     S    <- d S + k delta^T
// Columns c of S are independent (A[c], B[c], delta[c] and the update of column c only touch
// column c), so a CTA owns a 128-row x 32-column block: it streams the block in once with
// 128-bit loads, reduces A/B over the rows in shared memory, and writes the block back once.
// The kernel is HBM-bound: 2 x 4 bytes per state element per step.
#include "ptx.cuh"
#include "runtime.h"
#include "../../include/roaster_cuda.h"

#include <cuda_runtime.h>
#include <algorithm>
#include <cstring>
#include <vector>

namespace rb {
namespace {

constexpr int kD = 128;             // head dim (state is kD x kD per value head)
constexpr int kCB = 32;             // state columns per CTA
constexpr int kThreads = 128;       // 8 column quads x 16 row groups
constexpr int kRowsPerThread = 8;   // 16 row groups x 8 rows = 128 rows

struct DeltaJob {
    float *state;
    const float *q, *k, *v, *g, *beta;
    float *out;
};

template <int MAXJ>
struct DeltaParams {
    DeltaJob jobs[MAXJ];
};

template <int MAXJ>
__global__ void __launch_bounds__(kThreads) deltanet_step_kernel(const __grid_constant__ DeltaParams<MAXJ> p)
{
    __shared__ float sA[16][kCB], sB[16][kCB], sKQ[16], sDelta[kCB];
    griddep_wait();                  // inputs are written by the kernels before this one
    griddep_launch_dependents();
    const DeltaJob &J = p.jobs[blockIdx.y];
    const int vh = blockIdx.x / (kD / kCB);
    const int cb = blockIdx.x % (kD / kCB);
    const int kh = vh % 16;
    const int t = threadIdx.x;
    const int cq = t & 7, rg = t >> 3;
    const int c0 = cb * kCB + cq * 4;
    float *S = J.state + (size_t)vh * kD * kD;
    const float *kvec = J.k + kh * kD, *qvec = J.q + kh * kD;

    float4 s[kRowsPerThread];
    float kr[kRowsPerThread], qr[kRowsPerThread];
#pragma unroll
    for (int i = 0; i < kRowsPerThread; i++) {
        const int r = rg * kRowsPerThread + i;
        s[i] = __ldcs(reinterpret_cast<const float4 *>(S + r * kD + c0));
        kr[i] = __ldg(kvec + r);
        qr[i] = __ldg(qvec + r);
    }
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f, kq = 0.f;
#pragma unroll
    for (int i = 0; i < kRowsPerThread; i++) {
        a0 = fmaf(s[i].x, kr[i], a0); a1 = fmaf(s[i].y, kr[i], a1);
        a2 = fmaf(s[i].z, kr[i], a2); a3 = fmaf(s[i].w, kr[i], a3);
        b0 = fmaf(s[i].x, qr[i], b0); b1 = fmaf(s[i].y, qr[i], b1);
        b2 = fmaf(s[i].z, qr[i], b2); b3 = fmaf(s[i].w, qr[i], b3);
        kq = fmaf(kr[i], qr[i], kq);
    }
    sA[rg][cq * 4 + 0] = a0; sA[rg][cq * 4 + 1] = a1; sA[rg][cq * 4 + 2] = a2; sA[rg][cq * 4 + 3] = a3;
    sB[rg][cq * 4 + 0] = b0; sB[rg][cq * 4 + 1] = b1; sB[rg][cq * 4 + 2] = b2; sB[rg][cq * 4 + 3] = b3;
    if (cq == 0)
        sKQ[rg] = kq;
    __syncthreads();
    const float d = expf(__ldg(J.g + vh));
    if (t < kCB) {
        float A = 0.f, B = 0.f, KQ = 0.f;
#pragma unroll
        for (int j = 0; j < 16; j++) {
            A += sA[j][t];
            B += sB[j][t];
            KQ += sKQ[j];
        }
        const int c = cb * kCB + t;
        const float beta = __ldg(J.beta + vh);
        const float delta = (__ldg(J.v + vh * kD + c) - d * A) * beta;
        J.out[vh * kD + c] = (d * B + KQ * delta) * 0.08838834764831845f;  // 1/sqrt(128)
        sDelta[t] = delta;
    }
    __syncthreads();
    const float d0 = sDelta[cq * 4 + 0], d1 = sDelta[cq * 4 + 1];
    const float d2 = sDelta[cq * 4 + 2], d3 = sDelta[cq * 4 + 3];
#pragma unroll
    for (int i = 0; i < kRowsPerThread; i++) {
        const int r = rg * kRowsPerThread + i;
        float4 o;
        o.x = fmaf(d, s[i].x, kr[i] * d0);
        o.y = fmaf(d, s[i].y, kr[i] * d1);
        o.z = fmaf(d, s[i].z, kr[i] * d2);
        o.w = fmaf(d, s[i].w, kr[i] * d3);
        __stcs(reinterpret_cast<float4 *>(S + r * kD + c0), o);
    }
}

template <int MAXJ>
int launch_chunk(const KernelDeltaStepJob *jobs, int n)
{
    DeltaParams<MAXJ> p;
    for (int i = 0; i < n; i++) {
        const KernelDeltaStepJob &j = jobs[i];
        if (!j.state || !j.q || !j.k || !j.v || !j.g || !j.beta || !j.out || !aligned16(j.state))
            return fail("kernel_deltanet_step_batch: job %d has a null or misaligned pointer", i);
        p.jobs[i] = DeltaJob{j.state, j.q, j.k, j.v, j.g, j.beta, j.out};
    }
    return launch_dependent(deltanet_step_kernel<MAXJ>, dim3(32 * (kD / kCB), n), dim3(kThreads), 0, rt().stream,
                            "deltanet_step_kernel", p);
}

}  // namespace

int deltanet_step_batch(const KernelDeltaStepJob *jobs, int n)
{
    if (n < 0 || (n > 0 && !jobs))
        return fail("kernel_deltanet_step_batch: bad job array");
    for (int i = 0; i < n;) {
        const int left = n - i;
        int rc;
        if (left <= 32) {
            rc = launch_chunk<32>(jobs + i, left);
            i += left;
        } else {
            const int m = left < 256 ? left : 256;
            rc = launch_chunk<256>(jobs + i, m);
            i += m;
        }
        if (rc != 0)
            return -1;
    }
    return 0;
}

// Host buffers all registered: pipelined over three streams. The copy engine spends a few
// microseconds on every copy whatever its size (about the link time of 150 KB), so the call
// makes few: runs closer than 128 KB copy as one, first the small per-head inputs (g, beta) of
// every job, then each chunk's q, k, v runs, in at most kDnChunks chunks of at least 32 jobs.
// Chunk c's step launch waits for its inputs (an event). Outputs copy back on the out stream
// (the other copy engine), each chunk's once its launch is done and none before the last input
// has landed: device-to-host copies beside the input copies slow them down, and the inputs are
// the critical path. The work stream waits for the last output copy, so synchronising it covers
// the whole call.
#ifndef DN_HOST_CHUNKS
#define DN_HOST_CHUNKS 3
#endif
int step_registered(const KernelDeltaStepJob *jobs, int n)
{
    constexpr int kDnChunks = DN_HOST_CHUNKS;
    const size_t nq = 16 * 128, nv = 32 * 128, nh = 32;
    const int chunks = std::max(1, std::min(kDnChunks, n / 32));
    cudaStream_t ws = rt().stream;                 // may be the legacy default stream (null)
    cudaStream_t cs = ws, os = ws;
    if (chunks > 1 && (!(cs = copy_stream()) || !(os = out_stream())))
        return -1;
    // events: [0, kDnChunks) inputs landed, [kDnChunks, 2 kDnChunks) chunk launch done,
    // 2 kDnChunks: work stream start, 2 kDnChunks + 1: last output copy done
    static cudaEvent_t ev[2 * kDnChunks + 2];
    static int made = -1;
    if (made != rt().device) {
        for (auto &e : ev)
            if (check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate") != 0)
                return -1;
        made = rt().device;
    }
    cudaEvent_t *ev_in = ev, *ev_done = ev + kDnChunks, ev_start = ev[2 * kDnChunks],
                ev_out = ev[2 * kDnChunks + 1];
    auto rec = [](cudaEvent_t e, cudaStream_t st) { return check(cudaEventRecord(e, st), "cudaEventRecord"); };
    auto wait = [](cudaStream_t st, cudaEvent_t e) {
        return check(cudaStreamWaitEvent(st, e, 0), "cudaStreamWaitEvent");
    };
    auto up16 = [](size_t x) { return (x + 15) & ~(size_t)15; };
    HostRuns small;
    for (int i = 0; i < n; i++) {
        small.add(jobs[i].g, nh * 4);
        small.add(jobs[i].beta, nh * 4);
    }
    small.build(kRunGap);
    std::vector<HostRuns> in(chunks), out(chunks);
    std::vector<size_t> base(chunks + 1, up16(small.bytes) + 16);
    for (int c = 0; c < chunks; c++) {
        const int i0 = (int)((long long)n * c / chunks), i1 = (int)((long long)n * (c + 1) / chunks);
        for (int i = i0; i < i1; i++) {
            const KernelDeltaStepJob &s = jobs[i];
            in[c].add(s.q, nq * 4);
            in[c].add(s.k, nq * 4);
            in[c].add(s.v, nv * 4);
            out[c].add(s.out, nv * 4);
        }
        in[c].build(kRunGap);
        out[c].build(0);
        base[c + 1] = base[c] + up16(in[c].bytes) + up16(out[c].bytes) + 32;
    }
    char *d = static_cast<char *>(dstage(base[chunks]));
    if (!d)
        return -1;
    // both side streams start after everything queued on the work stream so far
    if (chunks > 1 && (rec(ev_start, ws) != 0 || wait(cs, ev_start) != 0 || wait(os, ev_start) != 0))
        return -1;
    if (runs_copy(small, d, cudaMemcpyHostToDevice, cs) != 0)
        return -1;
    for (int c = 0; c < chunks; c++) {
        if (runs_copy(in[c], d + base[c], cudaMemcpyHostToDevice, cs) != 0)
            return -1;
        if (chunks > 1 && rec(ev_in[c], cs) != 0)
            return -1;
    }
    if (chunks > 1 && wait(os, ev_in[chunks - 1]) != 0)
        return -1;
    std::vector<KernelDeltaStepJob> dj(jobs, jobs + n);
    for (int c = 0; c < chunks; c++) {
        const int i0 = (int)((long long)n * c / chunks), i1 = (int)((long long)n * (c + 1) / chunks);
        char *din = d + base[c];
        char *dout = din + up16(in[c].bytes) + 16;
        for (int i = i0; i < i1; i++) {
            const KernelDeltaStepJob &s = jobs[i];
            auto at = [&](const float *p) { return reinterpret_cast<const float *>(din + in[c].offset(p)); };
            dj[i].q = at(s.q);
            dj[i].k = at(s.k);
            dj[i].v = at(s.v);
            dj[i].g = reinterpret_cast<const float *>(d + small.offset(s.g));
            dj[i].beta = reinterpret_cast<const float *>(d + small.offset(s.beta));
            dj[i].out = reinterpret_cast<float *>(dout + out[c].offset(s.out));
        }
        if (chunks > 1 && wait(ws, ev_in[c]) != 0)
            return -1;
        if (deltanet_step_batch(dj.data() + i0, i1 - i0) != 0)
            return -1;
        if (chunks > 1 && (rec(ev_done[c], ws) != 0 || wait(os, ev_done[c]) != 0))
            return -1;
        if (runs_copy(out[c], dout, cudaMemcpyDeviceToHost, os) != 0)
            return -1;
    }
    if (chunks > 1 && (rec(ev_out, os) != 0 || wait(ws, ev_out) != 0))
        return -1;
    return kernel_cuda_synchronize() != 0 ? -1 : 0;
}

}  // namespace rb

using namespace rb;

extern "C" int kernel_deltanet_step_batch(const KernelDeltaStepJob *jobs, int n)
{
    if (ensure() != 0)
        return -1;
    return deltanet_step_batch(jobs, n);
}

extern "C" int kernel_deltanet_step_batch_host(const KernelDeltaStepJob *jobs, int n)
{
    if (ensure() != 0)
        return -1;
    if (n < 0 || (n > 0 && !jobs))
        return fail("kernel_deltanet_step_batch_host: bad job array");
    if (n == 0)
        return 0;
    // per job: q, k [16x128], v [32x128], g, beta [32] in; out [32x128]
    const size_t nq = 16 * 128, nv = 32 * 128, nh = 32;
    const size_t in_f = 2 * nq + nv + 2 * nh, out_f = nv;
    const size_t total = (size_t)n * (in_f + out_f);
    // Registered buffers: when every job's host buffers lie in memory registered with
    // kernel_cuda_host_register, the copy engine moves their contiguous runs straight between
    // host and device, with no staging memcpy on the host.
    {
        bool reg = true;
        for (int i = 0; i < n && reg; i++) {
            const KernelDeltaStepJob &s = jobs[i];
            if (!s.state || !s.q || !s.k || !s.v || !s.g || !s.beta || !s.out)
                return fail("kernel_deltanet_step_batch_host: job %d has a null pointer", i);
            reg = host_registered(s.q, nq * 4) && host_registered(s.k, nq * 4) && host_registered(s.v, nv * 4) &&
                  host_registered(s.g, nh * 4) && host_registered(s.beta, nh * 4) &&
                  host_registered(s.out, out_f * 4);
        }
        if (reg)
            return step_registered(jobs, n);
    }
    float *h = static_cast<float *>(pinned(total * sizeof(float)));
    float *d = static_cast<float *>(dstage(total * sizeof(float)));
    if (!h || !d)
        return -1;
    std::vector<KernelDeltaStepJob> dj(jobs, jobs + n);
    for (int i = 0; i < n; i++) {
        const KernelDeltaStepJob &s = jobs[i];
        if (!s.state || !s.q || !s.k || !s.v || !s.g || !s.beta || !s.out)
            return fail("kernel_deltanet_step_batch_host: job %d has a null pointer", i);
        float *db = d + (size_t)i * in_f;
        dj[i].q = db;
        dj[i].k = db + nq;
        dj[i].v = db + 2 * nq;
        dj[i].g = db + 2 * nq + nv;
        dj[i].beta = db + 2 * nq + nv + nh;
        dj[i].out = d + (size_t)n * in_f + (size_t)i * out_f;
    }
    const int in_ok = stage_in(h, d, n, in_f, [&](int i, float *b) {
        const KernelDeltaStepJob &s = jobs[i];
        memcpy(b, s.q, nq * 4);
        memcpy(b + nq, s.k, nq * 4);
        memcpy(b + 2 * nq, s.v, nv * 4);
        memcpy(b + 2 * nq + nv, s.g, nh * 4);
        memcpy(b + 2 * nq + nv + nh, s.beta, nh * 4);
    });
    if (in_ok != 0 || deltanet_step_batch(dj.data(), n) != 0)
        return -1;
    const int ok = stage_out(h + (size_t)n * in_f, d + (size_t)n * in_f, n, out_f,
                             [&](int i, const float *b) { memcpy(jobs[i].out, b, out_f * 4); });
    if (ok != 0)
        return -1;
    return kernel_cuda_synchronize() != 0 ? -1 : 0;
}

extern "C" int kernel_deltanet_step(float *state, const float *q, const float *k, const float *v,
                                    const float *g, const float *beta, float *out)
{
    if (ensure() != 0)
        return -1;
    if (!state || !q || !k || !v || !g || !beta || !out)
        return fail("kernel_deltanet_step: null pointer");
    // Stage q,k [16x128], v [32x128], g, beta [32] in one pinned block, one copy each way.
    const size_t nq = 16 * 128, nv = 32 * 128, nh = 32;
    const size_t in_floats = 2 * nq + nv + 2 * nh, out_floats = nv;
    float *h = static_cast<float *>(pinned((in_floats + out_floats) * sizeof(float)));
    float *d = static_cast<float *>(dstage((in_floats + out_floats) * sizeof(float)));
    if (!h || !d)
        return -1;
    memcpy(h, q, nq * 4);
    memcpy(h + nq, k, nq * 4);
    memcpy(h + 2 * nq, v, nv * 4);
    memcpy(h + 2 * nq + nv, g, nh * 4);
    memcpy(h + 2 * nq + nv + nh, beta, nh * 4);
    cudaStream_t s = rt().stream;
    if (check(cudaMemcpyAsync(d, h, in_floats * 4, cudaMemcpyHostToDevice, s), "stage in") != 0)
        return -1;
    KernelDeltaStepJob j{state, d, d + nq, d + 2 * nq, d + 2 * nq + nv, d + 2 * nq + nv + nh,
                         d + in_floats};
    if (deltanet_step_batch(&j, 1) != 0)
        return -1;
    if (check(cudaMemcpyAsync(h + in_floats, d + in_floats, out_floats * 4, cudaMemcpyDeviceToHost, s),
              "stage out") != 0)
        return -1;
    if (kernel_cuda_synchronize() != 0)
        return -1;
    memcpy(out, h + in_floats, out_floats * 4);
    return 0;
}
