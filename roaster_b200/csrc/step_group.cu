// Cross-slot batched step (the KernelStepGroup part of include/roaster_cuda.h).
//
// The reference runs one slot's model step at a time: step_forward (slots.c:864-880) takes the
// round-robin FairLock (slots.c:77-105) around model_forward, so with N slots decoding every
// hot-path call carries one slot's job and every projection reads its weights once per slot.
// Here the decoding slot threads meet in rounds; the i-th call of each member of a round is
// combined into one device batch, run by the member that arrives last (a combining barrier).
// Projections are regrouped by weight matrix: members that multiply the same matrix become the
// tokens of one multi-token product, gathered into a contiguous [T][cols] block by one copy-list
// launch, multiplied by kernel_cuda_matmul_quant_batch, and scattered back by a second launch.
//
// Host side. Arrival at a call is lock-free: a member writes its jobs into its own slot, then
// adds one to a single atomic word that packs (failed bit, members left in the round, members
// arrived at the open call); the arrival that makes arrived == left runs the batch, and so does
// an early kernel_step_group_end that makes left == arrived. Each waiting member sleeps on a
// futex word in its own slot; the runner releases the first kWakeFan waiters and every released
// member releases the next kWakeFan, so the wake-ups fan out over the host cores instead of
// queueing inside one thread's wake call. (With 64 slot threads on 16 host cores, arrivals
// through a mutex cost about 2.5 us each, in series: more than the device work of a layer.) A mutex guards only membership and round formation. Every
// wait is bounded: the straggler limit for a round to form, the call timeout for a call to fill
// (a waiter past it marks the call failed with a compare-and-swap that cannot succeed once the
// batch has a runner), the same timeout without progress for a running round to end. Device
// batches run under the group's FIFO lock (the FairLock counterpart), so work outside rounds
// that takes the same lock never overlaps them.
#include "runtime.h"
#include "../../include/roaster_cuda.h"

#include <linux/futex.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <climits>
#include <condition_variable>
#include <cstring>
#include <ctime>
#include <sched.h>
#include <mutex>
#include <unordered_map>
#include <vector>

using namespace rb;

namespace {

using Clock = std::chrono::steady_clock;

constexpr int kCopyMax = 512;   // copy-list entries per launch (10 KB of parameters)

struct CopyList {
    const float *src[kCopyMax];
    float *dst[kCopyMax];
    unsigned n[kCopyMax];       // floats
};

// One CTA per entry; 16-byte accesses when both ends and the length allow, else floats.
__global__ void __launch_bounds__(256) group_copy_kernel(const __grid_constant__ CopyList L)
{
    const int e = blockIdx.x;
    const float *s = L.src[e];
    float *d = L.dst[e];
    const unsigned n = L.n[e];
    if (((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d)) & 15u) == 0 && (n & 3u) == 0) {
        const float4 *s4 = reinterpret_cast<const float4 *>(s);
        float4 *d4 = reinterpret_cast<float4 *>(d);
        for (unsigned i = threadIdx.x; i < n / 4; i += blockDim.x)
            d4[i] = s4[i];
    } else {
        for (unsigned i = threadIdx.x; i < n; i += blockDim.x)
            d[i] = s[i];
    }
}

enum Kind { kAttn = 1, kDelta = 2, kMatvec = 3 };

struct Entry {
    int member;
    KernelCudaMatvecJob job;
};

// One member's submission to the open call (its own cache lines: no false sharing).
struct alignas(64) MemberSlot {
    std::atomic<uint32_t> go{0};     // futex: low bits of gen + 1 once this member's call is done
    std::atomic<int> sleeping{0};    // 1 while the member may be asleep on `go`
    int pos = 0;                     // place in the call's wake list
    uint64_t gen = ~0ull;            // call generation these jobs belong to
    int kind = 0, site = 0;
    KernelAttnDecodeJob attn;
    KernelDeltaStepJob delta;
    std::vector<KernelCudaMatvecJob> mv;
};

constexpr uint64_t kFailed = 1ull << 63;
constexpr uint64_t kLeftOne = 1ull << 32;
inline uint32_t w_arrived(uint64_t w) { return (uint32_t)w; }
inline uint32_t w_left(uint64_t w) { return (uint32_t)(w >> 32) & 0x7FFFFFFFu; }

}  // namespace

struct KernelStepGroup {
    int max_members = 0;
    long long straggler_us = 0;
    long long timeout_us = 0;

    // membership and round formation (mutex)
    mutable std::mutex m;
    std::condition_variable cv;
    std::vector<char> joined, pending, in_round;
    int n_joined = 0, n_pending = 0;
    Clock::time_point first_pending;
    bool round_active = false;
    int round_size = 0, round_ended = 0;
    std::atomic<uint64_t> round_id{0};

    // calls (lock-free arrival)
    std::vector<MemberSlot> slot;
    std::atomic<uint64_t> word{0};           // kFailed | left << 32 | arrived
    std::atomic<bool> round_failed{false};
    std::atomic<uint64_t> call_gen{0};       // completed (or failed) calls
    int call_status[16] = {};                // status of call generation c at [c & 15]
    std::vector<int> wake_list;              // the waiters of the last call run, in release order
    std::atomic<uint64_t> tree_gen{~0ull};   // the call generation wake_list belongs to

    // FIFO lock (ticket), the counterpart of the reference's FairLock
    std::mutex lm;
    std::condition_variable lc;
    unsigned long long next_ticket = 0, serving = 0;

    // device staging of merged projections (grow-only; used by the runner under the FIFO lock)
    float *xbuf = nullptr, *ybuf = nullptr;
    size_t xcap = 0, ycap = 0;

    KernelStepGroupStats st{};               // under m

    // Projection calls recorded as CUDA graphs (runner, under the FIFO lock). A call's key is its
    // job list: matrices, vectors, outputs and shapes in member order. Slots that keep their
    // buffers bring the same list every token, so from its third occurrence a layer's call
    // replays one graph instead of enqueueing its copy lists and matmul launches again.
    struct Recorded {
        std::vector<uintptr_t> key;
        cudaGraphExec_t exec = nullptr;
        uint64_t gen = 0;                    // Runtime::gen when recorded
        uint64_t plain_gen = ~0ull;          // Runtime::gen after its last plain run
        uint64_t launches = 0, products = 0, merged_jobs = 0;
    };
    std::unordered_map<uint64_t, Recorded> recorded;
    cudaStream_t rec_stream = nullptr;       // the stream recording happens on
};

namespace {

void fifo_lock(KernelStepGroup *g)
{
    std::unique_lock<std::mutex> l(g->lm);
    const unsigned long long t = g->next_ticket++;
    g->lc.wait(l, [&] { return g->serving == t; });
}

void fifo_unlock(KernelStepGroup *g)
{
    std::lock_guard<std::mutex> l(g->lm);
    g->serving++;
    g->lc.notify_all();
}

void futex_wait(std::atomic<uint32_t> *w, uint32_t v, long ns)
{
    timespec ts;
    ts.tv_sec = ns / 1000000000L;
    ts.tv_nsec = ns % 1000000000L;
    syscall(SYS_futex, reinterpret_cast<uint32_t *>(w), FUTEX_WAIT_PRIVATE, v, &ts, nullptr, 0);
}

#ifndef STEP_GROUP_WAKE_FAN
#define STEP_GROUP_WAKE_FAN 4
#endif
constexpr int kWakeFan = STEP_GROUP_WAKE_FAN;
#ifndef STEP_GROUP_SPIN_US
#define STEP_GROUP_SPIN_US 100
#endif
#ifndef STEP_GROUP_SPIN_YIELD
#define STEP_GROUP_SPIN_YIELD 1
#endif
constexpr long long kSpinUs = STEP_GROUP_SPIN_US;     // spin before sleeping on a call
constexpr bool kSpinYield = STEP_GROUP_SPIN_YIELD;   // yield the core on each spin

inline void cpu_relax()
{
#if defined(__x86_64__) || defined(__i386__)
    __builtin_ia32_pause();
#elif defined(__aarch64__)
    asm volatile("yield" ::: "memory");
#endif
}

// Release one waiter. The wake system call is made only when the waiter may be asleep: with
// sequentially consistent stores and loads on both sides (go then sleeping here, sleeping then
// go in the waiter), either the waiter sees go or this side sees sleeping.
void release(KernelStepGroup *g, int member, uint64_t gen)
{
    MemberSlot &s = g->slot[member];
    s.go.store((uint32_t)(gen + 1), std::memory_order_seq_cst);
    if (s.sleeping.load(std::memory_order_seq_cst))
        syscall(SYS_futex, reinterpret_cast<uint32_t *>(&s.go), FUTEX_WAKE_PRIVATE, 1, nullptr, nullptr, 0);
}

// A released waiter at place p of the wake list releases places kWakeFan (p + 1) .. + kWakeFan - 1
// (the runner took places 0 .. kWakeFan - 1).
void release_children(KernelStepGroup *g, int p, uint64_t gen)
{
    const int n = (int)g->wake_list.size();
    for (int c = kWakeFan * (p + 1); c < kWakeFan * (p + 2) && c < n; c++)
        release(g, g->wake_list[c], gen);
}

// Publish the result of call generation `gen` and release its waiters: through the wake tree
// when `waiters` lists them, else (a failed call) every member whose slot is in the call. Only
// the call's runner, or the waiter that failed it, calls this, once per call.
void complete(KernelStepGroup *g, uint64_t gen, int rc, uint64_t next_word, std::vector<int> *waiters)
{
    g->call_status[(gen + 1) & 15] = rc;
    if (waiters) {
        g->wake_list.swap(*waiters);
        for (int k = 0; k < (int)g->wake_list.size(); k++)
            g->slot[g->wake_list[k]].pos = k;
        g->tree_gen.store(gen, std::memory_order_release);
    }
    g->call_gen.store(gen + 1, std::memory_order_release);
    g->word.store(next_word, std::memory_order_release);
    if (waiters) {
        for (int k = 0; k < kWakeFan && k < (int)g->wake_list.size(); k++)
            release(g, g->wake_list[k], gen);
    } else {
        for (int i = 0; i < g->max_members; i++)
            if (g->slot[i].gen == gen)
                release(g, i, gen);
    }
    g->cv.notify_all();   // begin() watches the progress of a running round
}

int grow(float **buf, size_t *cap, size_t floats)
{
    if (floats <= *cap)
        return 0;
    // the previous buffer may still be read by queued work
    if (*buf) {
        if (check(cudaStreamSynchronize(rt().stream), "step group: stream sync") != 0)
            return -1;
        cudaFree(*buf);
        *buf = nullptr;
        *cap = 0;
    }
    size_t want = floats + floats / 2;
    if (check(cudaMalloc(reinterpret_cast<void **>(buf), want * sizeof(float)), "step group: cudaMalloc") != 0)
        return -1;
    *cap = want;
    rt().gen++;                      // recorded calls pointed to the old buffer
    return 0;
}

int copy_list(const std::vector<const float *> &src, const std::vector<float *> &dst, const std::vector<unsigned> &n)
{
    for (size_t i0 = 0; i0 < src.size(); i0 += kCopyMax) {
        CopyList L;
        memset(static_cast<void *>(&L), 0, sizeof(L));
        const size_t cnt = src.size() - i0 < (size_t)kCopyMax ? src.size() - i0 : (size_t)kCopyMax;
        for (size_t i = 0; i < cnt; i++) {
            L.src[i] = src[i0 + i];
            L.dst[i] = dst[i0 + i];
            L.n[i] = n[i0 + i];
        }
        group_copy_kernel<<<(unsigned)cnt, 256, 0, rt().stream>>>(L);
        if (launched("group_copy_kernel") != 0)
            return -1;
    }
    return 0;
}

// Regroup the members' projections by weight matrix; a matrix shared by T >= 2 members becomes
// one T-token product over gathered vectors. Counts go to `st` before any device work, so the
// plan is observable without a GPU.
int enqueue_matvec(KernelStepGroup *g, const std::vector<Entry> &mv, KernelStepGroupStats *st)
{
    struct Group {
        KernelCudaMatvecJob key;
        std::vector<int> idx;
    };
    std::vector<Group> groups;
    for (int i = 0; i < (int)mv.size(); i++) {
        const KernelCudaMatvecJob &j = mv[i].job;
        bool found = false;
        for (Group &gr : groups)
            if (gr.key.matrix == j.matrix && gr.key.is_q6 == j.is_q6 && gr.key.rows == j.rows && gr.key.cols == j.cols) {
                gr.idx.push_back(i);
                found = true;
                break;
            }
        if (!found)
            groups.push_back(Group{j, {i}});
    }
    // A layer's projections usually read the same input (q/k/v, or qkv/z/alpha/beta): matrices
    // whose members bring the same vectors, in the same order, share one gathered block, and the
    // matmul then prepares that block's activations once.
    struct XBlock {
        size_t cols, off;
        std::vector<const float *> vecs;
        bool gathered;
    };
    std::vector<XBlock> xblocks;
    std::vector<int> gxb(groups.size(), -1);
    size_t xfl = 0, yfl = 0;
    for (size_t q = 0; q < groups.size(); q++) {
        const Group &gr = groups[q];
        if (gr.idx.size() < 2)
            continue;
        st->products++;
        st->merged_jobs += gr.idx.size();
        yfl += ((gr.idx.size() * gr.key.rows + 3) & ~(size_t)3);
        std::vector<const float *> vecs;
        for (int i : gr.idx)
            vecs.push_back(mv[i].job.vector);
        int b = -1;
        for (size_t k = 0; k < xblocks.size() && b < 0; k++)
            if (xblocks[k].cols == gr.key.cols && xblocks[k].vecs == vecs)
                b = (int)k;
        if (b < 0) {
            xblocks.push_back(XBlock{gr.key.cols, xfl, std::move(vecs), false});
            b = (int)xblocks.size() - 1;
            xfl += gr.idx.size() * gr.key.cols;
        }
        gxb[q] = b;
    }
    if (ensure() != 0)
        return -1;
    for (const Entry &e : mv)
        if (!e.job.matrix || !e.job.vector || !e.job.output || e.job.rows == 0 || e.job.cols == 0 || e.job.cols % 256 != 0)
            return fail("kernel_step_group_matvec: member %d has an invalid job", e.member);
    {
        // First choice: the merged products read each member's vector and write each member's
        // output in place (per-token row tables of the tensor-core matmul), with no gather into
        // or scatter out of the group's staging. The matmul launches nothing and returns 1 when
        // a product cannot run that way (too few tokens for the tensor-core path, a vector not
        // 16-byte aligned); the gathered form below then runs instead.
        std::vector<KernelCudaMatmulJob> rj;
        std::vector<MmRows> rr;
        std::vector<std::vector<float *>> youts(groups.size());
        for (size_t q = 0; q < groups.size(); q++) {
            const Group &gr = groups[q];
            const KernelCudaMatvecJob &k = gr.key;
            if (gr.idx.size() == 1) {
                const KernelCudaMatvecJob &j = mv[gr.idx[0]].job;
                rj.push_back(KernelCudaMatmulJob{j.is_q6, j.matrix, j.vector, j.output, j.rows, j.cols, 1});
                rr.push_back(MmRows{nullptr, nullptr});
                continue;
            }
            for (int i : gr.idx)
                youts[q].push_back(mv[i].job.output);
            const XBlock &xb = xblocks[gxb[q]];
            // X and Y name the first token's rows; the tables carry every token's
            rj.push_back(KernelCudaMatmulJob{k.is_q6, k.matrix, xb.vecs[0], youts[q][0], k.rows, k.cols,
                                             gr.idx.size()});
            rr.push_back(MmRows{xb.vecs.data(), youts[q].data()});
        }
        const int rc = matmul_quant_rows(rj.data(), (int)rj.size(), rr.data());
        if (rc != 1)
            return rc;
    }
    if (grow(&g->xbuf, &g->xcap, xfl) != 0 || grow(&g->ybuf, &g->ycap, yfl) != 0)
        return -1;
    std::vector<KernelCudaMatmulJob> jobs;
    std::vector<const float *> gs, ss;
    std::vector<float *> gd, sd;
    std::vector<unsigned> gn, sn;
    size_t yo = 0;
    for (size_t q = 0; q < groups.size(); q++) {
        const Group &gr = groups[q];
        const KernelCudaMatvecJob &k = gr.key;
        if (gr.idx.size() == 1) {
            const KernelCudaMatvecJob &j = mv[gr.idx[0]].job;
            jobs.push_back(KernelCudaMatmulJob{j.is_q6, j.matrix, j.vector, j.output, j.rows, j.cols, 1});
            continue;
        }
        const size_t T = gr.idx.size();
        XBlock &xb = xblocks[gxb[q]];
        float *X = g->xbuf + xb.off, *Y = g->ybuf + yo;
        for (size_t t = 0; t < T; t++) {
            const KernelCudaMatvecJob &j = mv[gr.idx[t]].job;
            if (!xb.gathered) {
                gs.push_back(j.vector);
                gd.push_back(X + t * k.cols);
                gn.push_back((unsigned)k.cols);
            }
            ss.push_back(Y + t * k.rows);
            sd.push_back(j.output);
            sn.push_back((unsigned)k.rows);
        }
        xb.gathered = true;
        jobs.push_back(KernelCudaMatmulJob{k.is_q6, k.matrix, X, Y, k.rows, k.cols, T});
        yo += (T * k.rows + 3) & ~(size_t)3;
    }
    if (copy_list(gs, gd, gn) != 0)
        return -1;
    if (kernel_cuda_matmul_quant_batch(jobs.data(), (int)jobs.size()) != 0)
        return -1;
    return copy_list(ss, sd, sn);
}

bool recording_enabled()
{
    static const bool on = [] {
        const char *e = getenv("ROASTER_STEP_GRAPHS");
        return !(e && e[0] == '0');
    }();
    return on;
}

void drop_recorded(KernelStepGroup *g)
{
    for (auto &kv : g->recorded)
        if (kv.second.exec)
            cudaGraphExecDestroy(kv.second.exec);
    g->recorded.clear();
}

// A projection call: the first occurrence of a job list runs as plain launches (it sets up the
// buffers and tensor maps it needs), the second is recorded into a CUDA graph and launched, later
// ones replay the graph while the library's buffers are the ones it was recorded with. After the
// buffers change, the list runs plainly once more before it is recorded again. Where recording
// fails the call runs as plain launches.
int run_matvec(KernelStepGroup *g, const std::vector<Entry> &mv, KernelStepGroupStats *st)
{
    if (!recording_enabled())
        return enqueue_matvec(g, mv, st);
    std::vector<uintptr_t> key;
    key.reserve(mv.size() * 6);
    for (const Entry &e : mv) {
        const KernelCudaMatvecJob &j = e.job;
        key.push_back(reinterpret_cast<uintptr_t>(j.matrix));
        key.push_back(reinterpret_cast<uintptr_t>(j.vector));
        key.push_back(reinterpret_cast<uintptr_t>(j.output));
        key.push_back((uintptr_t)j.rows);
        key.push_back((uintptr_t)j.cols);
        key.push_back((uintptr_t)j.is_q6);
    }
    uint64_t h = 1469598103934665603ull;                 // FNV-1a over the key words
    for (const uintptr_t v : key) {
        h ^= (uint64_t)v;
        h *= 1099511628211ull;
    }
    if (g->recorded.size() >= 512 && !g->recorded.count(h))
        drop_recorded(g);
    KernelStepGroup::Recorded &r = g->recorded[h];
    if (r.key != key) {                                  // new, or another list with the same hash
        if (r.exec)
            cudaGraphExecDestroy(r.exec);
        r = KernelStepGroup::Recorded();
        r.key = std::move(key);
    }
    Runtime &R = rt();
    const uint64_t gen = R.gen;
    if (r.exec && r.gen == gen) {
        if (check(cudaGraphLaunch(r.exec, R.stream), "step group: graph launch") != 0)
            return -1;
        count_launches(r.launches);
        st->products += r.products;
        st->merged_jobs += r.merged_jobs;
        st->replayed++;
        return 0;
    }
    if (r.exec) {                                        // recorded with buffers since replaced
        cudaGraphExecDestroy(r.exec);
        r.exec = nullptr;
    }
    if (r.plain_gen != gen) {
        // Not yet run with the library's current buffers: run plainly (it allocates whatever it
        // needs), so that a recording made at the next occurrence allocates nothing -- an
        // allocation, a free or a synchronisation cannot be part of a capture.
        const int rc = enqueue_matvec(g, mv, st);
        r.plain_gen = R.gen;
        return rc;
    }
    if (!g->rec_stream && cudaStreamCreateWithFlags(&g->rec_stream, cudaStreamNonBlocking) != cudaSuccess) {
        (void)cudaGetLastError();
        g->rec_stream = nullptr;
        return enqueue_matvec(g, mv, st);
    }
    KernelStepGroupStats loc{};
    const uint64_t l0 = kernel_cuda_launch_count();
    bool ok = cudaStreamBeginCapture(g->rec_stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
    if (ok) {
        const cudaStream_t saved = R.stream;
        R.stream = g->rec_stream;                        // the launches below go into the recording
        const int rc = enqueue_matvec(g, mv, &loc);
        R.stream = saved;
        cudaGraph_t graph = nullptr;
        const bool ended = cudaStreamEndCapture(g->rec_stream, &graph) == cudaSuccess;
        ok = rc == 0 && ended && graph && R.gen == gen &&
             cudaGraphInstantiate(&r.exec, graph, 0) == cudaSuccess;
        if (graph)
            cudaGraphDestroy(graph);
    }
    (void)cudaGetLastError();                            // a failed recording leaves no error behind
    const uint64_t recorded_launches = kernel_cuda_launch_count() - l0;
    if (!ok) {
        if (r.exec)
            cudaGraphExecDestroy(r.exec);
        r.exec = nullptr;
        count_launches((uint64_t)0 - recorded_launches);  // nothing of the recording ran
        return enqueue_matvec(g, mv, st);
    }
    r.gen = gen;
    r.launches = recorded_launches;                      // counted already, run by the launch below
    r.products = loc.products;
    r.merged_jobs = loc.merged_jobs;
    st->products += loc.products;
    st->merged_jobs += loc.merged_jobs;
    return check(cudaGraphLaunch(r.exec, R.stream), "step group: graph launch");
}

// Run call generation `gen`: every member still in the round has submitted to its slot. The
// caller is the unique runner (its atomic update of the word made arrived == left).
void run_call(KernelStepGroup *g, uint64_t gen, int self)
{
    std::vector<KernelAttnDecodeJob> attn;
    std::vector<KernelDeltaStepJob> delta;
    std::vector<Entry> mv;
    std::vector<int> waiters;
    int kind = 0, site = 0, mismatch = 0, n = 0;
    for (int i = 0; i < g->max_members; i++) {
        const MemberSlot &s = g->slot[i];
        if (s.gen != gen)
            continue;
        if (i != self)
            waiters.push_back(i);
        if (n++ == 0) {
            kind = s.kind;
            site = s.site;
        } else if (s.kind != kind || s.site != site) {
            mismatch = 1;
        }
        if (s.kind == kAttn)
            attn.push_back(s.attn);
        else if (s.kind == kDelta)
            delta.push_back(s.delta);
        else
            for (const KernelCudaMatvecJob &j : s.mv)
                mv.push_back(Entry{i, j});
    }
    KernelStepGroupStats plan{};
    int rc = 0;
    if (mismatch) {
        rc = fail("kernel_step_group: members of a round reached different calls (site %d and others)", site);
        g->round_failed.store(true, std::memory_order_release);
    } else {
        fifo_lock(g);
        if (kind == kAttn)
            rc = kernel_attn_decode_batch(attn.data(), (int)attn.size());
        else if (kind == kDelta)
            rc = kernel_deltanet_step_batch(delta.data(), (int)delta.size());
        else
            rc = run_matvec(g, mv, &plan);
        fifo_unlock(g);
    }
    {
        std::lock_guard<std::mutex> l(g->m);
        if (!mismatch) {
            g->st.calls++;
            g->st.jobs += kind == kAttn ? attn.size() : kind == kDelta ? delta.size() : mv.size();
            g->st.products += plan.products;
            g->st.merged_jobs += plan.merged_jobs;
            g->st.replayed += plan.replayed;
        }
        if (rc != 0)
            g->st.errors++;
    }
    // nobody else can change the word now: every member still in the round is waiting here
    const uint64_t w = g->word.load(std::memory_order_acquire);
    complete(g, gen, rc, w & ~(uint64_t)0xFFFFFFFFu, &waiters);
}

// A waiter past its deadline: fail call `gen` unless it completed or has its runner.
void try_fail(KernelStepGroup *g, uint64_t gen, int site, const char *what)
{
    for (;;) {
        uint64_t w = g->word.load(std::memory_order_acquire);
        if (g->call_gen.load(std::memory_order_acquire) != gen)
            return;                                  // completed meanwhile
        if ((w & kFailed) || w_arrived(w) == w_left(w))
            return;                                  // already failed, or the batch is running
        const uint64_t seen = w;
        if (g->word.compare_exchange_weak(w, seen | kFailed, std::memory_order_acq_rel)) {
            fail("%s: not every member reached call site %d within the call timeout", what, site);
            g->round_failed.store(true, std::memory_order_release);
            {
                std::lock_guard<std::mutex> l(g->m);
                g->st.errors++;
            }
            // the failed bit stays until the round ends: late arrivals return at once
            complete(g, gen, -1, (seen & ~(uint64_t)0xFFFFFFFFu) | kFailed, nullptr);
            return;
        }
    }
}

template <typename Fill>
int rendezvous(KernelStepGroup *g, int member, int kind, int site, const char *what, Fill fill)
{
    if (!g)
        return fail("%s: null group", what);
    // joined / in_round of this member change only on this member's own thread
    if (member < 0 || member >= g->max_members || !g->joined[member] || !g->in_round[member])
        return fail("%s: member %d is not in a round", what, member);
    if (g->round_failed.load(std::memory_order_acquire))
        return fail("%s: an earlier call of this round failed", what);
    // the open call cannot complete before this member arrives (it can only fail)
    const uint64_t gen = g->call_gen.load(std::memory_order_acquire);
    MemberSlot &s = g->slot[member];
    s.kind = kind;
    s.site = site;
    fill(s);
    s.gen = gen;
    const uint64_t w = g->word.fetch_add(1, std::memory_order_acq_rel) + 1;
    if (w & kFailed) {
        s.gen = ~0ull;   // never part of a later call (the next round forms after this member ends)
        return fail("%s: an earlier call of this round failed", what);
    }
    if (w_arrived(w) == w_left(w)) {
        run_call(g, gen, member);
        return g->call_status[(gen + 1) & 15];
    }
    const Clock::time_point deadline = Clock::now() + std::chrono::microseconds(g->timeout_us);
    const uint32_t done = (uint32_t)(gen + 1);
    // Spin first: a thread woken from a futex takes tens of microseconds to run again, which on a
    // combined call of tens of members costs more than the device work of a layer.
    const Clock::time_point spin_end = Clock::now() + std::chrono::microseconds(kSpinUs);
    for (int i = 1; s.go.load(std::memory_order_acquire) != done; i++) {
        if (kSpinYield)
            sched_yield();
        else
            cpu_relax();
        if ((i & 63) == 0 && Clock::now() >= spin_end)
            break;
    }
    for (;;) {
        const uint32_t v = s.go.load(std::memory_order_acquire);
        if (v == done)
            break;
        s.sleeping.store(1, std::memory_order_seq_cst);
        if (s.go.load(std::memory_order_seq_cst) == v)
            futex_wait(&s.go, v, 2000000L);   // 2 ms slices
        s.sleeping.store(0, std::memory_order_relaxed);
        if (s.go.load(std::memory_order_acquire) != done && Clock::now() >= deadline)
            try_fail(g, gen, site, what);
    }
    if (g->tree_gen.load(std::memory_order_acquire) == gen)
        release_children(g, s.pos, gen);
    const int rc = g->call_status[(gen + 1) & 15];
    if (rc != 0)
        fail("%s: the combined call failed", what);
    return rc;
}

}  // namespace

extern "C" KernelStepGroup *kernel_step_group_create(int max_members, long long straggler_us, long long call_timeout_ms)
{
    if (max_members < 1 || max_members > 4096 || straggler_us < 0 || call_timeout_ms <= 0) {
        fail("kernel_step_group_create: bad arguments");
        return nullptr;
    }
    KernelStepGroup *g = new KernelStepGroup;
    g->max_members = max_members;
    g->straggler_us = straggler_us;
    g->timeout_us = call_timeout_ms * 1000;
    g->joined.assign(max_members, 0);
    g->pending.assign(max_members, 0);
    g->in_round.assign(max_members, 0);
    g->slot = std::vector<MemberSlot>(max_members);
    return g;
}

extern "C" void kernel_step_group_destroy(KernelStepGroup *g)
{
    if (!g)
        return;
    if (g->xbuf || g->ybuf || !g->recorded.empty()) {
        if (rt().device >= 0)
            cudaStreamSynchronize(rt().stream);
        drop_recorded(g);
        cudaFree(g->xbuf);
        cudaFree(g->ybuf);
    }
    if (g->rec_stream)
        cudaStreamDestroy(g->rec_stream);
    delete g;
}

extern "C" int kernel_step_group_join(KernelStepGroup *g)
{
    if (!g)
        return fail("kernel_step_group_join: null group");
    std::lock_guard<std::mutex> l(g->m);
    for (int i = 0; i < g->max_members; i++)
        if (!g->joined[i]) {
            g->joined[i] = 1;
            g->n_joined++;
            g->st.members = g->n_joined;
            g->cv.notify_all();
            return i;
        }
    return fail("kernel_step_group_join: all %d member places are taken", g->max_members);
}

extern "C" int kernel_step_group_leave(KernelStepGroup *g, int member)
{
    if (!g)
        return fail("kernel_step_group_leave: null group");
    std::lock_guard<std::mutex> l(g->m);
    if (member < 0 || member >= g->max_members || !g->joined[member])
        return fail("kernel_step_group_leave: member %d is not joined", member);
    if (g->in_round[member])
        return fail("kernel_step_group_leave: member %d is inside a round (end it first)", member);
    if (g->pending[member]) {
        g->pending[member] = 0;
        g->n_pending--;
    }
    g->joined[member] = 0;
    g->n_joined--;
    g->st.members = g->n_joined;
    g->cv.notify_all();   // the waiting members may now be everyone
    return 0;
}

extern "C" int kernel_step_group_begin(KernelStepGroup *g, int member)
{
    if (!g)
        return fail("kernel_step_group_begin: null group");
    std::unique_lock<std::mutex> l(g->m);
    if (member < 0 || member >= g->max_members || !g->joined[member])
        return fail("kernel_step_group_begin: member %d is not joined", member);
    if (g->in_round[member] || g->pending[member])
        return fail("kernel_step_group_begin: member %d has already begun", member);
    g->pending[member] = 1;
    if (g->n_pending++ == 0)
        g->first_pending = Clock::now();
    g->cv.notify_all();
    // bound on waiting for a running round: a call timeout without any progress of that round
    Clock::time_point give_up = Clock::now() + std::chrono::microseconds(g->timeout_us);
    uint64_t seen_gen = g->call_gen.load(), seen_round = g->round_id.load();
    for (;;) {
        const uint64_t cg = g->call_gen.load(), rid = g->round_id.load();
        if (cg != seen_gen || rid != seen_round) {
            seen_gen = cg;
            seen_round = rid;
            give_up = Clock::now() + std::chrono::microseconds(g->timeout_us);
        }
        if (g->in_round[member])
            return g->round_size;
        if (!g->round_active) {
            const Clock::time_point form = g->first_pending + std::chrono::microseconds(g->straggler_us);
            if (g->n_pending == g->n_joined || Clock::now() >= form) {
                g->round_active = true;
                g->round_size = g->n_pending;
                g->round_ended = 0;
                for (int i = 0; i < g->max_members; i++)
                    if (g->pending[i]) {
                        g->pending[i] = 0;
                        g->in_round[i] = 1;
                    }
                g->n_pending = 0;
                g->round_failed.store(false, std::memory_order_relaxed);
                g->word.store((uint64_t)g->round_size << 32, std::memory_order_release);
                g->round_id.fetch_add(1);
                g->st.rounds++;
                if (g->round_size > g->st.max_round)
                    g->st.max_round = g->round_size;
                g->cv.notify_all();
                return g->round_size;
            }
            g->cv.wait_until(l, form);
        } else {
            // completions notify without the mutex, so poll in short slices as well
            const Clock::time_point slice = Clock::now() + std::chrono::milliseconds(2);
            g->cv.wait_until(l, give_up < slice ? give_up : slice);
            if (Clock::now() >= give_up && !g->in_round[member] && g->round_active &&
                g->call_gen.load() == seen_gen && g->round_id.load() == seen_round) {
                g->pending[member] = 0;
                if (--g->n_pending == 0)
                    g->first_pending = Clock::time_point();
                return fail("kernel_step_group_begin: the running round did not end within the call timeout");
            }
        }
    }
}

extern "C" int kernel_step_group_end(KernelStepGroup *g, int member)
{
    if (!g)
        return fail("kernel_step_group_end: null group");
    std::unique_lock<std::mutex> l(g->m);
    if (member < 0 || member >= g->max_members || !g->joined[member] || !g->in_round[member])
        return fail("kernel_step_group_end: member %d is not in a round", member);
    g->in_round[member] = 0;
    const uint64_t w = g->word.fetch_sub(kLeftOne, std::memory_order_acq_rel) - kLeftOne;
    if (++g->round_ended == g->round_size) {
        g->round_active = false;
        g->word.store(0, std::memory_order_release);
        if (g->n_pending > 0)   // members that began meanwhile count their straggler limit from now
            g->first_pending = Clock::now();
        g->cv.notify_all();
        return 0;
    }
    g->cv.notify_all();
    const bool runner = !(w & kFailed) && w_arrived(w) > 0 && w_arrived(w) == w_left(w);
    const uint64_t gen = g->call_gen.load(std::memory_order_acquire);
    l.unlock();
    if (runner)   // the members still in the round are all waiting at the open call
        run_call(g, gen, -1);
    return 0;
}

extern "C" int kernel_step_group_attn(KernelStepGroup *g, int member, int site, const KernelAttnDecodeJob *job)
{
    if (!job)
        return fail("kernel_step_group_attn: null job");
    return rendezvous(g, member, kAttn, site, "kernel_step_group_attn", [&](MemberSlot &s) { s.attn = *job; });
}

extern "C" int kernel_step_group_delta(KernelStepGroup *g, int member, int site, const KernelDeltaStepJob *job)
{
    if (!job)
        return fail("kernel_step_group_delta: null job");
    return rendezvous(g, member, kDelta, site, "kernel_step_group_delta", [&](MemberSlot &s) { s.delta = *job; });
}

extern "C" int kernel_step_group_matvec(KernelStepGroup *g, int member, int site, const KernelCudaMatvecJob *jobs, int n)
{
    if (!jobs || n < 1)
        return fail("kernel_step_group_matvec: bad job array");
    return rendezvous(g, member, kMatvec, site, "kernel_step_group_matvec",
                      [&](MemberSlot &s) { s.mv.assign(jobs, jobs + n); });
}

extern "C" int kernel_step_group_lock(KernelStepGroup *g)
{
    if (!g)
        return fail("kernel_step_group_lock: null group");
    fifo_lock(g);
    return 0;
}

extern "C" int kernel_step_group_unlock(KernelStepGroup *g)
{
    if (!g)
        return fail("kernel_step_group_unlock: null group");
    fifo_unlock(g);
    return 0;
}

extern "C" int kernel_step_group_stats(const KernelStepGroup *g, KernelStepGroupStats *out)
{
    if (!g || !out)
        return fail("kernel_step_group_stats: null argument");
    std::lock_guard<std::mutex> l(g->m);
    *out = g->st;
    return 0;
}
