// Runtime and the lifecycle / residency part of the C-ABI (include/roaster_cuda.h).
#include "runtime.h"
#include <cuda_fp16.h>
#include "ptx.cuh"
#include "../../include/roaster_cuda.h"

#include <omp.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <vector>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace rb {

static Runtime g_rt;
static char g_err[512] = "";
static std::atomic<uint64_t> g_launches{0};

Runtime &rt() { return g_rt; }

bool pdl_enabled()
{
    static const bool on = [] {
        const char *e = getenv("ROASTER_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

int fail(const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return -1;
}

int check(cudaError_t e, const char *what)
{
    if (e == cudaSuccess)
        return 0;
    return fail("%s: %s", what, cudaGetErrorString(e));
}

void count_launches(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int launched(const char *what)
{
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check(cudaGetLastError(), what);
}

static int init_device(int device)
{
    int count = 0;
    if (check(cudaGetDeviceCount(&count), "cudaGetDeviceCount") != 0)
        return -1;
    if (device < 0 || device >= count)
        return fail("kernel_cuda_init: device %d not present (%d devices)", device, count);
    cudaDeviceProp prop;
    if (check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties") != 0)
        return -1;
    if (prop.major != 10)
        return fail("kernel_cuda_init: device %d is sm_%d%d; this library is built for sm_100a",
                    device, prop.major, prop.minor);
    if (check(cudaSetDevice(device), "cudaSetDevice") != 0)
        return -1;
    unsigned *err = nullptr;
    if (check(cudaMalloc(&err, 256), "cudaMalloc(error word)") != 0)
        return -1;
    if (check(cudaMemset(err, 0, 256), "cudaMemset(error word)") != 0) {
        cudaFree(err);
        return -1;
    }
    unsigned *err_host = nullptr;
    if (check(cudaHostAlloc(&err_host, 64, cudaHostAllocDefault), "cudaHostAlloc(error word copy)") != 0) {
        cudaFree(err);
        return -1;
    }
    g_rt.device = device;
    g_rt.num_sms = prop.multiProcessorCount;
    g_rt.err_word = err;
    g_rt.err_host = err_host;
    // RoPE inverse frequencies with the host libm powf, the same call the reference makes
    // (apply_rope_64, model.c:765), so both sides rotate by bit-identical angles.
    for (int j = 0; j < 32; j++)
        g_rt.inv_freq[j] = powf(10000000.0f, -2.0f * (float)j / 64.0f);
    return 0;
}

// Jobs [i0, i1) on up to 8 host threads (OpenMP, like the reference's own host code); serial
// for a handful of jobs, where starting threads costs more than the copies.
static void par_jobs(int i0, int i1, const std::function<void(int)> &f)
{
    const int n = i1 - i0;
    const int nt = std::min(std::min(8, omp_get_max_threads()), n / 2);
    if (nt <= 1) {
        for (int i = i0; i < i1; i++)
            f(i);
        return;
    }
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int i = i0; i < i1; i++)
        f(i);
}

constexpr int kStageChunks = 4;

static int stage_events(cudaEvent_t **out)
{
    static cudaEvent_t ev[kStageChunks];
    static int made = -1;                      // device the events were made on
    if (made != g_rt.device) {
        for (int c = 0; c < kStageChunks; c++)
            if (check(cudaEventCreateWithFlags(&ev[c], cudaEventDisableTiming), "cudaEventCreate") != 0)
                return -1;
        made = g_rt.device;
    }
    *out = ev;
    return 0;
}

static inline int stage_chunks(int n) { return n >= 4 * kStageChunks ? kStageChunks : 1; }

int stage_in(float *h, float *d, int n, size_t per, const std::function<void(int, float *)> &fill)
{
    const int chunks = stage_chunks(n);
    for (int c = 0; c < chunks; c++) {
        const int i0 = (int)((long long)n * c / chunks), i1 = (int)((long long)n * (c + 1) / chunks);
        par_jobs(i0, i1, [&](int i) { fill(i, h + (size_t)i * per); });
        if (check(cudaMemcpyAsync(d + (size_t)i0 * per, h + (size_t)i0 * per, (size_t)(i1 - i0) * per * sizeof(float),
                                  cudaMemcpyHostToDevice, g_rt.stream),
                  "stage in") != 0)
            return -1;
    }
    return 0;
}

int stage_out(float *h, const float *d, int n, size_t per, const std::function<void(int, const float *)> &drain)
{
    const int chunks = stage_chunks(n);
    cudaEvent_t *ev = nullptr;
    if (stage_events(&ev) != 0)
        return -1;
    for (int c = 0; c < chunks; c++) {
        const int i0 = (int)((long long)n * c / chunks), i1 = (int)((long long)n * (c + 1) / chunks);
        if (check(cudaMemcpyAsync(h + (size_t)i0 * per, d + (size_t)i0 * per, (size_t)(i1 - i0) * per * sizeof(float),
                                  cudaMemcpyDeviceToHost, g_rt.stream),
                  "stage out") != 0 ||
            check(cudaEventRecord(ev[c], g_rt.stream), "cudaEventRecord") != 0)
            return -1;
    }
    for (int c = 0; c < chunks; c++) {
        const int i0 = (int)((long long)n * c / chunks), i1 = (int)((long long)n * (c + 1) / chunks);
        if (check(cudaEventSynchronize(ev[c]), "stage out") != 0)
            return -1;
        par_jobs(i0, i1, [&](int i) { drain(i, h + (size_t)i * per); });
    }
    return 0;
}

int ensure()
{
    if (g_rt.device < 0 && init_device(0) != 0)
        return -1;
    return check(cudaSetDevice(g_rt.device), "cudaSetDevice");
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn()
{
    static EncodeTiledFn encode = nullptr;
    if (!encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    return encode;
}

int encode_tmap_f16_3d(CUtensorMap *map, const void *base, const uint64_t dims[3], const uint64_t strides[2],
                       const uint32_t box[3])
{
    const EncodeTiledFn encode = encode_fn();
    if (!encode)
        return fail("cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t gd[3] = {dims[0], dims[1], dims[2]};
    const cuuint64_t gs[2] = {strides[0], strides[1]};
    const cuuint32_t bd[3] = {box[0], box[1], box[2]};
    const cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), gd, gs, bd, es,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 0;
}

int encode_tmap_u8_2d(CUtensorMap *map, const void *base, uint64_t dim0, uint64_t dim1, uint64_t stride1,
                      uint32_t box0, uint32_t box1)
{
    const EncodeTiledFn encode = encode_fn();
    if (!encode)
        return fail("cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t gd[2] = {dim0, dim1};
    const cuuint64_t gs[1] = {stride1};
    const cuuint32_t bd[2] = {box0, box1};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), gd, gs, bd, es,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 0;
}

void *scratch(size_t bytes)
{
    if (bytes <= g_rt.scratch_bytes)
        return g_rt.scratch;
    if (g_rt.scratch) {
        cudaStreamSynchronize(g_rt.stream);
        cudaFree(g_rt.scratch);
        g_rt.scratch = nullptr;
        g_rt.scratch_bytes = 0;
    }
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes + bytes / 4;
    void *p = nullptr;
    if (check(cudaMalloc(&p, want), "cudaMalloc(scratch)") != 0)
        return nullptr;
    g_rt.scratch = p;
    g_rt.gen++;
    g_rt.scratch_bytes = want;
    return p;
}

void *dstage(size_t bytes)
{
    if (bytes <= g_rt.dstage_bytes)
        return g_rt.dstage;
    if (g_rt.dstage) {
        cudaStreamSynchronize(g_rt.stream);
        cudaFree(g_rt.dstage);
        g_rt.dstage = nullptr;
        g_rt.dstage_bytes = 0;
    }
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes + bytes / 4;
    void *p = nullptr;
    if (check(cudaMalloc(&p, want), "cudaMalloc(staging)") != 0)
        return nullptr;
    g_rt.dstage = p;
    g_rt.gen++;
    g_rt.dstage_bytes = want;
    return p;
}

cudaStream_t copy_stream()
{
    if (!g_rt.copy_stream &&
        check(cudaStreamCreateWithFlags(&g_rt.copy_stream, cudaStreamNonBlocking), "cudaStreamCreate(copy)") != 0)
        return nullptr;
    return g_rt.copy_stream;
}

cudaStream_t out_stream()
{
    if (!g_rt.out_stream &&
        check(cudaStreamCreateWithFlags(&g_rt.out_stream, cudaStreamNonBlocking), "cudaStreamCreate(out)") != 0)
        return nullptr;
    return g_rt.out_stream;
}

int *counters(size_t n)
{
    if (n <= g_rt.counters_n)
        return g_rt.counters;
    if (g_rt.counters) {
        cudaStreamSynchronize(g_rt.stream);
        cudaFree(g_rt.counters);
        g_rt.counters = nullptr;
        g_rt.counters_n = 0;
    }
    size_t want = n < 4096 ? 4096 : n * 2;
    int *p = nullptr;
    if (check(cudaMalloc(&p, want * sizeof(int)), "cudaMalloc(counters)") != 0)
        return nullptr;
    if (check(cudaMemset(p, 0, want * sizeof(int)), "cudaMemset(counters)") != 0) {
        cudaFree(p);
        return nullptr;
    }
    g_rt.counters = p;
    g_rt.gen++;
    g_rt.counters_n = want;
    return p;
}

void *pinned(size_t bytes)
{
    if (bytes <= g_rt.pinned_bytes)
        return g_rt.pinned;
    if (g_rt.pinned) {
        cudaStreamSynchronize(g_rt.stream);
        cudaFreeHost(g_rt.pinned);
        g_rt.pinned = nullptr;
        g_rt.pinned_bytes = 0;
    }
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes + bytes / 4;
    void *p = nullptr;
    if (check(cudaHostAlloc(&p, want, cudaHostAllocDefault), "cudaHostAlloc(staging)") != 0)
        return nullptr;
    g_rt.pinned = p;
    g_rt.pinned_bytes = want;
    return p;
}


// Host buffers registered by the caller (pinned), sorted by start address. The host-buffer entry
// points move such buffers with the copy engine directly, without a staging memcpy.
struct HostRange {
    uintptr_t lo, hi;
};
static std::mutex g_reg_mu;
static std::vector<HostRange> g_reg;

bool host_registered(const void *p, size_t bytes)
{
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    std::lock_guard<std::mutex> lk(g_reg_mu);
    auto it = std::upper_bound(g_reg.begin(), g_reg.end(), a,
                               [](uintptr_t x, const HostRange &r) { return x < r.lo; });
    if (it == g_reg.begin())
        return false;
    --it;
    return a >= it->lo && a + bytes <= it->hi && a + bytes >= a;
}

void HostRuns::build(size_t gap)
{
    std::sort(segs.begin(), segs.end());
    runs.clear();
    for (const auto &s : segs) {
        if (!runs.empty() && s.first <= runs.back().hi + gap)
            runs.back().hi = std::max(runs.back().hi, s.second);
        else
            runs.push_back(Run{s.first, s.second, 0});
    }
    // each run starts in staging at its host address modulo 16, so pointers keep their alignment
    bytes = 0;
    for (auto &r : runs) {
        r.off = ((bytes + 15) & ~(size_t)15) + (r.lo & 15);
        bytes = r.off + (r.hi - r.lo);
    }
}

size_t HostRuns::offset(const void *p) const
{
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    auto it = std::upper_bound(runs.begin(), runs.end(), a, [](uintptr_t x, const Run &r) { return x < r.lo; });
    if (it == runs.begin())                      // callers only ask for pointers they added
        return 0;
    --it;
    return it->off + (a - it->lo);
}

bool runs_overlap(const HostRuns &a, const HostRuns &b)
{
    size_t i = 0, j = 0;                          // both run lists are sorted and disjoint
    while (i < a.runs.size() && j < b.runs.size()) {
        if (a.runs[i].hi <= b.runs[j].lo)
            i++;
        else if (b.runs[j].hi <= a.runs[i].lo)
            j++;
        else
            return true;
    }
    return false;
}

int runs_copy(const HostRuns &r, char *d, cudaMemcpyKind kind, cudaStream_t st)
{
    for (const auto &x : r.runs) {
        void *h = reinterpret_cast<void *>(x.lo);
        const cudaError_t e = kind == cudaMemcpyHostToDevice
                                  ? cudaMemcpyAsync(d + x.off, h, x.hi - x.lo, kind, st)
                                  : cudaMemcpyAsync(h, d + x.off, x.hi - x.lo, kind, st);
        if (check(e, kind == cudaMemcpyHostToDevice ? "copy in" : "copy out") != 0)
            return -1;
    }
    return 0;
}

int runs_h2d(const HostRuns &r, char *d) { return runs_copy(r, d, cudaMemcpyHostToDevice, g_rt.stream); }

int runs_d2h(const HostRuns &r, const char *d)
{
    return runs_copy(r, const_cast<char *>(d), cudaMemcpyDeviceToHost, g_rt.stream);
}

}  // namespace rb

using namespace rb;

extern "C" {

int kernel_cuda_host_register(void *ptr, size_t bytes)
{
    if (ensure() != 0)
        return -1;
    if (!ptr || bytes == 0)
        return fail("kernel_cuda_host_register: empty range");
    if (check(cudaHostRegister(ptr, bytes, cudaHostRegisterPortable), "cudaHostRegister") != 0)
        return -1;
    const uintptr_t lo = reinterpret_cast<uintptr_t>(ptr);
    std::lock_guard<std::mutex> lk(g_reg_mu);
    HostRange r{lo, lo + bytes};
    g_reg.insert(std::upper_bound(g_reg.begin(), g_reg.end(), r,
                                  [](const HostRange &x, const HostRange &y) { return x.lo < y.lo; }),
                 r);
    return 0;
}

int kernel_cuda_host_unregister(void *ptr)
{
    if (ensure() != 0)
        return -1;
    const uintptr_t lo = reinterpret_cast<uintptr_t>(ptr);
    {
        std::lock_guard<std::mutex> lk(g_reg_mu);
        auto it = std::find_if(g_reg.begin(), g_reg.end(), [&](const HostRange &r) { return r.lo == lo; });
        if (it == g_reg.end())
            return fail("kernel_cuda_host_unregister: %p was not registered", ptr);
        g_reg.erase(it);
    }
    return check(cudaHostUnregister(ptr), "cudaHostUnregister");
}

int kernel_cuda_init(int device)
{
    if (g_rt.device == device)
        return check(cudaSetDevice(device), "cudaSetDevice");
    if (g_rt.device >= 0)
        kernel_cuda_shutdown();
    return init_device(device);
}

void kernel_cuda_trim_scratch(void)
{
    if (g_rt.device < 0)
        return;
    cudaSetDevice(g_rt.device);
    cudaStreamSynchronize(g_rt.stream);
    if (g_rt.scratch)
        cudaFree(g_rt.scratch);
    if (g_rt.pinned)
        cudaFreeHost(g_rt.pinned);
    if (g_rt.dstage)
        cudaFree(g_rt.dstage);
    g_rt.dstage = nullptr;
    g_rt.dstage_bytes = 0;
    g_rt.scratch = nullptr;
    g_rt.scratch_bytes = 0;
    g_rt.pinned = nullptr;
    g_rt.gen++;                      // recorded work may not point into the freed buffers
    g_rt.pinned_bytes = 0;
}

void kernel_cuda_shutdown(void)
{
    if (g_rt.device < 0)
        return;
    kernel_cuda_trim_scratch();
    if (g_rt.err_word)
        cudaFree(g_rt.err_word);
    if (g_rt.err_host)
        cudaFreeHost(g_rt.err_host);
    if (g_rt.copy_stream)
        cudaStreamDestroy(g_rt.copy_stream);
    if (g_rt.out_stream)
        cudaStreamDestroy(g_rt.out_stream);
    if (g_rt.counters)
        cudaFree(g_rt.counters);
    // the generation stays monotonic across a shutdown: recordings made before it never match
    const uint64_t gen = g_rt.gen + 1;
    g_rt = Runtime();
    g_rt.gen = gen;
}

int kernel_cuda_set_stream(void *stream)
{
    if (ensure() != 0)
        return -1;
    g_rt.stream = static_cast<cudaStream_t>(stream);
    return 0;
}

int kernel_cuda_synchronize(void)
{
    if (ensure() != 0)
        return -1;
    // the error word travels behind the stream's work, so one wait covers both
    if (check(cudaMemcpyAsync(g_rt.err_host, g_rt.err_word, sizeof(unsigned), cudaMemcpyDeviceToHost,
                              g_rt.stream), "read error word") != 0 ||
        check(cudaStreamSynchronize(g_rt.stream), "cudaStreamSynchronize") != 0)
        return -1;
    const unsigned word = *reinterpret_cast<volatile unsigned *>(g_rt.err_host);
    if (word) {
        cudaMemset(g_rt.err_word, 0, sizeof(unsigned));
        return fail("kernel-recorded failure 0x%x (%s%s)", word,
                    (word & kErrWaitTimeout) ? "bounded wait timed out " : "",
                    (word & kErrBadArgument) ? "bad argument" : "");
    }
    return 0;
}

const char *kernel_cuda_last_error(void) { return g_err; }

uint64_t kernel_cuda_launch_count(void) { return g_launches.load(); }

void *kernel_cuda_alloc(size_t bytes)
{
    if (ensure() != 0 || bytes == 0)
        return nullptr;
    void *p = nullptr;
    if (check(cudaMalloc(&p, bytes), "kernel_cuda_alloc") != 0)
        return nullptr;
    if (check(cudaMemset(p, 0, bytes), "kernel_cuda_alloc memset") != 0) {
        cudaFree(p);
        return nullptr;
    }
    return p;
}

int kernel_cuda_free(void *ptr)
{
    if (!ptr)
        return 0;
    if (ensure() != 0)
        return -1;
    return check(cudaFree(ptr), "kernel_cuda_free");
}

int kernel_cuda_upload(void *dst, const void *src, size_t bytes)
{
    if (ensure() != 0)
        return -1;
    if (check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, g_rt.stream), "upload") != 0)
        return -1;
    return check(cudaStreamSynchronize(g_rt.stream), "upload sync");
}

int kernel_cuda_download(void *dst, const void *src, size_t bytes)
{
    if (ensure() != 0)
        return -1;
    if (check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, g_rt.stream), "download") != 0)
        return -1;
    return check(cudaStreamSynchronize(g_rt.stream), "download sync");
}

int kernel_cuda_memset(void *dst, int value, size_t bytes)
{
    if (ensure() != 0)
        return -1;
    return check(cudaMemsetAsync(dst, value, bytes, g_rt.stream), "kernel_cuda_memset");
}

int kernel_cuda_memmove(void *dst, const void *src, size_t bytes)
{
    if (ensure() != 0)
        return -1;
    if (bytes == 0 || dst == src)
        return 0;
    const char *s = static_cast<const char *>(src);
    char *d = static_cast<char *>(dst);
    // Device-to-device cudaMemcpy does not promise overlap safety: move in chunks that never
    // overlap their own destination, walking in the safe direction.
    size_t gap = d > s ? (size_t)(d - s) : (size_t)(s - d);
    if (gap >= bytes)
        return check(cudaMemcpyAsync(d, s, bytes, cudaMemcpyDeviceToDevice, g_rt.stream), "memmove");
    if (d < s) {
        for (size_t off = 0; off < bytes; off += gap) {
            size_t n = bytes - off < gap ? bytes - off : gap;
            if (check(cudaMemcpyAsync(d + off, s + off, n, cudaMemcpyDeviceToDevice, g_rt.stream),
                      "memmove") != 0)
                return -1;
        }
    } else {
        for (size_t end = bytes; end > 0;) {
            size_t n = end < gap ? end : gap;
            end -= n;
            if (check(cudaMemcpyAsync(d + end, s + end, n, cudaMemcpyDeviceToDevice, g_rt.stream),
                      "memmove") != 0)
                return -1;
        }
    }
    return 0;
}

int kernel_cuda_ipc_handle(void *dev_ptr, void *handle)
{
    if (ensure() != 0)
        return -1;
    if (!dev_ptr || !handle)
        return fail("kernel_cuda_ipc_handle: null argument");
    static_assert(sizeof(cudaIpcMemHandle_t) == KERNEL_CUDA_IPC_HANDLE_BYTES, "IPC handle size");
    cudaIpcMemHandle_t h;
    if (check(cudaIpcGetMemHandle(&h, dev_ptr), "cudaIpcGetMemHandle") != 0)
        return -1;
    memcpy(handle, &h, sizeof(h));
    return 0;
}

int kernel_cuda_ipc_open(const void *handle, void **dev_ptr)
{
    if (ensure() != 0)
        return -1;
    if (!handle || !dev_ptr)
        return fail("kernel_cuda_ipc_open: null argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *dev_ptr = nullptr;
    return check(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

int kernel_cuda_ipc_close(void *dev_ptr)
{
    if (ensure() != 0)
        return -1;
    if (!dev_ptr)
        return 0;
    return check(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle");
}

}  // extern "C"

// ---------------------------------------------------------------- f16 window rows <-> host fp32

namespace {

__global__ void f16_to_f32_copy_kernel(const __half *s, float *d, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        d[i] = __half2float(s[i]);
}

__global__ void f32_to_f16_copy_kernel(const float *s, __half *d, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        d[i] = __float2half_rn(s[i]);
}

constexpr size_t kConvPiece = (size_t)1 << 22;     // values per staged piece (16 MB of fp32)

}  // namespace

extern "C" int kernel_cuda_download_f16_f32(float *dst_host, const uint16_t *src_dev, size_t n)
{
    if (ensure() != 0)
        return -1;
    if (n && (!dst_host || !src_dev))
        return fail("kernel_cuda_download_f16_f32: null pointer");
    for (size_t off = 0; off < n; off += kConvPiece) {
        const size_t m = n - off < kConvPiece ? n - off : kConvPiece;
        float *d = static_cast<float *>(dstage(m * sizeof(float)));
        float *h = static_cast<float *>(pinned(m * sizeof(float)));
        if (!d || !h)
            return -1;
        f16_to_f32_copy_kernel<<<(unsigned)std::min<size_t>((m + 255) / 256, 4096), 256, 0, g_rt.stream>>>(
            reinterpret_cast<const __half *>(src_dev) + off, d, m);
        if (launched("f16_to_f32_copy_kernel") != 0 ||
            check(cudaMemcpyAsync(h, d, m * sizeof(float), cudaMemcpyDeviceToHost, g_rt.stream), "download") != 0 ||
            check(cudaStreamSynchronize(g_rt.stream), "download sync") != 0)
            return -1;
        memcpy(dst_host + off, h, m * sizeof(float));
    }
    return 0;
}

extern "C" int kernel_cuda_upload_f32_f16(uint16_t *dst_dev, const float *src_host, size_t n)
{
    if (ensure() != 0)
        return -1;
    if (n && (!dst_dev || !src_host))
        return fail("kernel_cuda_upload_f32_f16: null pointer");
    for (size_t off = 0; off < n; off += kConvPiece) {
        const size_t m = n - off < kConvPiece ? n - off : kConvPiece;
        float *d = static_cast<float *>(dstage(m * sizeof(float)));
        float *h = static_cast<float *>(pinned(m * sizeof(float)));
        if (!d || !h)
            return -1;
        memcpy(h, src_host + off, m * sizeof(float));
        if (check(cudaMemcpyAsync(d, h, m * sizeof(float), cudaMemcpyHostToDevice, g_rt.stream), "upload") != 0)
            return -1;
        f32_to_f16_copy_kernel<<<(unsigned)std::min<size_t>((m + 255) / 256, 4096), 256, 0, g_rt.stream>>>(
            d, reinterpret_cast<__half *>(dst_dev) + off, m);
        // the pinned piece is refilled next: wait for its copy (and the conversion) first
        if (launched("f32_to_f16_copy_kernel") != 0 || check(cudaStreamSynchronize(g_rt.stream), "upload sync") != 0)
            return -1;
    }
    return 0;
}

// ---------------------------------------------------------------- bounded-wait probe

namespace {

// Waits on an mbarrier that nothing ever arrives at, for at most `budget` cycles: the wait must
// give up, record kErrWaitTimeout and return -- the path every pipelined kernel takes instead of
// hanging when a partner never signals.
__global__ void wait_probe_kernel(unsigned *err, long long budget)
{
    __shared__ unsigned long long bar;
    if (threadIdx.x == 0) {
        rb::mbar_init(rb::smem_addr(&bar), 1);
        rb::mbar_init_fence();
        if (!rb::mbar_wait(rb::smem_addr(&bar), 0, budget))
            atomicOr(err, rb::kErrWaitTimeout);
    }
}

}  // namespace

extern "C" int kernel_cuda_wait_probe(long long budget_cycles)
{
    if (ensure() != 0)
        return -1;
    if (budget_cycles <= 0 || budget_cycles > 4000000000ll)
        return fail("kernel_cuda_wait_probe: budget out of range");
    wait_probe_kernel<<<1, 32, 0, g_rt.stream>>>(g_rt.err_word, budget_cycles);
    if (launched("wait_probe_kernel") != 0)
        return -1;
    if (check(cudaStreamSynchronize(g_rt.stream), "wait probe") != 0)
        return -1;
    unsigned word = 0;
    if (check(cudaMemcpy(&word, g_rt.err_word, sizeof(word), cudaMemcpyDeviceToHost), "read error word") != 0)
        return -1;
    if (check(cudaMemset(g_rt.err_word, 0, sizeof(unsigned)), "clear error word") != 0)
        return -1;
    return (int)word;
}

