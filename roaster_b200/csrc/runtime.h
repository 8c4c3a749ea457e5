// Internal runtime of libroaster_b200: device selection, the work stream, grow-only device
// scratch and pinned staging, the device error word, and failure reporting. Not part of the
// C-ABI (include/roaster_cuda.h is).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include <functional>
#include <utility>
#include <vector>

#include "../../include/roaster_cuda.h"

namespace rb {

// Device error word bits, set by kernels instead of faulting.
enum : unsigned {
    kErrWaitTimeout = 1u << 0,   // a bounded mbarrier wait ran out
    kErrBadArgument = 1u << 1,   // a kernel found an argument it cannot process
};

struct Runtime {
    int device = -1;
    int num_sms = 0;
    cudaStream_t stream = nullptr;
    unsigned *err_word = nullptr;      // device, one word
    void *scratch = nullptr;           // device, grow-only
    size_t scratch_bytes = 0;
    int *counters = nullptr;           // device, zero-initialised, grow-only
    size_t counters_n = 0;
    void *dstage = nullptr;            // device staging of host-buffer calls, grow-only
    size_t dstage_bytes = 0;
    void *pinned = nullptr;            // host pinned, grow-only
    size_t pinned_bytes = 0;
    float inv_freq[32];                // RoPE inverse frequencies, computed with host powf
    unsigned *err_host = nullptr;      // pinned copy of the error word (read by synchronize)
    cudaStream_t copy_stream = nullptr;   // input copies that overlap kernels on `stream`
    cudaStream_t out_stream = nullptr;    // output copies that overlap later kernels on `stream`
    // Bumped whenever a library-owned device buffer or table that queued work may point to is
    // replaced (scratch, counters, staging, a reset of the tensor-map table): work recorded
    // earlier (a CUDA graph) is valid only while it is unchanged.
    uint64_t gen = 0;
};

Runtime &rt();
// Ensure the library is initialised (device 0 by default, or the one kernel_cuda_init chose)
// and make that device current on this thread. 0 = ok.
int ensure();
// Record a failure message; always returns -1.
int fail(const char *fmt, ...);
// Check a CUDA status; on error record it with `what` and return -1.
int check(cudaError_t e, const char *what);
// Check for a launch error after a kernel launch and count the launch.
int launched(const char *what);
// Add `n` to the launch count (kernels launched as part of a CUDA graph).
void count_launches(uint64_t n);

// Per-token rows of one k-quant matmul job: x[t] (16-byte aligned) holds token t's activations,
// y[t] receives its results. Both null: the job's contiguous X and Y.
struct MmRows {
    const float *const *x;
    float *const *y;
};
// kernel_cuda_matmul_quant_batch with optional row tables (one MmRows per job). The jobs with
// tables must all run on the tensor-core path; when one cannot, nothing is launched and 1 is
// returned. 0 = launched, -1 = error.
int matmul_quant_rows(const KernelCudaMatmulJob *jobs, int n, const MmRows *rows);
// Device scratch of at least `bytes` (grow-only; growing synchronises the stream).
void *scratch(size_t bytes);
// The library's second stream, for input copies that overlap kernels on the work stream
// (created on first use; null on failure, with the error recorded).
cudaStream_t copy_stream();
// Non-blocking stream for device-to-host output copies (the other copy engine), created on
// first use.
cudaStream_t out_stream();
// Zero-initialised device int counters (grow-only, separate from scratch). Kernels that use
// them return every counter to zero before they exit.
int *counters(size_t n);
// Device staging for the host-buffer entry points (grow-only, separate from scratch).
void *dstage(size_t bytes);
// Pinned host staging of at least `bytes` (grow-only; growing synchronises the stream).
void *pinned(size_t bytes);
// Encode a tiled tensor map for a 3-D f16 tensor in global memory (dims innermost first,
// strides in bytes of dims 1 and 2), 128-byte swizzle, zero fill outside the tensor. The map is
// plain data (128 bytes) that kernels read from global memory. 0 = ok.
int encode_tmap_f16_3d(CUtensorMap *map, const void *base, const uint64_t dims[3], const uint64_t strides[2],
                       const uint32_t box[3]);
// Encode a tiled tensor map for a 2-D byte array (dim0 bytes per row, dim1 rows, rows stride1
// bytes apart, a multiple of 16), no swizzle, zero fill outside the array. 0 = ok.
int encode_tmap_u8_2d(CUtensorMap *map, const void *base, uint64_t dim0, uint64_t dim1, uint64_t stride1,
                      uint32_t box0, uint32_t box1);
// Whether the host range [p, p + bytes) lies inside one buffer registered with
// kernel_cuda_host_register (pinned, so the copy engine moves it at full rate).
bool host_registered(const void *p, size_t bytes);

// The host buffers of one batch call, moved by the copy engine in as few copies as their layout
// allows. Segments are sorted by address and merged into runs. Input runs may bridge gaps of up
// to `gap` bytes, whose bytes are copied along; output runs merge only touching or overlapping
// segments, so a copy back never writes host bytes outside the outputs. Each run is one
// cudaMemcpyAsync to or from a device staging area laid out run after run; dev() gives the
// staging address of a host pointer inside a run.
// Host runs closer than this copy as one: a copy costs the engine a few microseconds whatever
// its size, about the link time of 150 KB.
constexpr size_t kRunGap = 128 << 10;
struct HostRuns {
    struct Run {
        uintptr_t lo, hi;
        size_t off;
    };
    std::vector<std::pair<uintptr_t, uintptr_t>> segs;
    std::vector<Run> runs;
    size_t bytes = 0;
    void add(const void *p, size_t n) { segs.emplace_back(reinterpret_cast<uintptr_t>(p), reinterpret_cast<uintptr_t>(p) + n); }
    void build(size_t gap);
    size_t offset(const void *p) const;
};
// Whether any run of `a` shares a byte with a run of `b` (both built).
bool runs_overlap(const HostRuns &a, const HostRuns &b);
// Copy every run host -> device (staging base `d`) or device -> host, on the library stream.
int runs_h2d(const HostRuns &r, char *d);
int runs_d2h(const HostRuns &r, const char *d);
// The same on stream `st` in direction `kind`.
int runs_copy(const HostRuns &r, char *d, cudaMemcpyKind kind, cudaStream_t st);
// 16-byte alignment check for pointers handed to bulk-copy engines.
inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch `kernel` as a programmatic dependent of the work before it on stream `st` (its launch
// overlaps the previous kernel's tail; the kernel calls griddep_wait() before reading any
// input), or as an ordinary launch where the attribute is not accepted. Counts the launch.
// ROASTER_PDL=0 in the environment makes every such launch an ordinary one.
bool pdl_enabled();
template <typename... Params, typename... Args>
int launch_dependent(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     const char *what, Args &&...args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...) != cudaSuccess) {
        (void)cudaGetLastError();
        cfg.numAttrs = 0;
        if (check(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...), what) != 0)
            return -1;
    }
    return launched(what);
}

// Host staging of the host-buffer entry points. A batch of n jobs of `per` floats each lives
// contiguously in pinned memory `h` and device memory `d`. stage_in fills the pinned copy job by
// job with fill(i, h + i * per) on several host threads, in chunks of jobs, and queues each
// chunk's host-to-device copy as soon as the chunk is filled, so the copies overlap the filling
// of the next chunk. stage_out queues the device-to-host copies by chunks and hands each chunk
// to drain(i, h + i * per) (several host threads) as soon as that chunk has arrived. Both use
// the library stream; 0 = ok.
int stage_in(float *h, float *d, int n, size_t per, const std::function<void(int, float *)> &fill);
int stage_out(float *h, const float *d, int n, size_t per, const std::function<void(int, const float *)> &drain);

}  // namespace rb
