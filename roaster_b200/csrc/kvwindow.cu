// Device-resident attention window of one slot: the policy of the reference's kvwindow.c over
// f16 K/V held in device memory, with the evicted tokens kept in a spill store of kvspill.c's
// format (reference src/kvwindow.c, src/kvspill.c).
//
// Window model (kvwindow.c:1-268): every attention layer holds the same `len` rows; the
// layout invariant stated above the policy functions says where each token lives (a fixed
// prefix, the spill store, the recent rows). The policy functions derive each operation from
// that invariant and select the same tokens as the reference (head from keep / pin, slides in
// blocks of a quarter of the window beyond the prefix, restore and rollback through the store's
// stack order); the data movement becomes device work:
//   - row moves inside a layer: device-to-device copies in chunks that never overlap their own
//     source (or through scratch when the shift is short);
//   - eviction: f16 rows -> fp32 on the device -> pinned staging -> the store;
//   - restore: store -> pinned staging -> device -> f16 rows (exact: the rows were f16).
// Spill store (kvspill.c:77-148): a stack of chunks, one per eviction; a chunk of n tokens holds,
// per layer a, a K block then a V block of n x 512 fp32; `head` is recorded when an eviction
// finds the store empty and cleared when it empties. The chunks live in a file when a path is
// given (the reference's SSD spill, same layout) or in host memory otherwise.
#include "runtime.h"
#include "../../include/roaster_cuda.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <unistd.h>
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

namespace rb {
namespace {

constexpr size_t kRow = 512;                          // f16 or fp32 values per token row
constexpr size_t kPiece = 1024;                       // tokens per staged transfer piece
constexpr size_t kMoveBlock = 8192;                   // rows per scratch-staged move block
constexpr int kMaxLayers = 64;

struct CvtParams {
    const void *src[2 * kMaxLayers];
    void *dst[2 * kMaxLayers];
};

// fp32 <-> f16 for 2 * layers row ranges of `count` values each (grid.y = range).
__global__ void f16_to_f32_kernel(const __grid_constant__ CvtParams p, size_t count)
{
    const __half *s = static_cast<const __half *>(p.src[blockIdx.y]);
    float *d = static_cast<float *>(p.dst[blockIdx.y]);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x)
        d[i] = __half2float(s[i]);
}

__global__ void f32_to_f16_kernel(const __grid_constant__ CvtParams p, size_t count)
{
    const float *s = static_cast<const float *>(p.src[blockIdx.y]);
    __half *d = static_cast<__half *>(p.dst[blockIdx.y]);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x)
        d[i] = __float2half_rn(s[i]);
}

struct Chunk {
    uint64_t off;
    size_t n_alloc, n_valid;
};

}  // namespace
}  // namespace rb

struct KernelKvWindow {
    int layers = 0;
    size_t ctx = 0, capacity = 0, len = 0, position = 0;
    bool slide = false;
    size_t keep = 0, pin = 0;
    std::vector<uint16_t *> k, v;                     // device [capacity][2][256] f16
    // spill store
    std::string path;
    int fd = -1;
    std::vector<char> mem;                            // in-memory store when no path
    std::vector<rb::Chunk> chunks;
    uint64_t end = 0;
    size_t count = 0, head = 0;
    // staging (the library's shared pinned / device buffers, set per operation)
    float *dstage = nullptr;                          // device fp32, 2 * layers * kPiece rows
    float *hstage = nullptr;                          // pinned fp32, same size
};

namespace rb {
namespace {

using W = KernelKvWindow;

size_t staged_floats(const W *w) { return (size_t)2 * w->layers * kPiece * kRow; }

int store_write(W *w, const void *buf, size_t bytes, uint64_t off)
{
    if (w->fd >= 0) {
        const char *p = static_cast<const char *>(buf);
        while (bytes) {
            const ssize_t r = pwrite(w->fd, p, bytes, (off_t)off);
            if (r <= 0)
                return fail("kv window: spill write failed");
            p += r;
            off += (uint64_t)r;
            bytes -= (size_t)r;
        }
        return 0;
    }
    if (w->mem.size() < off + bytes)
        w->mem.resize(off + bytes);
    memcpy(w->mem.data() + off, buf, bytes);
    return 0;
}

int store_read(W *w, void *buf, size_t bytes, uint64_t off)
{
    if (w->fd >= 0) {
        char *p = static_cast<char *>(buf);
        while (bytes) {
            const ssize_t r = pread(w->fd, p, bytes, (off_t)off);
            if (r <= 0)
                return fail("kv window: spill read failed");
            p += r;
            off += (uint64_t)r;
            bytes -= (size_t)r;
        }
        return 0;
    }
    if (off + bytes > w->mem.size())
        return fail("kv window: spill read past the store");
    memcpy(buf, w->mem.data() + off, bytes);
    return 0;
}

void store_truncate(W *w, uint64_t off)
{
    w->end = off;
    if (w->fd >= 0) {
        if (ftruncate(w->fd, (off_t)off) != 0) { /* best effort, as the file is overwritten anyway */ }
    } else {
        w->mem.resize(off);
    }
}

int ensure_staging(W *w)
{
    const size_t bytes = staged_floats(w) * sizeof(float);
    w->dstage = static_cast<float *>(dstage(bytes));
    w->hstage = static_cast<float *>(pinned(bytes));
    return (w->dstage && w->hstage) ? 0 : -1;
}

int launch_cvt(bool to_f32, const CvtParams &p, int ranges, size_t count)
{
    const unsigned gx = (unsigned)std::min<size_t>((count + 255) / 256, 1024);
    if (to_f32)
        f16_to_f32_kernel<<<dim3(gx, ranges), 256, 0, rt().stream>>>(p, count);
    else
        f32_to_f16_kernel<<<dim3(gx, ranges), 256, 0, rt().stream>>>(p, count);
    return launched(to_f32 ? "f16_to_f32_kernel" : "f32_to_f16_kernel");
}

// Move rows [src, src + n) to [dst, dst + n) in every layer's K and V (overlap-safe). A shift of
// at least kMoveBlock rows moves in blocks of `shift` rows directly (a block never overlaps its
// own source); a shorter shift moves kMoveBlock rows at a time through scratch. Either way the
// blocks go in the order that never overwrites a source not yet moved.
int move_rows(W *w, size_t dst, size_t src, size_t n)
{
    if (n == 0 || dst == src)
        return 0;
    cudaStream_t st = rt().stream;
    const size_t gap = dst > src ? dst - src : src - dst;
    const size_t rowb = kRow * sizeof(uint16_t);
    const bool direct = gap >= kMoveBlock || gap >= n;
    const size_t blk = direct ? gap : kMoveBlock;
    char *scr = nullptr;
    if (!direct) {
        scr = static_cast<char *>(scratch(kMoveBlock * rowb));
        if (!scr)
            return -1;
    }
    for (int t = 0; t < 2 * w->layers; t++) {
        char *b = reinterpret_cast<char *>((t & 1) ? w->v[t >> 1] : w->k[t >> 1]);
        const size_t nb = (n + blk - 1) / blk;
        for (size_t i = 0; i < nb; i++) {
            const size_t bi = dst < src ? i : nb - 1 - i;        // front to back when moving down
            const size_t o = bi * blk, m = std::min(blk, n - o);
            char *d = b + (dst + o) * rowb;
            const char *sp = b + (src + o) * rowb;
            if (direct) {
                if (check(cudaMemcpyAsync(d, sp, m * rowb, cudaMemcpyDeviceToDevice, st), "kv move") != 0)
                    return -1;
            } else if (check(cudaMemcpyAsync(scr, sp, m * rowb, cudaMemcpyDeviceToDevice, st), "kv move") != 0 ||
                       check(cudaMemcpyAsync(d, scr, m * rowb, cudaMemcpyDeviceToDevice, st), "kv move") != 0) {
                return -1;
            }
        }
    }
    return 0;
}

// Push rows [h, h + n) of every layer as one chunk (kvspill_append).
int spill_push(W *w, size_t h, size_t n)
{
    if (n == 0)
        return 0;
    if (ensure_staging(w) != 0)
        return -1;
    if (w->fd < 0 && !w->path.empty()) {
        w->fd = open(w->path.c_str(), O_RDWR | O_CREAT | O_TRUNC | O_CLOEXEC, 0600);
        if (w->fd < 0)
            return fail("kv window: cannot open spill file %s", w->path.c_str());
        w->end = 0;
    }
    const uint64_t off = w->end;
    const size_t blk = n * kRow * sizeof(float);
    for (size_t p0 = 0; p0 < n; p0 += kPiece) {
        const size_t m = std::min(kPiece, n - p0);
        CvtParams cp;
        for (int t = 0; t < 2 * w->layers; t++) {
            const uint16_t *base = (t & 1) ? w->v[t >> 1] : w->k[t >> 1];
            cp.src[t] = base + (h + p0) * kRow;
            cp.dst[t] = w->dstage + (size_t)t * kPiece * kRow;
        }
        if (launch_cvt(true, cp, 2 * w->layers, m * kRow) != 0)
            return -1;
        for (int t = 0; t < 2 * w->layers; t++)
            if (check(cudaMemcpyAsync(w->hstage + (size_t)t * kPiece * kRow, w->dstage + (size_t)t * kPiece * kRow,
                                      m * kRow * sizeof(float), cudaMemcpyDeviceToHost, rt().stream), "spill out") != 0)
                return -1;
        if (check(cudaStreamSynchronize(rt().stream), "spill out") != 0)
            return -1;
        for (int t = 0; t < 2 * w->layers; t++)
            if (store_write(w, w->hstage + (size_t)t * kPiece * kRow, m * kRow * sizeof(float),
                            off + (uint64_t)t * blk + p0 * kRow * sizeof(float)) != 0) {
                store_truncate(w, off);
                return -1;
            }
    }
    w->chunks.push_back(Chunk{off, n, n});
    w->end = off + (uint64_t)2 * w->layers * blk;
    if (w->count == 0)
        w->head = h;
    w->count += n;
    return 0;
}

// Take the n most recent tokens (kvspill_pop); with dst != SIZE_MAX they land in rows
// [dst, dst + n), oldest first; otherwise they are dropped.
int spill_pop(W *w, size_t n, size_t dst)
{
    if (n == 0)
        return 0;
    if (n > w->count)
        return fail("kv window: popping %zu of %zu spilled tokens", n, w->count);
    if (dst != (size_t)-1) {
        if (ensure_staging(w) != 0)
            return -1;
        // token j (0 = oldest of the n) of the popped range, located chunk by chunk from the top
        std::vector<std::pair<size_t, size_t>> where(n);             // (chunk index, index in chunk)
        {
            size_t left = n;
            size_t ci = w->chunks.size();
            while (left) {
                const Chunk &c = w->chunks[--ci];
                const size_t r = std::min(left, c.n_valid);
                for (size_t i = 0; i < r; i++)
                    where[left - r + i] = {ci, c.n_valid - r + i};
                left -= r;
            }
        }
        for (size_t p0 = 0; p0 < n; p0 += kPiece) {
            const size_t m = std::min(kPiece, n - p0);
            for (int t = 0; t < 2 * w->layers; t++)
                for (size_t j = 0; j < m;) {
                    // runs of consecutive tokens of one chunk in one read
                    const auto [ci, ii] = where[p0 + j];
                    size_t run = 1;
                    while (j + run < m && where[p0 + j + run].first == ci && where[p0 + j + run].second == ii + run)
                        run++;
                    const Chunk &c = w->chunks[ci];
                    const uint64_t o = c.off + ((uint64_t)t * c.n_alloc + ii) * kRow * sizeof(float);
                    if (store_read(w, w->hstage + ((size_t)t * kPiece + j) * kRow, run * kRow * sizeof(float), o) != 0)
                        return -1;
                    j += run;
                }
            CvtParams cp;
            for (int t = 0; t < 2 * w->layers; t++) {
                if (check(cudaMemcpyAsync(w->dstage + (size_t)t * kPiece * kRow, w->hstage + (size_t)t * kPiece * kRow,
                                          m * kRow * sizeof(float), cudaMemcpyHostToDevice, rt().stream), "spill in") != 0)
                    return -1;
                uint16_t *base = (t & 1) ? w->v[t >> 1] : w->k[t >> 1];
                cp.src[t] = w->dstage + (size_t)t * kPiece * kRow;
                cp.dst[t] = base + (dst + p0) * kRow;
            }
            if (launch_cvt(false, cp, 2 * w->layers, m * kRow) != 0)
                return -1;
            // the pinned staging is refilled by the next piece: wait for its uploads
            if (check(cudaStreamSynchronize(rt().stream), "spill in") != 0)
                return -1;
        }
    }
    size_t left = n;
    while (left) {
        Chunk &c = w->chunks.back();
        const size_t r = std::min(left, c.n_valid);
        c.n_valid -= r;
        w->count -= r;
        left -= r;
        if (c.n_valid == 0) {
            const uint64_t off = c.off;
            w->chunks.pop_back();
            store_truncate(w, off);
        }
    }
    if (w->count == 0)
        w->head = 0;
    return 0;
}

// ---------------------------------------------------------------- window policy
//
// Layout invariant. With P = position (tokens seen), S = count (tokens in the store) and
// H = head (the prefix length fixed when the store went from empty to non-empty), token t is
//   in row t          for t < H           (the prefix, which does not move while S > 0),
//   in the store      for H <= t < H + S  (a stack: the latest eviction on top),
//   in row t - S      for t >= H + S      (the recent part),
// so len = P - S rows are occupied. Each operation below keeps the invariant and selects the
// same tokens to keep, spill and bring back as the reference's policy (kvwindow.c), since the
// attention must see the same keys.

// Rows at the start of a window of `rows` rows that stay in place when it slides. While tokens
// are spilled it is the recorded head. Otherwise it is the larger of two requests, capped by the
// occupied rows: the configured keep, at most half the window; the pinned prompt, which must
// leave an eighth of the window (at least one row) free to slide through.
size_t prefix_rows(const W *w, size_t rows)
{
    if (w->count > 0)
        return w->head;
    const size_t keep_part = std::min(w->keep, rows / 2);
    const size_t must_free = std::max<size_t>(rows / 8, 1);
    size_t pin_part = w->pin;
    if (rows >= must_free && pin_part > rows - must_free)
        pin_part = rows > must_free ? rows - must_free : 0;
    return std::min(std::max(keep_part, pin_part), w->len);
}

// Pushes the `n` rows that follow the first `at` rows onto the store and shifts the rows after
// them down over the gap.
int spill_rows(W *w, size_t at, size_t n)
{
    if (n == 0)
        return 0;
    if (at > w->len || n > w->len - at)
        return fail("kv window: evicting %zu tokens after %zu of %zu", n, at, w->len);
    if (spill_push(w, at, n) != 0)
        return -1;
    if (move_rows(w, at, at + n, w->len - at - n) != 0)
        return -1;
    w->len -= n;
    return 0;
}

// Pops the `n` most recently spilled tokens and puts them back right after the prefix, shifting
// the recent rows up first to open the gap (and back again if the store cannot deliver).
int restore(W *w, size_t n)
{
    if (n == 0)
        return 0;
    if (n > w->count)
        return fail("kv window: restoring %zu of %zu spilled tokens", n, w->count);
    const size_t at = w->head;
    if (at > w->len || w->len + n > w->capacity)
        return fail("kv window: no room to restore %zu tokens", n);
    const size_t recent = w->len - at;
    if (move_rows(w, at + n, at, recent) != 0)
        return -1;
    if (spill_pop(w, n, at) != 0) {
        move_rows(w, at, at + n, recent);
        return -1;
    }
    w->len += n;
    return 0;
}

// Room for `need` more rows in the window (w->ctx rows). If they do not fit and sliding is on,
// the oldest rows after the prefix go to the store: the overflow, rounded up to a quarter of the
// rows beyond the prefix so the window slides in blocks and not one token at a time.
int ensure_room(W *w, size_t need)
{
    const size_t rows = w->ctx;
    if (w->len + need <= rows)
        return 0;
    if (!w->slide)
        return fail("kv window: full (%zu + %zu > %zu) and sliding is off", w->len, need, rows);
    const size_t pre = prefix_rows(w, rows);
    if (need > rows - pre)
        return fail("kv window: %zu tokens do not fit beside the kept head", need);
    const size_t overflow = w->len + need - rows;
    const size_t n = std::min(std::max(overflow, (rows - pre) / 4), w->len - pre);
    if (n < overflow)
        return fail("kv window: cannot free %zu tokens", overflow);
    return spill_rows(w, pre, n);
}

// Back to a snapshot taken at position p0 with s0 tokens spilled. At the snapshot the window held
// every token below p0 except the run then spilled, [H, H + s0) (the run only grows upwards from
// H while the store is non-empty). Relative to the invariant's layout that means:
//   - store entries for tokens at or above max(p0, H) did not exist then: drop them;
//   - store entries for tokens in [H + s0, min(p0, H + S)) were rows then: bring them back;
//   - recent rows for tokens in [H + S, p0) stay, rows for tokens from p0 on go;
//   - if p0 < H the snapshot had no store at all: only the first p0 rows stay.
int rollback(W *w, size_t p0, size_t s0)
{
    if (p0 > w->position || w->count < s0)
        return fail("kv window: cannot roll back to position %zu", p0);
    if (w->count == 0) {
        if (p0 > w->capacity)
            return fail("kv window: rollback target beyond the window");
        w->len = p0;
        w->position = p0;
        return 0;
    }
    const size_t H = w->head, S = w->count;
    const size_t run_end = H + S;                                // first token after the spilled run
    const size_t drop = run_end - std::min(run_end, std::max(p0, H));
    const size_t back_end = std::min(p0, run_end);
    const size_t back = back_end > H + s0 ? back_end - (H + s0) : 0;
    const size_t recent_keep = p0 > run_end ? p0 - run_end : 0;
    const size_t prefix_keep = std::min(p0, H);
    if (drop + back > S || prefix_keep + back + recent_keep > w->capacity)
        return fail("kv window: rollback does not fit");
    if (drop && spill_pop(w, drop, (size_t)-1) != 0)
        return -1;
    if (p0 < H) {
        w->len = p0;
        w->position = p0;
        return 0;
    }
    if (back) {
        if (recent_keep && move_rows(w, H + back, H, recent_keep) != 0)
            return -1;
        if (spill_pop(w, back, H) != 0)
            return -1;
    }
    w->len = H + back + recent_keep;
    w->position = p0;
    return 0;
}

// Fits the occupied rows into a smaller window of `rows` rows (a context change): the overflow
// goes to the store plus a quarter of the new window beyond the prefix, so the first appends
// after the change find room.
int shrink_to_fit(W *w, size_t rows)
{
    if (w->len <= rows)
        return 0;
    const size_t pre = prefix_rows(w, rows);
    if (pre >= rows)
        return fail("kv window: head does not fit a window of %zu", rows);
    const size_t overflow = w->len - rows;
    const size_t n = std::min(overflow + (rows - pre) / 4, w->len - pre);
    if (n < overflow)
        return fail("kv window: cannot shrink to %zu", rows);
    return spill_rows(w, pre, n);
}

int realloc_rows(W *w, size_t new_ctx)
{
    if (new_ctx == 0 || w->len > new_ctx)
        return fail("kv window: cannot reallocate to %zu rows", new_ctx);
    std::vector<uint16_t *> nk(w->layers, nullptr), nv(w->layers, nullptr);
    const size_t bytes = new_ctx * kRow * sizeof(uint16_t);
    for (int a = 0; a < w->layers; a++) {
        if (cudaMalloc(&nk[a], bytes) != cudaSuccess || cudaMalloc(&nv[a], bytes) != cudaSuccess ||
            cudaMemsetAsync(nk[a], 0, bytes, rt().stream) != cudaSuccess ||
            cudaMemsetAsync(nv[a], 0, bytes, rt().stream) != cudaSuccess) {
            for (int b = 0; b <= a; b++) {
                cudaFree(nk[b]);
                cudaFree(nv[b]);
            }
            return fail("kv window: out of device memory for %zu rows", new_ctx);
        }
    }
    for (int a = 0; a < w->layers; a++) {
        const size_t cp = w->len * kRow * sizeof(uint16_t);
        if (cp && (check(cudaMemcpyAsync(nk[a], w->k[a], cp, cudaMemcpyDeviceToDevice, rt().stream), "kv realloc") != 0 ||
                   check(cudaMemcpyAsync(nv[a], w->v[a], cp, cudaMemcpyDeviceToDevice, rt().stream), "kv realloc") != 0))
            return -1;
    }
    if (check(cudaStreamSynchronize(rt().stream), "kv realloc") != 0)
        return -1;
    for (int a = 0; a < w->layers; a++) {
        cudaFree(w->k[a]);
        cudaFree(w->v[a]);
        w->k[a] = nk[a];
        w->v[a] = nv[a];
    }
    w->capacity = new_ctx;
    return 0;
}

// After the window grew: spilled tokens come back, all of them when they fit, else as many as
// leave a quarter of the window beyond the prefix free (the next appends would evict them again).
int refill(W *w)
{
    const size_t rows = w->ctx;
    if (w->count == 0 || w->len >= rows)
        return 0;
    const size_t free_rows = rows - w->len;
    size_t n = w->count;
    if (n > free_rows) {
        const size_t headroom = rows > w->head ? (rows - w->head) / 4 : 0;
        n = free_rows > headroom ? free_rows - headroom : 0;
    }
    return n ? restore(w, n) : 0;
}

void destroy(W *w)
{
    if (!w)
        return;
    for (auto p : w->k)
        cudaFree(p);
    for (auto p : w->v)
        cudaFree(p);
    if (w->fd >= 0) {
        close(w->fd);
        unlink(w->path.c_str());
    }
    delete w;
}

}  // namespace
}  // namespace rb

using namespace rb;

extern "C" KernelKvWindow *kernel_kvw_create(int layers, size_t ctx, int slide, size_t keep, size_t pin,
                                            const char *spill_path)
{
    if (ensure() != 0)
        return nullptr;
    if (layers <= 0 || layers > kMaxLayers || ctx == 0) {
        fail("kernel_kvw_create: bad arguments (layers %d, ctx %zu)", layers, ctx);
        return nullptr;
    }
    W *w = new W();
    w->layers = layers;
    w->slide = slide != 0;
    w->keep = keep;
    w->pin = pin;
    w->path = spill_path ? spill_path : "";
    w->k.assign(layers, nullptr);
    w->v.assign(layers, nullptr);
    if (realloc_rows(w, ctx) != 0) {
        destroy(w);
        return nullptr;
    }
    w->ctx = ctx;
    return w;
}

extern "C" void kernel_kvw_destroy(KernelKvWindow *w)
{
    if (ensure() != 0)
        return;
    cudaStreamSynchronize(rt().stream);
    destroy(w);
}

extern "C" uint16_t *kernel_kvw_k(KernelKvWindow *w, int layer)
{
    return (w && layer >= 0 && layer < w->layers) ? w->k[layer] : nullptr;
}

extern "C" uint16_t *kernel_kvw_v(KernelKvWindow *w, int layer)
{
    return (w && layer >= 0 && layer < w->layers) ? w->v[layer] : nullptr;
}

extern "C" size_t kernel_kvw_len(const KernelKvWindow *w) { return w ? w->len : 0; }
extern "C" size_t kernel_kvw_spilled(const KernelKvWindow *w) { return w ? w->count : 0; }
extern "C" size_t kernel_kvw_head(const KernelKvWindow *w) { return w ? prefix_rows(w, w->ctx) : 0; }
extern "C" size_t kernel_kvw_position(const KernelKvWindow *w) { return w ? w->position : 0; }
extern "C" size_t kernel_kvw_context(const KernelKvWindow *w) { return w ? w->ctx : 0; }

extern "C" size_t kernel_kvw_max_chunk(const KernelKvWindow *w)
{
    if (!w)
        return 0;
    if (w->slide)
        return w->ctx - prefix_rows(w, w->ctx);
    return w->ctx > w->len ? w->ctx - w->len : 0;
}

extern "C" int kernel_kvw_set_policy(KernelKvWindow *w, int slide, size_t keep, size_t pin)
{
    if (!w)
        return fail("kernel_kvw_set_policy: null window");
    w->slide = slide != 0;
    w->keep = keep;
    w->pin = pin;
    return 0;
}

extern "C" int kernel_kvw_ensure_room(KernelKvWindow *w, size_t need)
{
    if (ensure() != 0 || !w)
        return -1;
    return ensure_room(w, need);
}

extern "C" int kernel_kvw_appended(KernelKvWindow *w, size_t n)
{
    if (!w)
        return fail("kernel_kvw_appended: null window");
    if (w->len + n > w->capacity)
        return fail("kernel_kvw_appended: %zu + %zu rows exceed the window", w->len, n);
    w->len += n;
    w->position += n;
    return 0;
}

extern "C" int kernel_kvw_evict(KernelKvWindow *w, size_t n)
{
    if (ensure() != 0 || !w)
        return -1;
    return spill_rows(w, prefix_rows(w, w->ctx), n);
}

extern "C" int kernel_kvw_restore(KernelKvWindow *w, size_t n)
{
    if (ensure() != 0 || !w)
        return -1;
    return restore(w, n);
}

extern "C" int kernel_kvw_rollback(KernelKvWindow *w, size_t p0, size_t s0)
{
    if (ensure() != 0 || !w)
        return -1;
    return rollback(w, p0, s0);
}

extern "C" int kernel_kvw_set_context(KernelKvWindow *w, size_t ctx)
{
    if (ensure() != 0 || !w)
        return -1;
    if (ctx == 0)
        return fail("kernel_kvw_set_context: zero context");
    const size_t old = w->ctx;
    if (ctx == old)
        return 0;
    if (ctx < old && shrink_to_fit(w, ctx) != 0)          // push what no longer fits to the store
        return -1;
    if (realloc_rows(w, ctx) != 0)
        return -1;
    w->ctx = ctx;
    if (ctx > old)
        refill(w);                                         // best effort, as in the reference
    return 0;
}
