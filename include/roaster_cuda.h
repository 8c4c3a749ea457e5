/*
 * roaster_cuda.h -- C-ABI of the B200 (sm_100a) hybrid-attention hot path.
 *
 * Plain C, in the style of the reference's src/kernels.h: size_t dims, caller-owned buffers,
 * no ownership transfer, `int` 0 = ok / -1 = failed (the caller maps -1 to
 * MODEL_FORWARD_ERROR, model.h:43-44). There is no CPU fallback: with no usable GPU every
 * compute entry point returns -1.
 *
 * The reference keeps the attention and DeltaNet math inline in src/model.c; each entry point
 * below names the model.c lines it replaces. The KV cache and the recurrent state become
 * device-resident ("buffer residency"): allocate them with kernel_cuda_alloc. The KV cache is
 * f16 [capacity][2 kv heads][256] for K and V separately (the reference's fp32 layout,
 * model.c:369-380, at half the bytes); the DeltaNet state keeps the reference layout
 * fp32 [32 value heads][128 key rows][128 value cols] (model.c:412-428).
 *
 * Threading: calls may come from any host thread but must not overlap (the reference
 * serialises model steps with its slot step lock, slots.c:864-891). All work goes to one CUDA
 * stream per process (kernel_cuda_set_stream). "Device" entry points are asynchronous on that
 * stream; "host" entry points stage their small per-step inputs/outputs through pinned memory
 * and return when the results are in the caller's buffers. The batched host entry points copy
 * into and out of that staging on up to 8 OpenMP threads (libgomp, as the reference's own host
 * code uses), in chunks that overlap the host-device copies.
 *
 * Device faults are never used for error reporting: kernels record failures (e.g. a bounded
 * wait that ran out) in a device error word, reported by kernel_cuda_synchronize().
 */
#ifndef ROASTER_CUDA_H
#define ROASTER_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Shapes fixed by the model (reference src/model.h:15-41). */
#define KERNEL_ATTN_Q_HEADS    16
#define KERNEL_ATTN_KV_HEADS   2
#define KERNEL_ATTN_HEAD_DIM   256
#define KERNEL_DN_K_HEADS      16
#define KERNEL_DN_V_HEADS      32
#define KERNEL_DN_HEAD_DIM     128
/* Floats in one split-KV softmax partial of a (slot, kv head): m[8], l[8], o[8][256]. */
#define KERNEL_ATTN_PARTIAL_FLOATS (8 + 8 + 8 * 256)

/* ------------------------------------------------------------------ lifecycle
 * Mirrors kernel_vk_shutdown / kernel_vk_trim_scratch (kernels.h:95-100). */

/* Select and initialise a device (primary context). 0 = ok, -1 = no usable sm_100 device. */
int  kernel_cuda_init(int device);
/* Free every library-owned device/pinned buffer. The library can be re-initialised. */
void kernel_cuda_shutdown(void);
/* Free the grow-only scratch (split-KV partials, staging); recreated on demand. Step groups then
 * run their recorded projection calls plainly once and record them again. */
void kernel_cuda_trim_scratch(void);
/* Stream for all subsequent work (a cudaStream_t; NULL = the legacy default stream). */
int  kernel_cuda_set_stream(void *stream);
/* Wait for the stream; 0 = ok, -1 = a CUDA error or a kernel-recorded failure (cleared). */
int  kernel_cuda_synchronize(void);
/* Text of the last failure recorded by the library (never NULL). */
const char *kernel_cuda_last_error(void);
/* Number of kernels this library launched since load (diagnostics / bench accounting). */
uint64_t kernel_cuda_launch_count(void);

/* ------------------------------------------------------------------ buffer residency
 * Replaces locked_calloc_checked / locked_buffer_free for KVCache.k/.v and SSMState.state
 * (model.c:54-99, 355-461) and the host memcpy/memmove that touch them (kvwindow.c, state.c). */

void *kernel_cuda_alloc(size_t bytes);                 /* zero-filled device memory, NULL on failure */
int   kernel_cuda_free(void *ptr);
int   kernel_cuda_upload(void *dst_dev, const void *src_host, size_t bytes);   /* synchronous */
int   kernel_cuda_download(void *dst_host, const void *src_dev, size_t bytes); /* synchronous */
int   kernel_cuda_memmove(void *dst_dev, const void *src_dev, size_t bytes);   /* overlap-safe, async */
int   kernel_cuda_memset(void *dst_dev, int value, size_t bytes);              /* async (model_reset) */
/* n f16 values of a device window (KVCache.k / .v rows) to host fp32, and host fp32 to device
 * f16 (round to nearest even): the state file's KV blocks (state.c:39 and 66 write and read
 * fp32 rows; the device window holds them as f16, and values that came from it convert back
 * exactly). Synchronous. */
int   kernel_cuda_download_f16_f32(float *dst_host, const uint16_t *src_dev, size_t n);
int   kernel_cuda_upload_f32_f16(uint16_t *dst_dev, const float *src_host, size_t n);

/* Register a long-lived host buffer (the model's attn_q / attn_k / attn_v / attn_out,
 * DeltaNet q / k / v / g / beta / out, model.c:801-861 and 1291-1343) once: its pages are
 * pinned (cudaHostRegister). When every buffer of a call to the host-buffer entry points
 * (kernel_attn_decode_batch_host, kernel_deltanet_step_batch_host) lies in registered memory,
 * the copy engine moves them directly, a few large copies per call (the buffers' contiguous
 * runs), with no staging memcpy on the host, overlapped with the call's kernels where the data
 * allows (gates beside the decode kernel; DeltaNet inputs and outputs in chunks on two more
 * streams); other calls go through pinned staging as before.
 * A buffer must not be freed while registered. 0 = ok, -1 = error (e.g. pages already
 * registered). */
int   kernel_cuda_host_register(void *ptr, size_t bytes);
int   kernel_cuda_host_unregister(void *ptr);

/* ------------------------------------------------------------------ gated attention, decode
 * Replaces model.c:801-861 (Q|G split, q/k RMSNorm, partial RoPE, KV append, GQA softmax
 * attention over the window, sigmoid output gate) for one token per slot. */

typedef struct {
    const float *q;          /* 16 rows of 256 floats, `qg_stride` floats apart                */
    const float *gate;       /* 16 rows of 256 gate logits, same stride                        */
    size_t qg_stride;        /* 256 for separate buffers, 512 for the interleaved projection    */
                             /* [Q0|G0|Q1|G1|...] (then q = qg, gate = qg + 256)                */
    const float *k_new;      /* [2][256] raw K projection of the new token                       */
    const float *v_new;      /* [2][256] V projection of the new token                           */
    const float *q_norm;     /* [256] attn_q_norm weight                                         */
    const float *k_norm;     /* [256] attn_k_norm weight                                         */
    uint16_t *k_cache;       /* f16 [capacity][2][256], device, 16-byte aligned                  */
    uint16_t *v_cache;       /* f16 [capacity][2][256]                                           */
    size_t capacity;         /* window capacity in tokens                                        */
    size_t length;           /* cached tokens before this step; the new token is written at     */
                             /* index `length` (must be < capacity when append != 0)            */
    size_t position;         /* absolute RoPE position of the new token                          */
    float *out;              /* [16][256] gated attention output                                 */
    int append;              /* 1 = normal decode. 0 = this window slice takes no new token and  */
                             /* k_new/v_new/gate/out are unused (split-KV partial mode only)     */
} KernelAttnDecodeJob;

/* Device-pointer batch: every pointer in every job is device memory. Asynchronous. The new
 * token attends at fp32 in this step and is stored rounded to f16 for later steps. */
int kernel_attn_decode_batch(const KernelAttnDecodeJob *jobs, int n);

/* Same, with q/gate/k_new/v_new/q_norm/k_norm/out in HOST memory (caches on the device).
 * Synchronous: returns when every `out` holds its result. */
int kernel_attn_decode_batch_host(const KernelAttnDecodeJob *jobs, int n);

/* Allocation-free form of kernel_attn_decode_batch. It has no counterpart in the reference: it
 * exists for callers that must not allocate device memory once they are serving -- a host
 * running under a device-memory budget fixed at start-up, or code that may not enter the CUDA
 * allocator (or an allocating library such as torch's caching allocator) at decode time.
 * It never calls cudaMalloc/cudaFree: its scratch (the split softmax partial records) is one
 * statically sized 8 MiB device array that every GPU loading this library holds until the
 * process exits. Limits: at most 64 slots per call (more is rejected with an error);
 * windows of any length (the split size grows so the partials fit the array).
 * Device: the call runs on the current device, which must be the one kernel_cuda_init chose;
 * kernel_cuda_init (which allocates the library's 256-byte error word) must run once at
 * start-up, and a call made with another device current is rejected with an error. Failures a
 * kernel records (a bounded wait that ran out, an argument it cannot process) land in that
 * error word and are reported by kernel_cuda_synchronize, as for kernel_attn_decode_batch.
 * The first call on each device does a one-time set-up (it looks up the array's device address
 * and the SM count) and should come before any stream capture. Every call shares the one array
 * (each call writes every record it reads, so nothing needs clearing between calls), so calls
 * whose work overlaps on the GPU (different streams, or different threads) race and must be
 * serialised by the caller. Same job semantics,
 * results and asynchrony as kernel_attn_decode_batch, on the library stream; all pointers device
 * memory. */
int kernel_attn_decode_batch_noalloc(const KernelAttnDecodeJob *jobs, int n);

/* Drop-in for full_attention's core (model.c:801-861) with model.c's own host buffers:
 * q_gate = the interleaved [16][512] projection, k_new/v_new = attn_k/attn_v [512],
 * q_norm/k_norm = R->qnorm/R->knorm, caches = the device-resident KVCache.k/.v, out = attn_out
 * [4096]. The caller then increments kv->length. Synchronous. */
int kernel_attn_decode(const float *q_gate, const float *k_new, const float *v_new,
                       const float *q_norm, const float *k_norm,
                       uint16_t *k_cache, uint16_t *v_cache, size_t capacity,
                       size_t length, size_t position, float *out);

/* Split-KV partial mode (long-context decode with the window split across GPUs): each job
 * covers this GPU's slice of a slot's window (`length` cached tokens in its own cache buffers);
 * the job with append = 1 also appends and scores the new token. Writes, per job and kv head,
 * one merged softmax partial of KERNEL_ATTN_PARTIAL_FLOATS floats to
 * partials[(job * 2 + kv_head) * KERNEL_ATTN_PARTIAL_FLOATS]: m[8] (max score, log2 units),
 * l[8] (sum of exp2(s - m)), o[8][256] (output normalised by l). Device pointers, async. */
int kernel_attn_decode_partial_batch(const KernelAttnDecodeJob *jobs, int n, float *partials);

/* Merge `nparts` partial buffers laid out [nparts][n][2][KERNEL_ATTN_PARTIAL_FLOATS] (e.g. one
 * per GPU after an all-gather) and apply the sigmoid gate: out_j = merged o * sigmoid(gate_j).
 * gates/outs: n device pointers each (16 rows of 256, gate rows `qg_stride` apart). Async. */
int kernel_attn_merge_partials(const float *partials, int nparts, int n,
                               const float *const *gates, size_t qg_stride,
                               float *const *outs);

/* Split-KV decode with the combine fused into the kernels (long-context decode across GPUs,
 * the exchange step of model.c:825-856 when the window is split): like
 * kernel_attn_decode_partial_batch, but job i's merged partial goes straight to dst[i] (two
 * records of KERNEL_ATTN_PARTIAL_FLOATS floats, kv head 0 then 1; 16-byte aligned), which may
 * be another GPU's memory opened with kernel_cuda_ipc_open (plain peer stores over NVLink), and
 * once a query head's part of a record is visible to every GPU, its tag
 * tags[i][kv_head * 8 + head] (16 words per job) is set to `epoch`. No collective library call:
 * the home GPU of a slot waits on the tags in kernel_attn_merge_wait. Async. */
int kernel_attn_decode_partial_push(const KernelAttnDecodeJob *jobs, int n, float *const *dst,
                                    unsigned *const *tags, unsigned epoch);

/* The home GPU's half of the fused combine: recv [nparts][n][2][KERNEL_ATTN_PARTIAL_FLOATS]
 * and tags [nparts][n][2][8] in this GPU's memory, filled by kernel_attn_decode_partial_push
 * on the nparts GPUs. Each (job, kv head, query head) waits until its nparts tags equal `epoch`
 * (bounded: a wait that runs out sets the error word kernel_cuda_synchronize reports, and that
 * output is not written), then merges as kernel_attn_merge_partials. A buffer may be reused for the
 * step after next (double buffering by step parity keeps a fast GPU from overwriting records
 * the home GPU has not merged yet). Async. */
int kernel_attn_merge_wait(const float *recv, const unsigned *tags, int nparts, int n,
                           const float *const *gates, size_t qg_stride, float *const *outs,
                           unsigned epoch);

/* Inter-process access to device memory (cudaIpcGetMemHandle / cudaIpcOpenMemHandle): the
 * handle of a buffer from kernel_cuda_alloc, exchanged between the processes of a job by the
 * caller, opens as a device pointer to that buffer on its GPU (peer access over NVLink).
 * KERNEL_CUDA_IPC_HANDLE_BYTES bytes of handle. 0 = ok, -1 = error. */
#define KERNEL_CUDA_IPC_HANDLE_BYTES 64
int kernel_cuda_ipc_handle(void *dev_ptr, void *handle);
int kernel_cuda_ipc_open(const void *handle, void **dev_ptr);
int kernel_cuda_ipc_close(void *dev_ptr);

/* ------------------------------------------------------------------ gated attention, prefill
 * Replaces pf_attention's attention part (model.c:1553-1600): per token q/k RMSNorm and partial
 * RoPE at position base + t, append of all T tokens' K/V at window index kbase + t, then causal
 * GQA attention of token t over window entries [0, kbase + t], times sigmoid(gate). */

#define KERNEL_DTYPE_F32  0
#define KERNEL_DTYPE_BF16 1

typedef struct {
    const void *q;           /* token t, head h at q + t*qg_tok_stride + h*qg_stride (elements)  */
    const void *gate;        /* same strides as q                                                */
    size_t qg_stride;        /* 256, or 512 for the interleaved [Q0|G0|Q1|G1|...] projection     */
    size_t qg_tok_stride;    /* elements from one token to the next (4096 or 8192)                */
    const void *k;           /* [T][2][256] raw K projections                                    */
    const void *v;           /* [T][2][256] V projections                                        */
    const float *q_norm;     /* [256]                                                            */
    const float *k_norm;     /* [256]                                                            */
    uint16_t *k_cache;       /* f16 [capacity][2][256], device, 16-byte aligned                  */
    uint16_t *v_cache;
    size_t capacity;         /* kbase + T must not exceed it                                     */
    size_t kbase;            /* tokens already in the window (the chunk appends after them)     */
    size_t base;             /* absolute RoPE position of token 0                                */
    size_t T;                /* tokens in this chunk (>= 1)                                      */
    float *out;              /* [T][16][256] gated attention output                              */
    int dtype;               /* element type of q, gate, k, v: KERNEL_DTYPE_F32 or _BF16         */
} KernelAttnPrefillJob;

/* Device-pointer batch (e.g. several prompts). Asynchronous. Tensor-core operands are f16. */
int kernel_attn_prefill_batch(const KernelAttnPrefillJob *jobs, int n);

/* Drop-in for pf_attention's core with its own host buffers (T <= 256 in the reference):
 * q_gate = p->qkv [T][8192] interleaved Q|G, k/v = p->k, p->v [T][512], caches device-resident,
 * kbase = kv->length, base = the absolute position; out = p->rec [T][4096]. The caller then sets
 * kv->length = kbase + T. Synchronous. */
int kernel_attn_prefill(const float *q_gate, const float *k, const float *v, const float *q_norm,
                        const float *k_norm, uint16_t *k_cache, uint16_t *v_cache, size_t capacity,
                        size_t kbase, size_t base, size_t T, float *out);

/* ------------------------------------------------------------------ Gated DeltaNet, decode
 * Replaces recurrent_delta_step (model.c:272-323): per value head vh (key head vh % 16),
 * d = exp(g), delta = (v - d S^T k) beta, out = (d S^T q + (k.q) delta) / sqrt(128),
 * S <- d S + k delta^T, one read and one write of the state. */

typedef struct {
    float *state;            /* fp32 [32][128][128], device, updated in place                    */
    const float *q;          /* [16][128] L2-normalised                                          */
    const float *k;          /* [16][128] L2-normalised                                          */
    const float *v;          /* [32][128]                                                        */
    const float *g;          /* [32] log decay (the `decay`/alpha argument of model.c:272)       */
    const float *beta;       /* [32] sigmoid(beta)                                               */
    float *out;              /* [32][128]                                                        */
} KernelDeltaStepJob;

/* Device-pointer batch (independent states: slots and/or layers). Asynchronous. */
int kernel_deltanet_step_batch(const KernelDeltaStepJob *jobs, int n);

/* Same, with q/k/v/g/beta/out in HOST memory (states on the device). Synchronous: one packed
 * host->device copy of all inputs, the device batch, one device->host copy of all outputs. */
int kernel_deltanet_step_batch_host(const KernelDeltaStepJob *jobs, int n);

/* Drop-in for recurrent_delta_step(&ssm_state[layer], q, k, v, alpha, beta, out) with host
 * q/k/v/g/beta/out and the device-resident state. Synchronous. */
int kernel_deltanet_step(float *state, const float *q, const float *k, const float *v,
                         const float *g, const float *beta, float *out);

/* ------------------------------------------------------------ Gated DeltaNet prefill
 * Replaces the per-token delta_head loop of pf_ssm (reference src/model.c:1644-1658; the
 * recurrence of delta_head, model.c:1507-1534) with the chunked form (chunk 64) on the tensor
 * cores. Same layouts as that loop: q, k [T][16][128] (L2-normalised by the caller, value head
 * vh reads key head vh % 16), v [T][32][128], g (log-decay) and beta [T][32], out
 * [T][32][128] = S_t^T q_t / sqrt(128) per token, before the gated RMSNorm. The state
 * [32][128 key][128 value] is read at the start and holds S_T on return. */
typedef struct {
    float *state;               /* device, [32][128][128] fp32, updated in place */
    const float *q, *k;         /* device, [T][16][128], 16-byte aligned */
    const float *v;             /* device, [T][32][128], 16-byte aligned */
    const float *g, *beta;      /* device, [T][32] */
    float *out;                 /* device, [T][32][128] */
    size_t T;                   /* tokens (0 = nothing to do) */
} KernelDeltaPrefillJob;

/* Device-pointer batch: one job per prompt (independent states). Asynchronous. */
int kernel_deltanet_prefill_batch(const KernelDeltaPrefillJob *jobs, int n);

/* Drop-in for one pf_ssm recurrence: host q/k/v/g/beta/out, device-resident state.
 * Synchronous. */
int kernel_deltanet_prefill(float *state, size_t T, const float *q, const float *k, const float *v,
                            const float *g, const float *beta, float *out);

/* ------------------------------------------------------------ Gated DeltaNet pre/post ops
 * Pre-ops (model.c:1291-1328 for a decode token; pf_ssm's prep loop 1619-1643 for a prompt), per
 * token t of a recurrent layer: depthwise causal conv1d (kernel 4) of the qkv projection over
 * the 3-token history (kernel_conv1d_causal_f32, kernels.c:693-719), SiLU, history shift, split
 * into q | k | v with q, k L2-normalised per 128 (eps 1e-6), beta' = sigmoid(beta) and
 * g = a * softplus(alpha + dt) (softplus(x) = x above 20). T = 1 is a decode step; T > 1 runs
 * the tokens in order (token t's conv sees the raw inputs of t-3 .. t-1). */
typedef struct {
    const float *qkv;           /* device, [T][8192] raw projection */
    const float *alpha, *beta;  /* device, [T][32] raw projections */
    float *conv_state;          /* device, [3][8192] history (oldest row first), updated */
    const float *conv_w;        /* device, [8192][4] (ssm_conv1d.weight), 16-byte aligned */
    const float *dt, *a;        /* device, [32] */
    float *q, *k;               /* device out, [T][16][128] */
    float *v;                   /* device out, [T][32][128] */
    float *g, *beta_out;        /* device out, [T][32] */
    size_t T;
} KernelDeltaPreopJob;

/* Device-pointer batch (one job per layer and slot/prompt). Asynchronous. */
int kernel_deltanet_preop_batch(const KernelDeltaPreopJob *jobs, int n);

/* Post-op (model.c:1333-1343; pf_ssm 1655-1658): per (token, value head) row of 128,
 * out = rmsnorm(out) * norm_w (eps 1e-6) * z * sigmoid(z), in place. */
typedef struct {
    float *out;                 /* device, [T][32][128], 16-byte aligned, updated */
    const float *z;             /* device, [T][4096] gate projection */
    const float *norm_w;        /* device, [128] (ssm_norm.weight) */
    size_t T;
} KernelDeltaPostopJob;

int kernel_deltanet_postop_batch(const KernelDeltaPostopJob *jobs, int n);

/* The whole recurrent-layer block of a decode step, model.c:1291-1343 without the projections:
 * pre-ops, the delta-rule step, gated RMSNorm. Host qkv [8192], z [4096], alpha, beta [32] in;
 * host out [4096] (before ssm_out). Device-resident state [32][128][128], conv_state [3][8192],
 * conv_w [8192][4], dt, a [32], ssm_norm [128]. Synchronous. */
int kernel_deltanet_layer_step(float *state, float *conv_state, const float *conv_w, const float *dt,
                               const float *a, const float *ssm_norm, const float *qkv, const float *z,
                               const float *alpha, const float *beta, float *out);

/* The same for a prompt of T tokens: pf_ssm (model.c:1604-1660) without its projections, the
 * recurrence in the chunked tensor-core form. Host qkv [T][8192], z [T][4096], alpha, beta
 * [T][32]; host out [T][4096]. Synchronous. */
int kernel_deltanet_layer_prefill(float *state, float *conv_state, const float *conv_w, const float *dt,
                                  const float *a, const float *ssm_norm, size_t T, const float *qkv,
                                  const float *z, const float *alpha, const float *beta, float *out);

/* Diagnostic: launch a kernel whose bounded mbarrier wait cannot complete (nothing arrives) with
 * a budget of `budget_cycles` SM cycles, and return the device error bits it recorded (1 = a
 * bounded wait timed out), clearing them; -1 if the launch failed. Exercises the path every
 * pipelined kernel takes instead of hanging when a partner never signals: the kernel returns,
 * the error surfaces at the next synchronize, the context stays usable. */
int kernel_cuda_wait_probe(long long budget_cycles);

/* ------------------------------------------------------------ attention window (device KV)
 * The attention window of one slot with its K/V in device memory (f16 [ctx][2][256] per
 * attention layer) and the policy of kvwindow.c: a kept head (slide_keep / slide_pin), sliding
 * in blocks of a quarter of the free window when full, evicted tokens pushed to a spill store in
 * kvspill.c's fp32 chunk format (a file when `spill_path` is non-empty, host memory otherwise),
 * restore / rollback / context changes as in kvwindow.c:1-268 and model_set_context
 * (model.c:1870-1899). Calls are synchronous with respect to the host (the spill moves data). */
typedef struct KernelKvWindow KernelKvWindow;

/* NULL on failure (kernel_cuda_last_error()). layers <= 64. */
KernelKvWindow *kernel_kvw_create(int layers, size_t ctx, int slide, size_t keep, size_t pin,
                                  const char *spill_path);
void kernel_kvw_destroy(KernelKvWindow *w);
int kernel_kvw_set_policy(KernelKvWindow *w, int slide, size_t keep, size_t pin);

/* Device K/V of attention layer `layer` (0-based among the window's layers); the pointers change
 * when the context size changes. */
uint16_t *kernel_kvw_k(KernelKvWindow *w, int layer);
uint16_t *kernel_kvw_v(KernelKvWindow *w, int layer);

size_t kernel_kvw_len(const KernelKvWindow *w);        /* kvw_len: tokens in the window */
size_t kernel_kvw_spilled(const KernelKvWindow *w);    /* kvw_spilled */
size_t kernel_kvw_head(const KernelKvWindow *w);       /* kvw_head */
size_t kernel_kvw_max_chunk(const KernelKvWindow *w);  /* kvw_max_chunk */
size_t kernel_kvw_position(const KernelKvWindow *w);   /* absolute position of the next token */
size_t kernel_kvw_context(const KernelKvWindow *w);    /* context_length */

/* kvw_ensure_room: make room for `need` more tokens (sliding if enabled). Then the attention
 * kernels append at index kernel_kvw_len() (position kernel_kvw_position()), and
 * kernel_kvw_appended(w, need) records them. */
int kernel_kvw_ensure_room(KernelKvWindow *w, size_t need);
int kernel_kvw_appended(KernelKvWindow *w, size_t n);
int kernel_kvw_evict(KernelKvWindow *w, size_t n);                    /* kvw_evict */
int kernel_kvw_restore(KernelKvWindow *w, size_t n);                  /* kvw_restore */
int kernel_kvw_rollback(KernelKvWindow *w, size_t p0, size_t s0);     /* kvw_rollback */
int kernel_kvw_set_context(KernelKvWindow *w, size_t ctx);            /* model_set_context's window part */

/* ------------------------------------------------------------ k-quant projections (decode)
 * Replaces kernel_matvec_quant_batch (kernels.h:30-44; CPU matvec_q4_cpu / matvec_q6_cpu,
 * kernels.c:405-431, 553-578): y[r] = dot(W[r], x) for Q4_K (144-byte blocks) or Q6_K (210-byte
 * blocks) rows of cols/256 blocks, weights resident in device memory (uploaded once). Jobs are
 * independent (no job reads another's output). cols must be a positive multiple of 256; vector
 * and output 16-byte aligned; a Q4_K matrix 16-byte aligned, a Q6_K matrix 2-byte aligned (16
 * bytes for the fast path). Device pointers, asynchronous. */
typedef struct {
    int is_q6;                  /* 0 = Q4_K, 1 = Q6_K */
    const void *matrix;         /* device, rows x cols quantized */
    const float *vector;        /* device, [cols] */
    float *output;              /* device, [rows] */
    size_t rows, cols;
} KernelCudaMatvecJob;

int kernel_cuda_matvec_quant_batch(const KernelCudaMatvecJob *jobs, int n);

/* Replaces kernel_matmul_quant_batch (kernels.h:51-64; CPU matmul_quant_cpu, kernels.c:1877-1913):
 * multi-token (prefill) projections Y[t*rows + r] = dot(W[r], X[t*cols ...]) for t < T. Same
 * job validity as the reference (non-null pointers, rows, cols, T > 0, cols a multiple of 256,
 * each dimension at most 2^32 - 1; -1 otherwise) plus the alignment of
 * kernel_cuda_matvec_quant_batch (X 16-byte aligned). Device pointers, asynchronous. Jobs whose
 * matrix is 16-byte aligned with rows a multiple of 16 bytes run token-batched: jobs of 64 or
 * more tokens on the tcgen05 tensor cores (a CTA per tile of 128 rows x 64 tokens; a call with
 * fewer tiles than SMs splits its larger jobs along the blocks into parts summed in a fixed
 * order) when together they make at least 64 tiles, the other jobs of 8 or more tokens (at most
 * 128 blocks a row) on
 * the warp MMA (256 rows x 32 tokens per CTA, split along the blocks when there are few tiles);
 * the rest run as T matrix-vector products sharing the (L2-resident) weights.
 * Results do not depend on the route beyond fp32 summation order, and repeat bit for bit. */
typedef struct {
    int is_q6;                  /* 0 = Q4_K, 1 = Q6_K */
    const void *matrix;         /* device, rows x cols quantized */
    const float *X;             /* device, [T][cols] */
    float *Y;                   /* device, [T][rows] */
    size_t rows, cols, T;
} KernelCudaMatmulJob;

int kernel_cuda_matmul_quant_batch(const KernelCudaMatmulJob *jobs, int n);

/* ------------------------------------------------------------ cross-slot batched step
 * The batched counterpart of the reference's step lock (FairLock, slots.c:77-105, taken once
 * per token by step_forward, slots.c:864-880): instead of running one slot's model step at a
 * time, the slot threads that are decoding meet in rounds, and the i-th hot-path call of every
 * member of a round becomes ONE device batch -- the members' attention jobs one
 * kernel_attn_decode_batch, their DeltaNet jobs one kernel_deltanet_step_batch, their k-quant
 * projections one kernel_cuda_matmul_quant_batch in which the members' vectors for the same
 * weight matrix form the tokens of one multi-token product (the weights are read once per round
 * instead of once per slot).
 *
 * Protocol, per slot thread: kernel_step_group_join once when the slot starts decoding; per
 * token, kernel_step_group_begin, the layer calls in model order, kernel_step_group_end;
 * kernel_step_group_leave when the slot stops. A round forms when every joined member has
 * called begin, or `straggler_us` after the first begin, with whoever has begun; the others
 * take the next round. Every member of a round must make the same calls in the same order
 * (`site` names the call, e.g. layer * 16 + op, and must agree); a call runs once every member
 * of the round that has not ended has reached it, on the thread that arrives last. Jobs hold
 * device pointers; the batch is asynchronous on the library stream, like the calls it replaces.
 * A call returns the device batch's status to every member of it (0 / -1). A member that does
 * not reach a call within `call_timeout_ms` fails that call for all (-1, message in
 * kernel_cuda_last_error) and the rest of the round's calls (they return -1 at once); the
 * round still ends normally. Work outside rounds (prefill chunks, rollbacks) takes
 * kernel_step_group_lock / unlock, the FIFO lock the group's own batches also run under, which
 * keeps the single-stream, non-overlapping rule of this library. All functions are thread-safe;
 * none may be called with the group lock held except kernel_step_group_unlock.
 * Projection calls are recorded: slots that keep their buffers bring the same job list
 * (matrices, vectors, outputs, shapes, in member order) every token, so the second occurrence of
 * a list is captured into a CUDA graph on a stream of the group's own and later ones replay it
 * (one graph launch instead of the call's host work and launches), as long as the library's
 * own buffers are the ones the recording used; a list that cannot be recorded runs as plain
 * launches. The environment variable ROASTER_STEP_GRAPHS=0 turns recording off. */
typedef struct KernelStepGroup KernelStepGroup;

typedef struct {
    unsigned long long rounds;       /* rounds formed */
    unsigned long long calls;        /* combined calls run (one device batch each) */
    unsigned long long jobs;         /* member jobs those calls carried */
    unsigned long long products;     /* projections merged: weight matrices shared by 2+ members */
    unsigned long long merged_jobs;  /* member projection jobs inside those merged products */
    unsigned long long errors;       /* calls that returned -1 */
    int max_round;                   /* largest round */
    int members;                     /* members joined now */
    unsigned long long replayed;     /* projection calls replayed from a recording (a CUDA graph
                                        of the same job list's earlier launches) */
} KernelStepGroupStats;

/* max_members >= 1; straggler_us >= 0; call_timeout_ms > 0. NULL on bad arguments. */
KernelStepGroup *kernel_step_group_create(int max_members, long long straggler_us, long long call_timeout_ms);
/* Waits for no one: destroy only when no thread is inside the group. Frees its device buffers. */
void kernel_step_group_destroy(KernelStepGroup *g);
int  kernel_step_group_join(KernelStepGroup *g);                /* member id >= 0, -1 when full */
int  kernel_step_group_leave(KernelStepGroup *g, int member);   /* outside a round only */
int  kernel_step_group_begin(KernelStepGroup *g, int member);   /* size of the round joined, or -1 */
int  kernel_step_group_end(KernelStepGroup *g, int member);
int  kernel_step_group_attn(KernelStepGroup *g, int member, int site, const KernelAttnDecodeJob *job);
int  kernel_step_group_delta(KernelStepGroup *g, int member, int site, const KernelDeltaStepJob *job);
int  kernel_step_group_matvec(KernelStepGroup *g, int member, int site, const KernelCudaMatvecJob *jobs, int n);
int  kernel_step_group_lock(KernelStepGroup *g);
int  kernel_step_group_unlock(KernelStepGroup *g);
int  kernel_step_group_stats(const KernelStepGroup *g, KernelStepGroupStats *out);

#ifdef __cplusplus
}
#endif
#endif
