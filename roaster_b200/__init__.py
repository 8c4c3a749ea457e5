"""roaster_b200 -- B200 (sm_100a) hybrid-attention hot path behind a plain-C ABI.

The product is ``libroaster_b200.so`` (CUDA kernels + the C-ABI declared in
``include/roaster_cuda.h``). This module is a thin ctypes binding for Python callers (tests,
bench.py): it mirrors the C job structs and forwards to the library. There is no fallback --
if the library is missing, or no B200 is present, calls raise.

Device buffers are passed as raw addresses (e.g. ``torch.Tensor.data_ptr()``); the library never
sees torch types.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libroaster_b200.so")
HEADER = os.path.join(HERE, "..", "include", "roaster_cuda.h")

ATTN_Q_HEADS = 16
ATTN_KV_HEADS = 2
ATTN_HEAD_DIM = 256
DN_K_HEADS = 16
DN_V_HEADS = 32
DN_HEAD_DIM = 128
ATTN_PARTIAL_FLOATS = 8 + 8 + 8 * 256

_vp = C.c_void_p
_sz = C.c_size_t


class KernelAttnDecodeJob(C.Structure):
    """Mirror of ``KernelAttnDecodeJob`` (include/roaster_cuda.h)."""
    _fields_ = [
        ("q", _vp), ("gate", _vp), ("qg_stride", _sz), ("k_new", _vp), ("v_new", _vp),
        ("q_norm", _vp), ("k_norm", _vp), ("k_cache", _vp), ("v_cache", _vp),
        ("capacity", _sz), ("length", _sz), ("position", _sz), ("out", _vp), ("append", C.c_int),
    ]


class KernelAttnPrefillJob(C.Structure):
    """Mirror of ``KernelAttnPrefillJob`` (include/roaster_cuda.h)."""
    _fields_ = [
        ("q", _vp), ("gate", _vp), ("qg_stride", _sz), ("qg_tok_stride", _sz), ("k", _vp),
        ("v", _vp), ("q_norm", _vp), ("k_norm", _vp), ("k_cache", _vp), ("v_cache", _vp),
        ("capacity", _sz), ("kbase", _sz), ("base", _sz), ("T", _sz), ("out", _vp),
        ("dtype", C.c_int),
    ]


class KernelDeltaStepJob(C.Structure):
    """Mirror of ``KernelDeltaStepJob`` (include/roaster_cuda.h)."""
    _fields_ = [("state", _vp), ("q", _vp), ("k", _vp), ("v", _vp), ("g", _vp), ("beta", _vp),
                ("out", _vp)]


class KernelDeltaPrefillJob(C.Structure):
    """Mirror of ``KernelDeltaPrefillJob`` (include/roaster_cuda.h)."""
    _fields_ = [("state", _vp), ("q", _vp), ("k", _vp), ("v", _vp), ("g", _vp), ("beta", _vp),
                ("out", _vp), ("T", _sz)]


class KernelDeltaPreopJob(C.Structure):
    """Mirror of ``KernelDeltaPreopJob`` (include/roaster_cuda.h)."""
    _fields_ = [("qkv", _vp), ("alpha", _vp), ("beta", _vp), ("conv_state", _vp), ("conv_w", _vp),
                ("dt", _vp), ("a", _vp), ("q", _vp), ("k", _vp), ("v", _vp), ("g", _vp),
                ("beta_out", _vp), ("T", _sz)]


class KernelDeltaPostopJob(C.Structure):
    """Mirror of ``KernelDeltaPostopJob`` (include/roaster_cuda.h)."""
    _fields_ = [("out", _vp), ("z", _vp), ("norm_w", _vp), ("T", _sz)]


class KernelCudaMatmulJob(C.Structure):
    """Mirror of ``KernelCudaMatmulJob`` (include/roaster_cuda.h); the reference's KernelMatmulJob
    (src/kernels.h:57-63) with device pointers."""
    _fields_ = [("is_q6", C.c_int), ("matrix", _vp), ("X", _vp), ("Y", _vp), ("rows", _sz), ("cols", _sz),
                ("T", _sz)]


class KernelCudaMatvecJob(C.Structure):
    """Mirror of ``KernelCudaMatvecJob`` (include/roaster_cuda.h); the reference's KernelMatvecJob
    (src/kernels.h:34-41) with device pointers."""
    _fields_ = [("is_q6", C.c_int), ("matrix", _vp), ("vector", _vp), ("output", _vp), ("rows", _sz),
                ("cols", _sz)]


class KernelStepGroupStats(C.Structure):
    """Mirror of ``KernelStepGroupStats`` (include/roaster_cuda.h)."""
    _fields_ = [("rounds", C.c_ulonglong), ("calls", C.c_ulonglong), ("jobs", C.c_ulonglong),
                ("products", C.c_ulonglong), ("merged_jobs", C.c_ulonglong), ("errors", C.c_ulonglong),
                ("max_round", C.c_int), ("members", C.c_int), ("replayed", C.c_ulonglong)]


_lib = None


def lib():
    """Load libroaster_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m roaster_b200.build`")
    L = C.CDLL(LIB_PATH)
    sig = {
        "kernel_cuda_init": (C.c_int, [C.c_int]),
        "kernel_cuda_shutdown": (None, []),
        "kernel_cuda_trim_scratch": (None, []),
        "kernel_cuda_set_stream": (C.c_int, [_vp]),
        "kernel_cuda_synchronize": (C.c_int, []),
        "kernel_cuda_last_error": (C.c_char_p, []),
        "kernel_cuda_launch_count": (C.c_uint64, []),
        "kernel_cuda_alloc": (_vp, [_sz]),
        "kernel_cuda_free": (C.c_int, [_vp]),
        "kernel_cuda_upload": (C.c_int, [_vp, _vp, _sz]),
        "kernel_cuda_download": (C.c_int, [_vp, _vp, _sz]),
        "kernel_cuda_memmove": (C.c_int, [_vp, _vp, _sz]),
        "kernel_cuda_memset": (C.c_int, [_vp, C.c_int, _sz]),
        "kernel_cuda_host_register": (C.c_int, [_vp, _sz]),
        "kernel_cuda_download_f16_f32": (C.c_int, [_vp, _vp, _sz]),
        "kernel_cuda_upload_f32_f16": (C.c_int, [_vp, _vp, _sz]),
        "kernel_cuda_host_unregister": (C.c_int, [_vp]),
        "kernel_attn_decode_batch": (C.c_int, [C.POINTER(KernelAttnDecodeJob), C.c_int]),
        "kernel_attn_decode_batch_host": (C.c_int, [C.POINTER(KernelAttnDecodeJob), C.c_int]),
        "kernel_attn_decode_batch_noalloc": (C.c_int, [C.POINTER(KernelAttnDecodeJob), C.c_int]),
        "kernel_attn_decode": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _vp]),
        "kernel_attn_decode_partial_batch": (C.c_int, [C.POINTER(KernelAttnDecodeJob), C.c_int,
                                                       _vp]),
        "kernel_attn_merge_partials": (C.c_int, [_vp, C.c_int, C.c_int, C.POINTER(_vp), _sz,
                                                 C.POINTER(_vp)]),
        "kernel_attn_decode_partial_push": (C.c_int, [C.POINTER(KernelAttnDecodeJob), C.c_int,
                                                      C.POINTER(_vp), C.POINTER(_vp), C.c_uint]),
        "kernel_attn_merge_wait": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.POINTER(_vp), _sz,
                                             C.POINTER(_vp), C.c_uint]),
        "kernel_cuda_ipc_handle": (C.c_int, [_vp, _vp]),
        "kernel_cuda_ipc_open": (C.c_int, [_vp, C.POINTER(_vp)]),
        "kernel_cuda_ipc_close": (C.c_int, [_vp]),
        "kernel_attn_prefill_batch": (C.c_int, [C.POINTER(KernelAttnPrefillJob), C.c_int]),
        "kernel_attn_prefill": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _sz, _vp]),
        "kernel_deltanet_step_batch": (C.c_int, [C.POINTER(KernelDeltaStepJob), C.c_int]),
        "kernel_deltanet_step": (C.c_int, [_vp] * 7),
        "kernel_deltanet_step_batch_host": (C.c_int, [C.POINTER(KernelDeltaStepJob), C.c_int]),
        "kernel_deltanet_prefill_batch": (C.c_int, [C.POINTER(KernelDeltaPrefillJob), C.c_int]),
        "kernel_deltanet_prefill": (C.c_int, [_vp, _sz] + [_vp] * 6),
        "kernel_cuda_wait_probe": (C.c_int, [C.c_longlong]),
        "kernel_kvw_create": (_vp, [C.c_int, _sz, C.c_int, _sz, _sz, C.c_char_p]),
        "kernel_kvw_destroy": (None, [_vp]),
        "kernel_kvw_set_policy": (C.c_int, [_vp, C.c_int, _sz, _sz]),
        "kernel_kvw_k": (_vp, [_vp, C.c_int]),
        "kernel_kvw_v": (_vp, [_vp, C.c_int]),
        "kernel_kvw_len": (_sz, [_vp]),
        "kernel_kvw_spilled": (_sz, [_vp]),
        "kernel_kvw_head": (_sz, [_vp]),
        "kernel_kvw_max_chunk": (_sz, [_vp]),
        "kernel_kvw_position": (_sz, [_vp]),
        "kernel_kvw_context": (_sz, [_vp]),
        "kernel_kvw_ensure_room": (C.c_int, [_vp, _sz]),
        "kernel_kvw_appended": (C.c_int, [_vp, _sz]),
        "kernel_kvw_evict": (C.c_int, [_vp, _sz]),
        "kernel_kvw_restore": (C.c_int, [_vp, _sz]),
        "kernel_kvw_rollback": (C.c_int, [_vp, _sz, _sz]),
        "kernel_kvw_set_context": (C.c_int, [_vp, _sz]),
        "kernel_deltanet_preop_batch": (C.c_int, [C.POINTER(KernelDeltaPreopJob), C.c_int]),
        "kernel_deltanet_postop_batch": (C.c_int, [C.POINTER(KernelDeltaPostopJob), C.c_int]),
        "kernel_deltanet_layer_step": (C.c_int, [_vp] * 11),
        "kernel_deltanet_layer_prefill": (C.c_int, [_vp] * 6 + [_sz] + [_vp] * 5),
        "kernel_cuda_matvec_quant_batch": (C.c_int, [C.POINTER(KernelCudaMatvecJob), C.c_int]),
        "kernel_cuda_matmul_quant_batch": (C.c_int, [C.POINTER(KernelCudaMatmulJob), C.c_int]),
        "kernel_step_group_create": (_vp, [C.c_int, C.c_longlong, C.c_longlong]),
        "kernel_step_group_destroy": (None, [_vp]),
        "kernel_step_group_join": (C.c_int, [_vp]),
        "kernel_step_group_leave": (C.c_int, [_vp, C.c_int]),
        "kernel_step_group_begin": (C.c_int, [_vp, C.c_int]),
        "kernel_step_group_end": (C.c_int, [_vp, C.c_int]),
        "kernel_step_group_attn": (C.c_int, [_vp, C.c_int, C.c_int, C.POINTER(KernelAttnDecodeJob)]),
        "kernel_step_group_delta": (C.c_int, [_vp, C.c_int, C.c_int, C.POINTER(KernelDeltaStepJob)]),
        "kernel_step_group_matvec": (C.c_int, [_vp, C.c_int, C.c_int, C.POINTER(KernelCudaMatvecJob), C.c_int]),
        "kernel_step_group_lock": (C.c_int, [_vp]),
        "kernel_step_group_unlock": (C.c_int, [_vp]),
        "kernel_step_group_stats": (C.c_int, [_vp, C.POINTER(KernelStepGroupStats)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def header_symbols(path: str = HEADER) -> list[str]:
    """Names of the functions include/roaster_cuda.h declares."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kernel_\w+)\s*\(", text)))


def last_error() -> str:
    return (lib().kernel_cuda_last_error() or b"").decode()


def check(rc: int, what: str = "roaster_b200") -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed: {last_error()}")


def init(device: int = 0) -> None:
    check(lib().kernel_cuda_init(device), "kernel_cuda_init")


def set_stream(stream) -> None:
    """Use a CUDA stream (torch.cuda.Stream, raw handle int, or None for the default)."""
    handle = getattr(stream, "cuda_stream", stream)
    check(lib().kernel_cuda_set_stream(_vp(handle or 0)), "kernel_cuda_set_stream")


def synchronize() -> None:
    check(lib().kernel_cuda_synchronize(), "kernel_cuda_synchronize")


def launch_count() -> int:
    return int(lib().kernel_cuda_launch_count())


def _ptr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    return int(x.data_ptr())


def attn_job(q, gate, k_new, v_new, q_norm, k_norm, k_cache, v_cache, length, position, out,
             qg_stride: int = 256, append: bool = True, capacity: int | None = None):
    """Build a KernelAttnDecodeJob from tensors (or raw addresses)."""
    cap = capacity if capacity is not None else int(k_cache.shape[0])
    return KernelAttnDecodeJob(_ptr(q), _ptr(gate), qg_stride, _ptr(k_new), _ptr(v_new),
                               _ptr(q_norm), _ptr(k_norm), _ptr(k_cache), _ptr(v_cache), cap,
                               int(length), int(position), _ptr(out), 1 if append else 0)


def delta_job(state, q, k, v, g, beta, out):
    return KernelDeltaStepJob(_ptr(state), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta),
                              _ptr(out))


def delta_prefill_job(state, q, k, v, g, beta, out, T: int):
    return KernelDeltaPrefillJob(_ptr(state), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta),
                                 _ptr(out), int(T))


def _arr(struct, jobs):
    arr = (struct * len(jobs))(*jobs)
    return arr, len(jobs)


def attn_decode_batch(jobs) -> None:
    arr, n = _arr(KernelAttnDecodeJob, jobs)
    check(lib().kernel_attn_decode_batch(arr, n), "kernel_attn_decode_batch")


def attn_decode_batch_noalloc(jobs) -> None:
    """The allocation-free decode entry point (static 8 MiB device scratch, <= 64 slots)."""
    arr, n = _arr(KernelAttnDecodeJob, jobs)
    check(lib().kernel_attn_decode_batch_noalloc(arr, n), "kernel_attn_decode_batch_noalloc")


def attn_decode_batch_host(jobs) -> None:
    arr, n = _arr(KernelAttnDecodeJob, jobs)
    check(lib().kernel_attn_decode_batch_host(arr, n), "kernel_attn_decode_batch_host")


def attn_decode_partial_batch(jobs, partials) -> None:
    arr, n = _arr(KernelAttnDecodeJob, jobs)
    check(lib().kernel_attn_decode_partial_batch(arr, n, _ptr(partials)),
          "kernel_attn_decode_partial_batch")


def attn_merge_partials(partials, nparts: int, gates, outs, qg_stride: int = 256) -> None:
    n = len(gates)
    g = (_vp * n)(*[_ptr(x) for x in gates])
    o = (_vp * n)(*[_ptr(x) for x in outs])
    check(lib().kernel_attn_merge_partials(_ptr(partials), nparts, n, g, qg_stride, o),
          "kernel_attn_merge_partials")


def attn_decode_partial_push(jobs, dst, tags, epoch: int) -> None:
    """Split-KV partials pushed to per-job record addresses (any GPU), tags set to `epoch`."""
    arr, n = _arr(KernelAttnDecodeJob, jobs)
    d = (_vp * n)(*[_ptr(x) for x in dst])
    t = (_vp * n)(*[_ptr(x) for x in tags])
    check(lib().kernel_attn_decode_partial_push(arr, n, d, t, int(epoch) & 0xFFFFFFFF),
          "kernel_attn_decode_partial_push")


def attn_merge_wait(recv, tags, nparts: int, gates, outs, epoch: int, qg_stride: int = 256) -> None:
    n = len(gates)
    g = (_vp * n)(*[_ptr(x) for x in gates])
    o = (_vp * n)(*[_ptr(x) for x in outs])
    check(lib().kernel_attn_merge_wait(_ptr(recv), _ptr(tags), nparts, n, g, qg_stride, o,
                                       int(epoch) & 0xFFFFFFFF), "kernel_attn_merge_wait")


IPC_HANDLE_BYTES = 64


def ipc_handle(ptr) -> bytes:
    """The inter-process handle of a kernel_cuda_alloc buffer."""
    buf = C.create_string_buffer(IPC_HANDLE_BYTES)
    check(lib().kernel_cuda_ipc_handle(_ptr(ptr), buf), "kernel_cuda_ipc_handle")
    return buf.raw


def ipc_open(handle: bytes) -> int:
    """Open another process's buffer by its handle; returns the device address."""
    out = _vp()
    check(lib().kernel_cuda_ipc_open(C.create_string_buffer(handle, IPC_HANDLE_BYTES), C.byref(out)),
          "kernel_cuda_ipc_open")
    return int(out.value)


def ipc_close(ptr: int) -> None:
    check(lib().kernel_cuda_ipc_close(_ptr(ptr)), "kernel_cuda_ipc_close")


def attn_prefill_batch(jobs) -> None:
    """jobs: KernelAttnPrefillJob instances or tuples of its fields in order."""
    js = [j if isinstance(j, KernelAttnPrefillJob) else KernelAttnPrefillJob(*j) for j in jobs]
    arr, n = _arr(KernelAttnPrefillJob, js)
    check(lib().kernel_attn_prefill_batch(arr, n), "kernel_attn_prefill_batch")


def deltanet_step_batch_host(jobs) -> None:
    arr, n = _arr(KernelDeltaStepJob, jobs)
    check(lib().kernel_deltanet_step_batch_host(arr, n), "kernel_deltanet_step_batch_host")


def deltanet_step_batch(jobs) -> None:
    arr, n = _arr(KernelDeltaStepJob, jobs)
    check(lib().kernel_deltanet_step_batch(arr, n), "kernel_deltanet_step_batch")


def deltanet_prefill_batch(jobs) -> None:
    arr, n = _arr(KernelDeltaPrefillJob, jobs)
    check(lib().kernel_deltanet_prefill_batch(arr, n), "kernel_deltanet_prefill_batch")


def deltanet_preop_batch(jobs) -> None:
    js = [j if isinstance(j, KernelDeltaPreopJob) else KernelDeltaPreopJob(*[_ptr(x) for x in j[:-1]], int(j[-1]))
          for j in jobs]
    arr, n = _arr(KernelDeltaPreopJob, js)
    check(lib().kernel_deltanet_preop_batch(arr, n), "kernel_deltanet_preop_batch")


def deltanet_postop_batch(jobs) -> None:
    js = [j if isinstance(j, KernelDeltaPostopJob) else KernelDeltaPostopJob(*[_ptr(x) for x in j[:-1]], int(j[-1]))
          for j in jobs]
    arr, n = _arr(KernelDeltaPostopJob, js)
    check(lib().kernel_deltanet_postop_batch(arr, n), "kernel_deltanet_postop_batch")


def matvec_quant_batch(jobs) -> None:
    """kernel_cuda_matvec_quant_batch over jobs given as KernelCudaMatvecJob or
    (is_q6, matrix, vector, output, rows, cols) with device tensors or addresses."""
    js = [j if isinstance(j, KernelCudaMatvecJob) else
          KernelCudaMatvecJob(int(bool(j[0])), _ptr(j[1]), _ptr(j[2]), _ptr(j[3]), int(j[4]), int(j[5]))
          for j in jobs]
    arr, n = _arr(KernelCudaMatvecJob, js)
    check(lib().kernel_cuda_matvec_quant_batch(arr, n), "kernel_cuda_matvec_quant_batch")


def matmul_quant_batch(jobs) -> None:
    """kernel_cuda_matmul_quant_batch over jobs given as KernelCudaMatmulJob or
    (is_q6, matrix, X, Y, rows, cols, T) with device tensors or addresses."""
    js = [j if isinstance(j, KernelCudaMatmulJob) else
          KernelCudaMatmulJob(int(bool(j[0])), _ptr(j[1]), _ptr(j[2]), _ptr(j[3]), int(j[4]), int(j[5]), int(j[6]))
          for j in jobs]
    arr, n = _arr(KernelCudaMatmulJob, js)
    check(lib().kernel_cuda_matmul_quant_batch(arr, n), "kernel_cuda_matmul_quant_batch")


class StepGroup:
    """Cross-slot batched step (``kernel_step_group_*``): the batched counterpart of the
    reference's per-token step lock (src/slots.c:77-105, 864-880). Each slot thread joins once,
    then per token calls begin(), its hot-path calls in model order, end(). The calls return the
    combined device batch's status (0 / -1); ``raise_on_error`` turns -1 into RuntimeError."""

    def __init__(self, max_members: int, straggler_us: int = 200, call_timeout_ms: int = 10000):
        self._h = lib().kernel_step_group_create(int(max_members), int(straggler_us), int(call_timeout_ms))
        if not self._h:
            raise RuntimeError(f"kernel_step_group_create failed: {last_error()}")

    def close(self) -> None:
        if self._h:
            lib().kernel_step_group_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def join(self) -> int:
        m = lib().kernel_step_group_join(self._h)
        if m < 0:
            raise RuntimeError(f"kernel_step_group_join failed: {last_error()}")
        return m

    def leave(self, member: int) -> int:
        return lib().kernel_step_group_leave(self._h, member)

    def begin(self, member: int) -> int:
        return lib().kernel_step_group_begin(self._h, member)

    def end(self, member: int) -> int:
        return lib().kernel_step_group_end(self._h, member)

    def attn(self, member: int, site: int, job: KernelAttnDecodeJob) -> int:
        return lib().kernel_step_group_attn(self._h, member, site, C.byref(job))

    def delta(self, member: int, site: int, job: KernelDeltaStepJob) -> int:
        return lib().kernel_step_group_delta(self._h, member, site, C.byref(job))

    def matvec(self, member: int, site: int, jobs) -> int:
        js = [j if isinstance(j, KernelCudaMatvecJob) else
              KernelCudaMatvecJob(int(bool(j[0])), _ptr(j[1]), _ptr(j[2]), _ptr(j[3]), int(j[4]), int(j[5]))
              for j in jobs]
        arr, n = _arr(KernelCudaMatvecJob, js)
        return lib().kernel_step_group_matvec(self._h, member, site, arr, n)

    def lock(self) -> None:
        check(lib().kernel_step_group_lock(self._h), "kernel_step_group_lock")

    def unlock(self) -> None:
        check(lib().kernel_step_group_unlock(self._h), "kernel_step_group_unlock")

    def stats(self) -> dict:
        st = KernelStepGroupStats()
        check(lib().kernel_step_group_stats(self._h, C.byref(st)), "kernel_step_group_stats")
        return {name: getattr(st, name) for name, _ in KernelStepGroupStats._fields_}
