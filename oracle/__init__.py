"""CPU oracle for the hybrid-attention hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, bench.py's CPU-baseline leg and __graft_entry__.smoke() import this package; it is
the checker, never the thing measured as the product or shipped with it. Two implementations sit
behind the same numpy-level functions:

* ``impl="port"``: the plain-C restatement in ``roaster_oracle.c`` (liboracle.so), each function
  citing the reference lines it follows;
* ``impl="ref"``: the reference's own CPU code (KKB007X/Roaster ``src/model.c`` +
  ``src/kernels.c`` lines 1-721) compiled from its sources into ``_ref/libroaster_ref.so`` by
  ``oracle/Makefile`` (see ``ref_harness.c`` for how its static functions are driven).

Shapes (fp32 unless stated): q/gate ``[16, 256]`` (or interleaved ``[16, 512]``), k/v new
``[2, 256]``, KV cache f16 ``[L, 2, 256]``, DeltaNet state ``[32, 128, 128]``.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_PORT = os.path.join(HERE, "liboracle.so")
_REF = os.path.join(HERE, "_ref", "libroaster_ref.so")
_REF_NATIVE = os.path.join(HERE, "_ref", "libroaster_ref_native.so")

_fp = C.POINTER(C.c_float)
_u16p = C.POINTER(C.c_uint16)
_libs: dict = {}


# Where the reference checkout lives (its src/ holds model.c): by default a directory named
# `reference` beside this repository's root; ROASTER_REFERENCE overrides.
REFERENCE_ROOT = os.environ.get("ROASTER_REFERENCE",
                                os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))
# CPU architecture of the GPU host (what -march=native selects there), for the reference build
# with the reference's own flags; ROASTER_REF_MARCH overrides.
REF_MARCH = os.environ.get("ROASTER_REF_MARCH", "sapphirerapids")


def build(quiet: bool = True) -> None:
    """Compile liboracle.so and, when the reference sources are present, _ref (make)."""
    cmd = ["make", "-C", HERE]
    src = os.path.join(REFERENCE_ROOT, "src")
    if os.path.exists(os.path.join(src, "model.c")):
        cmd += [f"REF={src}", f"REF_MARCH={REF_MARCH}"]
    out = subprocess.run(cmd, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def have_ref() -> bool:
    return os.path.exists(_REF)


def native_ref_available() -> bool:
    """Whether the reference build with -march=<GPU host CPU> exists (see REF_MARCH)."""
    return os.path.exists(_REF_NATIVE)


def native_ref_march() -> str | None:
    try:
        with open(os.path.join(HERE, "_ref", "native_march.txt")) as f:
            return f.read().strip()
    except OSError:
        return None


def _load(which: str):
    if which in _libs:
        return _libs[which]
    # ROASTER_REF_NATIVE=1 selects the -march build of the reference (timed CPU baseline only)
    native = which == "ref" and os.environ.get("ROASTER_REF_NATIVE") == "1" and native_ref_available()
    path = _PORT if which == "port" else (_REF_NATIVE if native else _REF)
    if not os.path.exists(path):
        raise FileNotFoundError(f"oracle library missing: {path} (run make -C oracle)")
    lib = C.CDLL(path)
    if which == "port":
        lib.orc_attn_prefill.argtypes = [C.c_size_t, _fp, _fp, C.c_size_t, C.c_size_t, _fp, _fp,
                                         _fp, _fp, _u16p, _u16p, C.c_size_t, C.c_size_t,
                                         _fp, _fp, _fp]
        lib.orc_attn_prefill.restype = C.c_int
        lib.orc_attn_decode_partial.argtypes = [_fp, C.c_size_t, _fp, _u16p, _u16p, C.c_size_t,
                                                C.c_size_t, C.c_size_t, _fp, _fp, _fp]
        lib.orc_attn_decode_partial.restype = C.c_int
        lib.orc_attn_prefill_rows.argtypes = [C.c_size_t, _fp, _fp, C.c_size_t, C.c_size_t, _fp,
                                              _fp, _fp, _fp, _u16p, _u16p, C.c_size_t, C.c_size_t,
                                              C.POINTER(C.c_long), C.c_size_t, _fp]
        lib.orc_attn_prefill_rows.restype = C.c_int
        lib.orc_delta_step.argtypes = [_fp] * 7
        lib.orc_delta_step.restype = None
        lib.orc_delta_prefill.argtypes = [_fp, C.c_size_t] + [_fp] * 6
        lib.orc_delta_prefill.restype = None
        lib.orc_delta_preop.argtypes = [C.c_size_t] + [_fp] * 12
        lib.orc_delta_preop.restype = None
        lib.orc_delta_postop.argtypes = [C.c_size_t, _fp, _fp, _fp]
        lib.orc_matvec_q.argtypes = [C.c_int, C.c_void_p, _fp, _fp, C.c_size_t, C.c_size_t]
        lib.orc_matvec_q.restype = None
        lib.orc_delta_postop.restype = None
        lib.orc_f32_to_f16.argtypes = [C.c_float]
        lib.orc_f32_to_f16.restype = C.c_uint16
    else:
        lib.ref_attn_decode.argtypes = [_fp] * 7 + [C.c_size_t, C.c_size_t, _fp, _fp, _fp]
        lib.ref_attn_decode.restype = C.c_int
        lib.ref_attn_prefill.argtypes = [C.c_int] + [_fp] * 7 + [C.c_size_t, C.c_size_t,
                                                                   _fp, _fp, _fp]
        lib.ref_attn_prefill.restype = C.c_int
        lib.ref_delta_step.argtypes = [_fp] * 7
        lib.ref_delta_step.restype = None
        lib.ref_delta_prefill.argtypes = [_fp, C.c_int] + [_fp] * 6
        lib.ref_delta_prefill.restype = None
        lib.ref_delta_layer_prefill.argtypes = [C.c_int] + [_fp] * 11
        lib.ref_delta_layer_prefill.restype = C.c_int
        lib.ref_matvec_q.argtypes = [C.c_int, C.c_void_p, _fp, _fp, C.c_size_t, C.c_size_t]
        lib.ref_matvec_q.restype = None
        lib.ref_matmul_q.argtypes = [C.c_int, C.c_void_p, _fp, _fp, C.c_size_t, C.c_size_t, C.c_size_t]
        lib.ref_matmul_q.restype = None
        lib.ref_kvw_new.argtypes = [C.c_size_t, C.c_int, C.c_size_t, C.c_size_t, C.c_char_p]
        lib.ref_kvw_new.restype = C.c_void_p
        lib.ref_kvw_free.argtypes = [C.c_void_p]
        lib.ref_kvw_free.restype = None
        lib.ref_kvw_layers.argtypes = [C.c_void_p]
        lib.ref_kvw_layers.restype = C.c_int
        lib.ref_kvw_append.argtypes = [C.c_void_p, C.c_size_t, _fp, _fp]
        lib.ref_kvw_append.restype = C.c_int
        for nm in ("evict", "restore", "set_context"):
            getattr(lib, "ref_kvw_" + nm).argtypes = [C.c_void_p, C.c_size_t]
            getattr(lib, "ref_kvw_" + nm).restype = C.c_int
        lib.ref_kvw_rollback.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t]
        lib.ref_kvw_rollback.restype = C.c_int
        for nm in ("len", "spilled", "head", "max_chunk", "position", "context"):
            getattr(lib, "ref_kvw_" + nm).argtypes = [C.c_void_p]
            getattr(lib, "ref_kvw_" + nm).restype = C.c_size_t
        lib.ref_kvw_read.argtypes = [C.c_void_p, C.c_int, _fp, _fp]
        lib.ref_kvw_read.restype = None
        lib.ref_decode_ctx_new.argtypes = [C.c_size_t, _fp, _fp]
        lib.ref_decode_ctx_new.restype = C.c_void_p
        lib.ref_decode_ctx_k.argtypes = [C.c_void_p]
        lib.ref_decode_ctx_k.restype = _fp
        lib.ref_decode_ctx_v.argtypes = [C.c_void_p]
        lib.ref_decode_ctx_v.restype = _fp
        lib.ref_decode_ctx_step.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t]
        lib.ref_decode_ctx_step.restype = C.c_int
        lib.ref_decode_ctx_projections.argtypes = [C.c_void_p]
        lib.ref_decode_ctx_projections.restype = None
        lib.ref_decode_ctx_free.argtypes = [C.c_void_p]
        lib.ref_decode_ctx_free.restype = None
        lib.ref_prefill_ctx_new.argtypes = [C.c_size_t, _fp, _fp]
        lib.ref_prefill_ctx_new.restype = C.c_void_p
        lib.ref_prefill_ctx_k.argtypes = [C.c_void_p]
        lib.ref_prefill_ctx_k.restype = _fp
        lib.ref_prefill_ctx_v.argtypes = [C.c_void_p]
        lib.ref_prefill_ctx_v.restype = _fp
        lib.ref_prefill_ctx_chunk.argtypes = [C.c_void_p, C.c_int, C.c_size_t, C.c_size_t]
        lib.ref_prefill_ctx_chunk.restype = C.c_int
        lib.ref_prefill_ctx_projections.argtypes = [C.c_void_p, C.c_int]
        lib.ref_prefill_ctx_projections.restype = C.c_int
        lib.ref_prefill_ctx_free.argtypes = [C.c_void_p]
        lib.ref_prefill_ctx_free.restype = None
        lib.ref_state_new.argtypes = [C.c_size_t]
        lib.ref_state_new.restype = C.c_void_p
        lib.ref_state_free.argtypes = [C.c_void_p]
        lib.ref_state_free.restype = None
        for nm in ("k", "v", "ssm", "conv"):
            getattr(lib, "ref_state_" + nm).argtypes = [C.c_void_p, C.c_int]
            getattr(lib, "ref_state_" + nm).restype = _fp
        lib.ref_state_is_attention.argtypes = [C.c_int]
        lib.ref_state_is_attention.restype = C.c_int
        lib.ref_state_layers.argtypes = []
        lib.ref_state_layers.restype = C.c_int
        lib.ref_state_set_len.argtypes = [C.c_void_p, C.c_size_t]
        lib.ref_state_set_len.restype = None
        lib.ref_state_len.argtypes = [C.c_void_p, C.c_int]
        lib.ref_state_len.restype = C.c_size_t
        lib.ref_state_position.argtypes = [C.c_void_p]
        lib.ref_state_position.restype = C.c_size_t
        for nm in ("save", "load"):
            getattr(lib, "ref_state_" + nm).argtypes = [C.c_void_p, C.c_char_p]
            getattr(lib, "ref_state_" + nm).restype = C.c_int
        lib.ref_max_threads.argtypes = []
        lib.ref_max_threads.restype = C.c_int
    _libs[which] = lib
    return lib


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous, (a.dtype, a.flags)
    return a.ctypes.data_as(_fp)


def _h(a: np.ndarray):
    assert a.dtype == np.float16 and a.flags.c_contiguous
    return a.ctypes.data_as(_u16p)


def maxrel(a, b) -> float:
    """max|a-b| / max|ref| -- the reference's test metric (src/test_kernels.c:31)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    ref = float(np.abs(b).max()) if b.size else 0.0
    return float(np.abs(a - b).max()) / (ref if ref > 0 else 1.0)


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> f16 (numpy's conversion is RNE as well)."""
    return np.asarray(x, np.float32).astype(np.float16)


# ----------------------------------------------------------------------------- attention

def attn_decode(q, gate, k_new, v_new, qnorm, knorm, k_cache, v_cache, length, position,
                impl: str = "port"):
    """One gated-attention decode step for one slot.

    q, gate: [16, 256]; k_new, v_new: [2, 256]; k_cache, v_cache: f16 [>=length, 2, 256].
    Returns (out [16, 256], k_appended [2, 256], v_appended [2, 256]) in fp32."""
    q = np.ascontiguousarray(q, np.float32)
    gate = np.ascontiguousarray(gate, np.float32)
    k_new = np.ascontiguousarray(k_new, np.float32)
    v_new = np.ascontiguousarray(v_new, np.float32)
    qnorm = np.ascontiguousarray(qnorm, np.float32)
    knorm = np.ascontiguousarray(knorm, np.float32)
    kc = np.ascontiguousarray(k_cache[:length], np.float16)
    vc = np.ascontiguousarray(v_cache[:length], np.float16)
    out = np.zeros((16, 256), np.float32)
    ka = np.zeros((2, 256), np.float32)
    va = np.zeros((2, 256), np.float32)
    if impl == "port":
        lib = _load("port")
        kcp = kc if length else np.zeros((1, 2, 256), np.float16)
        vcp = vc if length else np.zeros((1, 2, 256), np.float16)
        rc = lib.orc_attn_prefill(1, _f(q), _f(gate), 256, 0, _f(k_new), _f(v_new), _f(qnorm),
                                  _f(knorm), _h(kcp), _h(vcp), length, position, _f(out),
                                  _f(ka), _f(va))
    else:
        lib = _load("ref")
        qg = np.ascontiguousarray(np.concatenate([q, gate], axis=1), np.float32)
        kcf = np.ascontiguousarray(kc.astype(np.float32)) if length else np.zeros(512, np.float32)
        vcf = np.ascontiguousarray(vc.astype(np.float32)) if length else np.zeros(512, np.float32)
        rc = lib.ref_attn_decode(_f(qg), _f(k_new), _f(v_new), _f(qnorm), _f(knorm), _f(kcf),
                                 _f(vcf), length, position, _f(out), _f(ka), _f(va))
    if rc != 0:
        raise RuntimeError(f"oracle attn_decode ({impl}) failed")
    return out, ka, va


def attn_decode_partial(q, qnorm, k_cache, v_cache, t0, t1, position):
    """Softmax partial (m [16], l [16], o [16, 256]) over cached tokens [t0, t1) (port only)."""
    lib = _load("port")
    q = np.ascontiguousarray(q, np.float32)
    qnorm = np.ascontiguousarray(qnorm, np.float32)
    kc = np.ascontiguousarray(k_cache, np.float16)
    vc = np.ascontiguousarray(v_cache, np.float16)
    m = np.zeros(16, np.float32)
    l = np.zeros(16, np.float32)
    o = np.zeros((16, 256), np.float32)
    if lib.orc_attn_decode_partial(_f(q), 256, _f(qnorm), _h(kc), _h(vc), t0, t1, position,
                                   _f(m), _f(l), _f(o)) != 0:
        raise RuntimeError("oracle attn_decode_partial failed")
    return m, l, o


def attn_prefill(q, gate, k, v, qnorm, knorm, k_cache, v_cache, kbase, base, impl: str = "port"):
    """Causal prefill of T tokens. q, gate: [T, 16, 256]; k, v: [T, 2, 256];
    k_cache, v_cache: f16 [>=kbase, 2, 256]. Returns (out [T,16,256], k_app, v_app [T,2,256]).
    impl="ref" goes through the reference's pf_attention, 256 tokens per call (PF_MAX_T)."""
    q = np.ascontiguousarray(q, np.float32)
    gate = np.ascontiguousarray(gate, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    qnorm = np.ascontiguousarray(qnorm, np.float32)
    knorm = np.ascontiguousarray(knorm, np.float32)
    T = q.shape[0]
    out = np.zeros((T, 16, 256), np.float32)
    ka = np.zeros((T, 2, 256), np.float32)
    va = np.zeros((T, 2, 256), np.float32)
    if impl == "port":
        lib = _load("port")
        kc = np.ascontiguousarray(k_cache[:kbase] if kbase else np.zeros((1, 2, 256)), np.float16)
        vc = np.ascontiguousarray(v_cache[:kbase] if kbase else np.zeros((1, 2, 256)), np.float16)
        rc = lib.orc_attn_prefill(T, _f(q), _f(gate), 256, 16 * 256, _f(k), _f(v), _f(qnorm),
                                  _f(knorm), _h(kc), _h(vc), kbase, base, _f(out), _f(ka), _f(va))
        if rc != 0:
            raise RuntimeError("oracle attn_prefill (port) failed")
        return out, ka, va
    lib = _load("ref")
    # The reference window is fp32: earlier chunks' appends stay unrounded, as in model.c.
    win_k = np.zeros((kbase + T, 2, 256), np.float32)
    win_v = np.zeros((kbase + T, 2, 256), np.float32)
    if kbase:
        win_k[:kbase] = np.asarray(k_cache[:kbase], np.float16).astype(np.float32)
        win_v[:kbase] = np.asarray(v_cache[:kbase], np.float16).astype(np.float32)
    qg = np.ascontiguousarray(np.concatenate([q, gate], axis=2), np.float32)  # [T,16,512]
    t0 = 0
    while t0 < T:
        n = min(256, T - t0)
        cur = kbase + t0
        kcf = np.ascontiguousarray(win_k[:cur]) if cur else np.zeros(512, np.float32)
        vcf = np.ascontiguousarray(win_v[:cur]) if cur else np.zeros(512, np.float32)
        o = np.zeros((n, 16, 256), np.float32)
        kk = np.zeros((n, 2, 256), np.float32)
        vv = np.zeros((n, 2, 256), np.float32)
        rc = lib.ref_attn_prefill(n, _f(np.ascontiguousarray(qg[t0:t0 + n])),
                                  _f(np.ascontiguousarray(k[t0:t0 + n])),
                                  _f(np.ascontiguousarray(v[t0:t0 + n])), _f(qnorm), _f(knorm),
                                  _f(kcf), _f(vcf), cur, base + t0, _f(o), _f(kk), _f(vv))
        if rc != 0:
            raise RuntimeError("oracle attn_prefill (ref) failed")
        out[t0:t0 + n] = o
        ka[t0:t0 + n] = kk
        va[t0:t0 + n] = vv
        win_k[cur:cur + n] = kk
        win_v[cur:cur + n] = vv
        t0 += n
    return out, ka, va


def attn_prefill_rows(q, gate, k, v, qnorm, knorm, k_cache, v_cache, kbase, base, rows):
    """Prefill outputs for the listed token indices only (port). Returns [len(rows), 16, 256]."""
    lib = _load("port")
    q = np.ascontiguousarray(q, np.float32)
    gate = np.ascontiguousarray(gate, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    qnorm = np.ascontiguousarray(qnorm, np.float32)
    knorm = np.ascontiguousarray(knorm, np.float32)
    T = q.shape[0]
    r = np.ascontiguousarray(rows, np.int64)
    kc = np.ascontiguousarray(k_cache[:kbase] if kbase else np.zeros((1, 2, 256)), np.float16)
    vc = np.ascontiguousarray(v_cache[:kbase] if kbase else np.zeros((1, 2, 256)), np.float16)
    out = np.zeros((len(r), 16, 256), np.float32)
    rc = lib.orc_attn_prefill_rows(T, _f(q), _f(gate), 256, 16 * 256, _f(k), _f(v), _f(qnorm),
                                   _f(knorm), _h(kc), _h(vc), kbase, base,
                                   r.ctypes.data_as(C.POINTER(C.c_long)), len(r), _f(out))
    if rc != 0:
        raise RuntimeError("oracle attn_prefill_rows failed")
    return out


# ----------------------------------------------------------------------------- DeltaNet

def delta_step(state, q, k, v, g, beta, impl: str = "port"):
    """One DeltaNet decode step; `state` [32,128,128] fp32 is updated IN PLACE.
    q, k: [16,128]; v: [32,128]; g, beta: [32]. Returns out [32,128]."""
    assert state.dtype == np.float32 and state.flags.c_contiguous
    args = [np.ascontiguousarray(x, np.float32) for x in (q, k, v, g, beta)]
    out = np.zeros((32, 128), np.float32)
    fn = _load("port").orc_delta_step if impl == "port" else _load("ref").ref_delta_step
    fn(_f(state), *[_f(a) for a in args], _f(out))
    return out


def delta_prefill(state, q, k, v, g, beta, impl: str = "port"):
    """T sequential DeltaNet steps; `state` updated IN PLACE. q,k: [T,16,128]; v: [T,32,128];
    g, beta: [T,32]. Returns out [T,32,128]."""
    assert state.dtype == np.float32 and state.flags.c_contiguous
    args = [np.ascontiguousarray(x, np.float32) for x in (q, k, v, g, beta)]
    T = args[0].shape[0]
    out = np.zeros((T, 32, 128), np.float32)
    if impl == "port":
        _load("port").orc_delta_prefill(_f(state), T, *[_f(a) for a in args], _f(out))
    else:
        _load("ref").ref_delta_prefill(_f(state), T, *[_f(a) for a in args], _f(out))
    return out


def delta_preop(qkv, alpha, beta, conv_state, conv_w, dt, a):
    """Pre-ops of one recurrent layer over T tokens (model.c:1293-1328 per token).
    qkv [T,8192], alpha/beta [T,32]; conv_state [3,8192] fp32 is updated IN PLACE; conv_w
    [8192,4]; dt, a [32]. Returns dict q, k [T,16,128], v [T,32,128], g, beta [T,32]."""
    assert conv_state.dtype == np.float32 and conv_state.flags.c_contiguous
    qkv, alpha, beta, conv_w, dt, a = [np.ascontiguousarray(x, np.float32)
                                       for x in (qkv, alpha, beta, conv_w, dt, a)]
    T = qkv.shape[0]
    o = {"q": np.zeros((T, 16, 128), np.float32), "k": np.zeros((T, 16, 128), np.float32),
         "v": np.zeros((T, 32, 128), np.float32), "g": np.zeros((T, 32), np.float32),
         "beta": np.zeros((T, 32), np.float32)}
    _load("port").orc_delta_preop(T, _f(qkv), _f(alpha), _f(beta), _f(conv_state), _f(conv_w),
                                  _f(dt), _f(a), _f(o["q"]), _f(o["k"]), _f(o["v"]), _f(o["g"]),
                                  _f(o["beta"]))
    return o


def delta_postop(out, z, w):
    """Gated RMSNorm (model.c:1333-1343) of rows of 128: returns a new array."""
    x = np.ascontiguousarray(out, np.float32).copy()
    z = np.ascontiguousarray(z, np.float32)
    _load("port").orc_delta_postop(x.size // 128, _f(x), _f(z), _f(np.ascontiguousarray(w, np.float32)))
    return x


def delta_layer(state, conv_state, qkv, z, alpha, beta, conv_w, dt, a, ssm_norm, impl: str = "port"):
    """One recurrent layer over T tokens: pre-ops, the delta rule, gated RMSNorm -- pf_ssm
    (model.c:1604-1660) without its projections. state [32,128,128] and conv_state [3,8192]
    are updated IN PLACE. Returns out [T,32,128]. impl="ref" drives the reference's pf_ssm
    itself (T <= 256)."""
    qkv = np.ascontiguousarray(qkv, np.float32)
    T = qkv.shape[0]
    if impl == "port":
        p = delta_preop(qkv, alpha, beta, conv_state, conv_w, dt, a)
        out = delta_prefill(state, p["q"], p["k"], p["v"], p["g"], p["beta"])
        return delta_postop(out, z, ssm_norm).reshape(T, 32, 128)
    out = np.zeros((T, 32, 128), np.float32)
    args = [np.ascontiguousarray(x, np.float32) for x in (z, alpha, beta, conv_w, dt, a, ssm_norm)]
    rc = _load("ref").ref_delta_layer_prefill(T, _f(qkv), *[_f(x) for x in args], _f(state),
                                              _f(conv_state), _f(out))
    assert rc == 0, "ref_delta_layer_prefill failed"
    return out


class RefWindow:
    """The reference's own attention window (kvwindow.c + kvspill.c, compiled into oracle/_ref)
    over a rig holding the 10 attention layers' fp32 KV; appends follow forward_impl
    (kvw_ensure_room first). For checking the device window."""

    def __init__(self, ctx: int, slide: bool, keep: int, pin: int, spill_path: str):
        self.lib = _load("ref")
        self.h = self.lib.ref_kvw_new(ctx, int(slide), keep, pin, spill_path.encode())
        assert self.h, "ref_kvw_new failed"
        self.layers = self.lib.ref_kvw_layers(self.h)

    def append(self, k, v) -> int:
        """k, v: [layers, n, 512]."""
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        return self.lib.ref_kvw_append(self.h, k.shape[1], _f(k), _f(v))

    def evict(self, n) -> int:
        return self.lib.ref_kvw_evict(self.h, n)

    def restore(self, n) -> int:
        return self.lib.ref_kvw_restore(self.h, n)

    def rollback(self, p0, s0) -> int:
        return self.lib.ref_kvw_rollback(self.h, p0, s0)

    def set_context(self, ctx) -> int:
        return self.lib.ref_kvw_set_context(self.h, ctx)

    def state(self) -> dict:
        return {k: int(getattr(self.lib, "ref_kvw_" + k)(self.h))
                for k in ("len", "spilled", "head", "max_chunk", "position", "context")}

    def read(self, a):
        n = self.lib.ref_kvw_len(self.h)
        k = np.zeros((n, 512), np.float32)
        v = np.zeros((n, 512), np.float32)
        self.lib.ref_kvw_read(self.h, a, _f(k), _f(v))
        return k, v

    def close(self):
        if self.h:
            self.lib.ref_kvw_free(self.h)
            self.h = None


def matvec_q(is_q6: bool, m, x, rows: int, cols: int, impl: str = "port"):
    """k-quant projection (matvec_q4_cpu / matvec_q6_cpu, kernels.c:405-431, 553-578): uint8
    blocks ``m`` (rows x cols/256 Q4_K or Q6_K blocks) times fp32 ``x`` [cols] -> [rows]."""
    m = np.ascontiguousarray(m, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    assert m.size == rows * (cols // 256) * (210 if is_q6 else 144) and x.size == cols
    out = np.zeros(rows, np.float32)
    fn = _load("port").orc_matvec_q if impl == "port" else _load("ref").ref_matvec_q
    fn(int(bool(is_q6)), m.ctypes.data_as(C.c_void_p), _f(x), _f(out), rows, cols)
    return out


def matmul_q(is_q6: bool, m, X, rows: int, cols: int, impl: str = "port"):
    """Multi-token k-quant projection Y[t] = W X[t] for X [T][cols] -> [T][rows]. impl "ref" runs the
    reference's CPU prefill matmul itself (matmul_quant_cpu, kernels.c:1877-1913: each block
    dequantised to fp32 once per 32-row tile, then dotted with every token); "port" runs the
    oracle's per-row restatement once per token."""
    m = np.ascontiguousarray(m, np.uint8)
    X = np.ascontiguousarray(X, np.float32)
    T = X.shape[0]
    assert m.size == rows * (cols // 256) * (210 if is_q6 else 144) and X.shape == (T, cols)
    if impl == "port":
        return np.stack([matvec_q(is_q6, m, X[t], rows, cols) for t in range(T)])
    Y = np.zeros((T, rows), np.float32)
    _load("ref").ref_matmul_q(int(bool(is_q6)), m.ctypes.data_as(C.c_void_p), _f(X), _f(Y), rows, cols, T)
    return Y


class RefState:
    """The reference's state file (state.c, "RSTA" v2) through its own model_state_save /
    model_state_load on a Model rig of host fp32 windows (`ctx` rows) and DeltaNet states."""

    def __init__(self, ctx: int):
        self.lib = _load("ref")
        self.ctx = ctx
        self.h = self.lib.ref_state_new(ctx)
        if not self.h:
            raise MemoryError("ref_state_new")
        self.layers = self.lib.ref_state_layers()

    def is_attention(self, layer: int) -> bool:
        return bool(self.lib.ref_state_is_attention(layer))

    def kv(self, layer: int):
        """(K, V) views [ctx][512] of an attention layer's window."""
        n = self.ctx * 512
        return (np.ctypeslib.as_array(self.lib.ref_state_k(self.h, layer), shape=(n,)).reshape(self.ctx, 512),
                np.ctypeslib.as_array(self.lib.ref_state_v(self.h, layer), shape=(n,)).reshape(self.ctx, 512))

    def ssm(self, layer: int):
        """(state [32][128][128], conv history [3][8192]) views of a recurrent layer."""
        return (np.ctypeslib.as_array(self.lib.ref_state_ssm(self.h, layer), shape=(32 * 128 * 128,)).reshape(32, 128, 128),
                np.ctypeslib.as_array(self.lib.ref_state_conv(self.h, layer), shape=(3 * 8192,)).reshape(3, 8192))

    def set_len(self, n: int) -> None:
        self.lib.ref_state_set_len(self.h, n)

    def length(self, layer: int) -> int:
        return self.lib.ref_state_len(self.h, layer)

    def position(self) -> int:
        return self.lib.ref_state_position(self.h)

    def save(self, path: str) -> int:
        return self.lib.ref_state_save(self.h, path.encode())

    def load(self, path: str) -> int:
        return self.lib.ref_state_load(self.h, path.encode())

    def close(self) -> None:
        if self.h:
            self.lib.ref_state_free(self.h)
            self.h = None


def ref_lib():
    """The reference build's ctypes handle (for the timed CPU baseline)."""
    return _load("ref")
