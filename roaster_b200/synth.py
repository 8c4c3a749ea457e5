"""Seeded synthetic inputs with the shapes and distributions of the benchmark configurations.

The reference has no dataset for this path; every input is drawn from numpy's PCG64
(``np.random.default_rng(seed)``) in the order documented per function, so tests, the golden
fixtures and the bench see identical values for the same seed. Large bench-only tensors (KV
windows of thousands of tokens for many slots) are drawn on the device with torch's seeded
generator instead (``device_normal``); they are checked through size-independent properties and
the small-case parity of the same kernels.
"""
from __future__ import annotations

import numpy as np


def _n(rng, *shape):
    return rng.standard_normal(shape).astype(np.float32)


def softplus(x):
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def attn_decode_inputs(seed: int = 0, length: int = 512, position: int | None = None):
    """Config 0: one gated-attention decode step for one slot.

    Draw order: q [16,256], gate [16,256], k_new [2,256], v_new [2,256] ~ N(0,1);
    q_norm, k_norm [256] ~ 1 + 0.1 N(0,1); K cache, V cache f16 [length,2,256] ~ N(0,1).
    RoPE position defaults to `length` (the new token's index in an unslid window)."""
    rng = np.random.default_rng(seed)
    d = {
        "q": _n(rng, 16, 256),
        "gate": _n(rng, 16, 256),
        "k_new": _n(rng, 2, 256),
        "v_new": _n(rng, 2, 256),
        "q_norm": (1.0 + 0.1 * _n(rng, 256)).astype(np.float32),
        "k_norm": (1.0 + 0.1 * _n(rng, 256)).astype(np.float32),
    }
    d["k_cache"] = _n(rng, length, 2, 256).astype(np.float16)
    d["v_cache"] = _n(rng, length, 2, 256).astype(np.float16)
    d["length"] = length
    d["position"] = length if position is None else position
    return d


def delta_state(seed: int, layers: int = 1):
    """Initial DeltaNet states [layers, 32, 128, 128] ~ N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    return (0.02 * rng.standard_normal((layers, 32, 128, 128))).astype(np.float32)


def delta_step_inputs(rng, layers: int = 1):
    """Config 1 per-step inputs for `layers` layers. Draw order per layer: q [16,128], k [16,128]
    (both L2-normalised per head), v [32,128] ~ N(0,1), beta = sigmoid(N(0,1)) [32],
    g = -exp(N(-1, 0.5)) * softplus(N(0,1)) [32]."""
    out = {k: [] for k in ("q", "k", "v", "beta", "g")}
    for _ in range(layers):
        q = _n(rng, 16, 128)
        k = _n(rng, 16, 128)
        q /= np.sqrt((q * q).sum(1, keepdims=True) + 1e-6)
        k /= np.sqrt((k * k).sum(1, keepdims=True) + 1e-6)
        v = _n(rng, 32, 128)
        beta = (1.0 / (1.0 + np.exp(-rng.standard_normal(32)))).astype(np.float32)
        g = (-np.exp(rng.normal(-1.0, 0.5, 32)) * softplus(rng.standard_normal(32))).astype(np.float32)
        for name, x in zip(("q", "k", "v", "beta", "g"), (q, k, v, beta, g)):
            out[name].append(x.astype(np.float32))
    return {k: np.stack(v) for k, v in out.items()}


def delta_sequence(seed: int, steps: int, layers: int = 1):
    """`steps` consecutive config-1 inputs: dict of arrays [steps, layers, ...]."""
    rng = np.random.default_rng(seed)
    per = [delta_step_inputs(rng, layers) for _ in range(steps)]
    return {k: np.stack([p[k] for p in per]) for k in per[0]}


def delta_prompt(seed: int, T: int):
    """One prompt of config-3 DeltaNet inputs (config-1 distributions), drawn vectorised:
    q, k [T,16,128] L2-normalised per head, v [T,32,128] ~ N(0,1), beta = sigmoid(N(0,1)) and
    g = -exp(N(-1, 0.5)) * softplus(N(0,1)), both [T,32]."""
    rng = np.random.default_rng(seed)
    q = _n(rng, T, 16, 128)
    k = _n(rng, T, 16, 128)
    q /= np.sqrt((q * q).sum(-1, keepdims=True) + 1e-6)
    k /= np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
    v = _n(rng, T, 32, 128)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((T, 32))))).astype(np.float32)
    g = (-np.exp(rng.normal(-1.0, 0.5, (T, 32))) * softplus(rng.standard_normal((T, 32)))).astype(np.float32)
    return {"q": q.astype(np.float32), "k": k.astype(np.float32), "v": v, "beta": beta, "g": g}


def delta_layer_inputs(seed: int, T: int):
    """Raw inputs of one recurrent layer (before its pre-ops) for T tokens: qkv [T,8192] and z
    [T,4096] ~ N(0,1); alpha, beta [T,32] ~ N(0,1); conv_w [8192,4] ~ 0.5 N(0,1); dt ~ N(0,1);
    a = -exp(N(-1, 0.5)) [32]; ssm_norm ~ 1 + 0.1 N(0,1) [128]; conv_state [3,8192] ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    return {
        "qkv": _n(rng, T, 8192), "z": _n(rng, T, 4096), "alpha": _n(rng, T, 32), "beta": _n(rng, T, 32),
        "conv_w": (0.5 * rng.standard_normal((8192, 4))).astype(np.float32),
        "dt": _n(rng, 32), "a": (-np.exp(rng.normal(-1.0, 0.5, 32))).astype(np.float32),
        "ssm_norm": (1.0 + 0.1 * rng.standard_normal(128)).astype(np.float32),
        "conv_state": _n(rng, 3, 8192),
    }


def quant_matrix(seed: int, rows: int, cols: int, is_q6: bool):
    """Random k-quant weights (uint8 blocks) with realistic scale ranges: Q4_K d, dmin ~ U[1e-3,
    1e-2] as f16 and random 6-bit scales/mins and nibbles; Q6_K d ~ U[1e-3, 1e-2], int8 scales
    in [-64, 63], random 6-bit values. Shape [rows * cols/256 * (210 | 144)]."""
    rng = np.random.default_rng(seed)
    nb = rows * (cols // 256)
    if not is_q6:
        blk = rng.integers(0, 256, (nb, 144), dtype=np.uint8)
        d = rng.uniform(1e-3, 1e-2, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
        m = rng.uniform(1e-3, 1e-2, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
        blk[:, 0:2] = d
        blk[:, 2:4] = m
    else:
        blk = rng.integers(0, 256, (nb, 210), dtype=np.uint8)
        blk[:, 192:208] = rng.integers(-64, 64, (nb, 16)).astype(np.int8).view(np.uint8)
        blk[:, 208:210] = rng.uniform(1e-3, 1e-2, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return blk.reshape(-1)


def slot_lengths(seed: int, slots: int, lo: int = 1024, hi: int = 32768):
    """Config 2: per-slot context lengths ~ U[lo, hi] (integers, inclusive)."""
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=slots).astype(np.int64)


def prefill_inputs(seed: int, T: int, kbase: int = 0):
    """Config 3 shapes for one prompt (small T for parity): q, gate [T,16,256], k, v [T,2,256]
    ~ N(0,1) rounded to bf16 (the configuration's input type), norms ~ 1 + 0.1 N(0,1), and an
    f16 window of `kbase` earlier tokens."""
    rng = np.random.default_rng(seed)

    def bf16(x):
        u = np.ascontiguousarray(x, np.float32).view(np.uint32).copy()
        u += 0x7FFF + ((u >> 16) & 1)
        u &= 0xFFFF0000
        return u.view(np.float32)

    d = {
        "q": bf16(_n(rng, T, 16, 256)),
        "gate": bf16(_n(rng, T, 16, 256)),
        "k": bf16(_n(rng, T, 2, 256)),
        "v": bf16(_n(rng, T, 2, 256)),
        "q_norm": (1.0 + 0.1 * _n(rng, 256)).astype(np.float32),
        "k_norm": (1.0 + 0.1 * _n(rng, 256)).astype(np.float32),
    }
    d["k_cache"] = _n(rng, max(kbase, 1), 2, 256).astype(np.float16)[:kbase]
    d["v_cache"] = _n(rng, max(kbase, 1), 2, 256).astype(np.float16)[:kbase]
    return d


def device_normal(torch, shape, seed: int, device, dtype, std: float = 1.0):
    """N(0, std) drawn on the device with a seeded torch generator (bench-size tensors)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = torch.empty(shape, device=device, dtype=dtype)
    # chunked so the fp32 temporary never exceeds ~1 GiB
    fo = out.view(-1)
    step = 1 << 28
    for i in range(0, fo.numel(), step):
        n = min(step, fo.numel() - i)
        tmp = torch.randn(n, generator=g, device=device, dtype=torch.float32)
        fo[i:i + n] = (tmp * std).to(dtype)
    return out
