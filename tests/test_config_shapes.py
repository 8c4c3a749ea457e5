"""Parity at the shapes bench.py times: the batched decode of config 2, the split-KV decode of
config 4 and the 30-layer, 1024-step DeltaNet decode of config 1, each against the CPU oracle
(the restatement of model.c:801-861 and model.c:272-323, pinned to the reference build by
tests/test_oracle.py).

Bars (maxrel = max|a-b| / max|ref|, src/test_kernels.c:31): 2e-3 on gated attention outputs,
1e-4 on the fp32 DeltaNet state and outputs.

The large KV windows are drawn on the device with torch's seeded generator (as bench.py draws
them) and copied to the host for the oracle; the small per-step vectors come from numpy.
"""
import numpy as np
import pytest
import torch

import oracle as O
from roaster_b200 import splitkv, synth
from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu
ATTN_TOL = 2e-3
STATE_TOL = 1e-4


def _vectors(rng):
    n = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    return {"q": n(16, 256), "gate": n(16, 256), "k_new": n(2, 256), "v_new": n(2, 256)}


def _window(L, cap, seed):
    kc = torch.zeros(cap, 2, 256, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    if L:
        kc[:L] = synth.device_normal(torch, (L, 2, 256), seed, "cuda", torch.float16)
        vc[:L] = synth.device_normal(torch, (L, 2, 256), seed + 1, "cuda", torch.float16)
    return kc, vc


def test_config2_batch_at_bench_shape(rb, oracle_lib):
    """bench.py's config-2 step: the 64 windows of rank 0 (synth.slot_lengths(1000, 64, 1024,
    32768), the same split plan the timed launch runs) in one kernel_attn_decode_batch call, plus
    3 DeltaNet layers per slot (192 states) in one kernel_deltanet_step_batch call. Every slot's
    gated output and appended row, and every state and output, against the oracle."""
    lens = [int(x) for x in synth.slot_lengths(1000, 64, 1024, 32768)]
    rng = np.random.default_rng(2002)
    qn = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    dqn, dkw = dev(qn), dev(kw)
    slots = []
    for s, L in enumerate(lens):
        v = _vectors(rng)
        kc, vc = _window(L, L + 1, 3000 + 2 * s)
        d = {k: dev(x) for k, x in v.items()}
        slots.append((v, d, kc, vc))
    out = torch.zeros(64, 16, 256, device="cuda")
    jobs = [rb.attn_job(d["q"], d["gate"], d["k_new"], d["v_new"], dqn, dkw, kc, vc, L, L, out[s])
            for s, ((v, d, kc, vc), L) in enumerate(zip(slots, lens))]
    st0 = (0.02 * rng.standard_normal((64 * 3, 32, 128, 128))).astype(np.float32)
    dn = synth.delta_step_inputs(rng, 64 * 3)
    ds = dev(st0)
    ddn = {k: dev(x) for k, x in dn.items()}
    dout = torch.zeros(64 * 3, 32, 128, device="cuda")
    djobs = [rb.delta_job(ds[i], ddn["q"][i], ddn["k"][i], ddn["v"][i], ddn["g"][i], ddn["beta"][i],
                          dout[i]) for i in range(64 * 3)]
    rb.attn_decode_batch(jobs)
    rb.deltanet_step_batch(djobs)
    rb.synchronize()
    got = host(out)
    assert np.isfinite(got).all()
    worst = 0.0
    for s, ((v, d, kc, vc), L) in enumerate(zip(slots, lens)):
        hk, hv = host(kc), host(vc)
        ref, ka, va = O.attn_decode(v["q"], v["gate"], v["k_new"], v["v_new"], qn, kw, hk[:L], hv[:L],
                                    L, L)
        e = O.maxrel(got[s], ref)
        worst = max(worst, e)
        assert e <= ATTN_TOL, (s, L, e)
        assert np.array_equal(hv[L], va.astype(np.float16))
        assert np.abs(hk[L].astype(np.float32) - ka).max() <= 2e-3 * max(1.0, np.abs(ka).max())
    gst, gout = host(ds), host(dout)
    for i in range(64 * 3):
        st = st0[i].copy()
        ref = O.delta_step(st, dn["q"][i], dn["k"][i], dn["v"][i], dn["g"][i], dn["beta"][i])
        assert O.maxrel(gst[i], st) <= STATE_TOL, i
        assert O.maxrel(gout[i], ref) <= STATE_TOL, i
    print(f"config 2: 64 slots, windows {min(lens)}..{max(lens)}, worst attention maxrel {worst:.2e}")


@pytest.mark.parametrize("slices", [2, 4, 8])
def test_config4_split_window_and_merge(rb, oracle_lib, slices):
    """Config 4's long-context step on one GPU: 2 slots of 262144 cached positions, each window
    cut into `slices` contiguous slices as on `slices` GPUs (roaster_b200.splitkv.slice_bounds;
    the newest slice appends), one kernel_attn_decode_partial_batch call per slice (the plan each
    rank would make), then kernel_attn_merge_partials. Against the oracle's decode over the whole
    window."""
    W, S = 262144, 2
    rng = np.random.default_rng(4004)
    qn = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    dqn, dkw = dev(qn), dev(kw)
    vs, ds, caches = [], [], []
    for s in range(S):
        v = _vectors(rng)
        vs.append(v)
        ds.append({k: dev(x) for k, x in v.items()})
        caches.append(_window(W, W + 1, 5000 + 2 * s))
    parts = torch.zeros(slices, S, 2, splitkv.PARTIAL_FLOATS, device="cuda")
    for r in range(slices):
        lo, hi = splitkv.slice_bounds(W, slices, r)
        app = splitkv.appends(slices, r)
        jobs = [rb.attn_job(d["q"], d["gate"], d["k_new"], d["v_new"], dqn, dkw,
                            kc.data_ptr() + lo * 1024, vc.data_ptr() + lo * 1024, hi - lo, W, 0,
                            append=app, capacity=hi - lo + (1 if app else 0))
                for d, (kc, vc) in zip(ds, caches)]
        rb.attn_decode_partial_batch(jobs, parts[r])
    out = torch.zeros(S, 16, 256, device="cuda")
    rb.attn_merge_partials(parts, slices, [d["gate"] for d in ds], [out[s] for s in range(S)])
    rb.synchronize()
    got = host(out)
    assert np.isfinite(got).all()
    for s in range(S):
        kc, vc = caches[s]
        hk, hv = host(kc), host(vc)
        v = vs[s]
        ref, ka, va = O.attn_decode(v["q"], v["gate"], v["k_new"], v["v_new"], qn, kw, hk[:W], hv[:W], W, W)
        e = O.maxrel(got[s], ref)
        assert e <= ATTN_TOL, (slices, s, e)
        assert np.array_equal(hv[W], va.astype(np.float16))
        del hk, hv


def test_config1_thirty_layers_1024_steps(rb, oracle_lib):
    """Config 1 as configured: 30 DeltaNet layers, 1024 sequential steps, one
    kernel_deltanet_step_batch call per step (30 jobs), fresh inputs every step; every layer's
    state after the last step and the last step's outputs within 1e-4 of the oracle."""
    L, T = 30, 1024
    st0 = synth.delta_state(41, L)
    rng = np.random.default_rng(42)
    ds = dev(st0)
    st = st0.copy()
    outs = torch.zeros(L, 32, 128, device="cuda")
    ref = np.zeros((L, 32, 128), np.float32)
    for t in range(T):
        inp = synth.delta_step_inputs(rng, L)
        di = {k: dev(x) for k, x in inp.items()}
        rb.deltanet_step_batch([rb.delta_job(ds[l], di["q"][l], di["k"][l], di["v"][l], di["g"][l],
                                             di["beta"][l], outs[l]) for l in range(L)])
        for l in range(L):
            ref[l] = O.delta_step(st[l], inp["q"][l], inp["k"][l], inp["v"][l], inp["g"][l], inp["beta"][l])
    rb.synchronize()
    gst, gout = host(ds), host(outs)
    errs = [O.maxrel(gst[l], st[l]) for l in range(L)]
    assert max(errs) <= STATE_TOL, (int(np.argmax(errs)), max(errs))
    assert O.maxrel(gout, ref) <= STATE_TOL
    print(f"config 1: 30 layers x 1024 steps, worst state maxrel {max(errs):.2e}")
