"""Causal gated prefill attention (tcgen05/TMEM kernel) vs the CPU oracle (restating
model.c:1536-1602) and the reference-produced golden vectors. Tolerance: maxrel <= 2e-3 on the
gated outputs (f16 tensor-core operands, fp32 accumulation)."""
import os

import numpy as np
import pytest
import torch

import oracle as O
from roaster_b200 import synth
from tests.golden import make_golden as G
from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu
TOL = 2e-3
BF16 = 1


def run_prefill(rb, cases, dtype=0):
    """cases: list of (inputs dict, kbase, base). Runs one batch; returns (outs, kcaches, vcaches)."""
    jobs, keep = [], []
    for d, kbase, base in cases:
        T = d["q"].shape[0]
        cap = kbase + T + 3
        kc = torch.zeros(cap, 2, 256, dtype=torch.float16, device="cuda")
        vc = torch.zeros_like(kc)
        if kbase:
            kc[:kbase] = dev(d["k_cache"][:kbase])
            vc[:kbase] = dev(d["v_cache"][:kbase])
        tdt = torch.bfloat16 if dtype == BF16 else torch.float32
        q, g = dev(d["q"], tdt), dev(d["gate"], tdt)
        k, v = dev(d["k"], tdt), dev(d["v"], tdt)
        qn, kn = dev(d["q_norm"]), dev(d["k_norm"])
        out = torch.full((T, 16, 256), float("nan"), device="cuda")
        keep.append((q, g, k, v, qn, kn, kc, vc, out))
        jobs.append((q.data_ptr(), g.data_ptr(), 256, 4096, k.data_ptr(), v.data_ptr(), qn.data_ptr(),
                     kn.data_ptr(), kc.data_ptr(), vc.data_ptr(), cap, kbase, base, T, out.data_ptr(),
                     dtype))
    rb.attn_prefill_batch(jobs)
    rb.synchronize()
    return [host(x[8]) for x in keep], [host(x[6]) for x in keep], [host(x[7]) for x in keep]


def oracle_of(d, kbase, base):
    return O.attn_prefill(d["q"], d["gate"], d["k"], d["v"], d["q_norm"], d["k_norm"],
                          d["k_cache"], d["v_cache"], kbase, base)


def check(out, kc, vc, d, kbase, base):
    ref, ka, va = oracle_of(d, kbase, base)
    assert np.isfinite(out).all()
    err = O.maxrel(out, ref)
    assert err <= TOL, err
    T = d["q"].shape[0]
    kapp = kc[kbase:kbase + T].astype(np.float32)
    assert np.abs(kapp - ka).max() <= 2e-3 * max(1.0, np.abs(ka).max())
    assert np.array_equal(vc[kbase:kbase + T], va.astype(np.float16))
    if kbase:
        assert np.array_equal(kc[:kbase], d["k_cache"][:kbase])


def test_golden_reference_t12(rb):
    """GPU output against the vectors the reference's own pf_attention produced."""
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "attn_prefill_t12.npz"))
    d, dg = G.prefill_case()
    assert dg == str(g["digest"])
    outs, kcs, vcs = run_prefill(rb, [(d, 50, 300)])
    assert O.maxrel(outs[0], g["out"]) <= TOL
    assert np.abs(kcs[0][50:62].astype(np.float32) - g["k_app"]).max() <= 2e-3 * np.abs(g["k_app"]).max()


@pytest.mark.parametrize("T,kbase,base", [(1, 0, 0), (40, 100, 700), (128, 0, 0), (130, 0, 5),
                                          (257, 63, 63), (600, 0, 1000)])
def test_shapes(rb, T, kbase, base):
    d = synth.prefill_inputs(seed=T * 7 + kbase, T=T, kbase=kbase)
    outs, kcs, vcs = run_prefill(rb, [(d, kbase, base)])
    check(outs[0], kcs[0], vcs[0], d, kbase, base)


def test_bf16_inputs(rb):
    d = synth.prefill_inputs(seed=31, T=300, kbase=0)        # values already bf16-representable
    outs, kcs, vcs = run_prefill(rb, [(d, 0, 0)], dtype=BF16)
    check(outs[0], kcs[0], vcs[0], d, 0, 0)


def test_batch_of_prompts(rb):
    cases = [(synth.prefill_inputs(seed=40 + i, T=T, kbase=kb), kb, kb)
             for i, (T, kb) in enumerate([(200, 0), (77, 300), (513, 0), (1, 1000)])]
    outs, kcs, vcs = run_prefill(rb, cases)
    for o, kc, vc, (d, kb, base) in zip(outs, kcs, vcs, cases):
        check(o, kc, vc, d, kb, base)


def test_host_dropin_interleaved(rb):
    """kernel_attn_prefill with pf_attention's own host buffers (p->qkv interleaved Q|G)."""
    lib = rb.lib()
    T, kbase, base = 90, 40, 500
    d = synth.prefill_inputs(seed=55, T=T, kbase=kbase)
    qg = np.ascontiguousarray(np.concatenate([d["q"], d["gate"]], axis=2))   # [T][16][512]
    kc = torch.zeros(kbase + T, 2, 256, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    kc[:kbase] = dev(d["k_cache"])
    vc[:kbase] = dev(d["v_cache"])
    out = np.zeros((T, 16, 256), np.float32)
    k = np.ascontiguousarray(d["k"])
    v = np.ascontiguousarray(d["v"])
    rc = lib.kernel_attn_prefill(qg.ctypes.data, k.ctypes.data, v.ctypes.data, d["q_norm"].ctypes.data,
                                 d["k_norm"].ctypes.data, kc.data_ptr(), vc.data_ptr(), kbase + T, kbase,
                                 base, T, out.ctypes.data)
    assert rc == 0, rb.last_error()
    ref, _, _ = oracle_of(d, kbase, base)
    assert O.maxrel(out, ref) <= TOL


def test_config3_prompt_sampled_rows(rb):
    """One config-3 prompt (8192 tokens, bf16 inputs): sampled rows against the row oracle."""
    T = 8192
    d = synth.prefill_inputs(seed=3, T=T, kbase=0)
    outs, kcs, vcs = run_prefill(rb, [(d, 0, 0)], dtype=BF16)
    rows = np.array([0, 1, 63, 64, 127, 128, 129, 1000, 4095, 4096, 6000, 8190, 8191])
    ref = O.attn_prefill_rows(d["q"], d["gate"], d["k"], d["v"], d["q_norm"], d["k_norm"],
                              d["k_cache"], d["v_cache"], 0, 0, rows)
    got = outs[0][rows]
    assert np.isfinite(outs[0]).all()
    assert O.maxrel(got, ref) <= TOL, O.maxrel(got, ref)
