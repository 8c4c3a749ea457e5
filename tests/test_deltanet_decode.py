"""Gated DeltaNet decode step (libroaster_b200) vs the CPU oracle (restating model.c:272-323).
Tolerance (maxrel = max|a-b|/max|ref|, src/test_kernels.c:31): 1e-4 on the fp32 state after
1024 steps and on the outputs."""
import numpy as np
import pytest
import torch

import oracle as O
from roaster_b200 import synth
from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu
TOL = 1e-4


def step_jobs(R, states, seq, t, outs):
    L = states.shape[0]
    return [R.delta_job(states[l], seq["q"][t, l], seq["k"][t, l], seq["v"][t, l], seq["g"][t, l],
                        seq["beta"][t, l], outs[l]) for l in range(L)]


def test_single_step(rb, oracle_lib):
    st0 = synth.delta_state(1, 1)
    seq = synth.delta_sequence(2, 1, 1)
    ds, dseq = dev(st0), {k: dev(v) for k, v in seq.items()}
    out = torch.zeros(1, 32, 128, device="cuda")
    rb.deltanet_step_batch(step_jobs(rb, ds, dseq, 0, out))
    rb.synchronize()
    st = st0[0].copy()
    ref = O.delta_step(st, seq["q"][0, 0], seq["k"][0, 0], seq["v"][0, 0], seq["g"][0, 0],
                       seq["beta"][0, 0])
    assert O.maxrel(host(out)[0], ref) < 1e-5
    assert O.maxrel(host(ds)[0], st) < 1e-5


def test_1024_steps_state_tolerance(rb, oracle_lib):
    """fp32 state within 1e-4 of the reference after 1k sequential steps."""
    T = 1024
    st0 = synth.delta_state(3, 1)
    seq = synth.delta_sequence(4, T, 1)
    ds, dseq = dev(st0), {k: dev(v) for k, v in seq.items()}
    outs = torch.zeros(T, 1, 32, 128, device="cuda")
    for t in range(T):
        rb.deltanet_step_batch(step_jobs(rb, ds, dseq, t, outs[t]))
    rb.synchronize()
    st = st0[0].copy()
    ref = O.delta_prefill(st, seq["q"][:, 0], seq["k"][:, 0], seq["v"][:, 0], seq["g"][:, 0],
                          seq["beta"][:, 0])
    got = host(outs)[:, 0]
    assert O.maxrel(host(ds)[0], st) < TOL
    assert O.maxrel(got[-1], ref[-1]) < TOL
    assert O.maxrel(got, ref) < TOL


def test_thirty_layers_one_launch(rb, oracle_lib):
    """Config 1 step shape: 30 independent layer states in one batch, a few steps."""
    L, T = 30, 3
    st0 = synth.delta_state(5, L)
    seq = synth.delta_sequence(6, T, L)
    ds, dseq = dev(st0), {k: dev(v) for k, v in seq.items()}
    outs = torch.zeros(T, L, 32, 128, device="cuda")
    for t in range(T):
        rb.deltanet_step_batch(step_jobs(rb, ds, dseq, t, outs[t]))
    rb.synchronize()
    got_st, got = host(ds), host(outs)
    for l in (0, 13, 29):
        st = st0[l].copy()
        ref = O.delta_prefill(st, seq["q"][:, l], seq["k"][:, l], seq["v"][:, l], seq["g"][:, l],
                              seq["beta"][:, l])
        assert O.maxrel(got_st[l], st) < TOL
        assert O.maxrel(got[:, l], ref) < TOL


def test_host_dropin(rb, oracle_lib):
    """kernel_deltanet_step: host q/k/v/g/beta/out, device-resident state (model.c call site)."""
    import ctypes as C
    st0 = synth.delta_state(8, 1)[0]
    seq = synth.delta_sequence(9, 4, 1)
    ds = dev(st0)
    st = st0.copy()
    lib = rb.lib()
    for t in range(4):
        args = [np.ascontiguousarray(seq[k][t, 0]) for k in ("q", "k", "v", "g", "beta")]
        out = np.zeros((32, 128), np.float32)
        rc = lib.kernel_deltanet_step(ds.data_ptr(), *[a.ctypes.data for a in args], out.ctypes.data)
        assert rc == 0, rb.last_error()
        ref = O.delta_step(st, *args)
        assert O.maxrel(out, ref) < 1e-5
    assert O.maxrel(host(ds), st) < 1e-5
