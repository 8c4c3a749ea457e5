"""Chunked Gated DeltaNet prefill (libroaster_b200, tcgen05) vs the CPU oracle's sequential
recurrence (restating delta_head, model.c:1507-1534, as pf_ssm runs it, model.c:1644-1658).

Tolerance (maxrel = max|a-b|/max|ref|, src/test_kernels.c:31): 1e-4 on the fp32 state -- the
bar for the state after 1k steps -- and on the per-token outputs. The chunked form regroups the
same arithmetic, so the gap is rounding only."""
import numpy as np
import pytest
import torch

import oracle as O
from roaster_b200 import synth
from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu
TOL = 1e-4


def run_gpu(rb, prompts, states):
    """prompts: list of input dicts; states: [n,32,128,128]. Returns (outs, final states)."""
    ds = dev(states)
    d = [{k: dev(v) for k, v in p.items()} for p in prompts]
    outs = [torch.zeros(p["q"].shape[0], 32, 128, device="cuda") for p in prompts]
    jobs = [rb.delta_prefill_job(ds[i], x["q"], x["k"], x["v"], x["g"], x["beta"], outs[i], x["q"].shape[0])
            for i, x in enumerate(d)]
    rb.deltanet_prefill_batch(jobs)
    rb.synchronize()
    return [host(o) for o in outs], host(ds)


def run_ref(prompt, state):
    st = state.copy()
    out = O.delta_prefill(st, prompt["q"], prompt["k"], prompt["v"], prompt["g"], prompt["beta"])
    return out, st


@pytest.mark.parametrize("T", [64, 1, 63, 65, 200])
def test_short_prompts(rb, oracle_lib, T):
    """One chunk, a partial chunk, and ragged tails."""
    p = synth.delta_prompt(10 + T, T)
    st0 = synth.delta_state(20 + T, 1)
    (out,), st = run_gpu(rb, [p], st0)
    ref, st_ref = run_ref(p, st0[0])
    assert O.maxrel(out, ref) < TOL
    assert O.maxrel(st[0], st_ref) < TOL


def test_zero_initial_state(rb, oracle_lib):
    """A fresh prompt starts from S = 0 (every row scale of S_0 degenerate)."""
    p = synth.delta_prompt(31, 130)
    st0 = np.zeros((1, 32, 128, 128), np.float32)
    (out,), st = run_gpu(rb, [p], st0)
    ref, st_ref = run_ref(p, st0[0])
    assert O.maxrel(out, ref) < TOL
    assert O.maxrel(st[0], st_ref) < TOL


def test_1024_tokens_state_tolerance(rb, oracle_lib):
    """the fp32 state within 1e-4 of the reference after 1k tokens."""
    p = synth.delta_prompt(41, 1024)
    st0 = synth.delta_state(42, 1)
    (out,), st = run_gpu(rb, [p], st0)
    ref, st_ref = run_ref(p, st0[0])
    assert O.maxrel(st[0], st_ref) < TOL
    assert O.maxrel(out, ref) < TOL
    assert O.maxrel(out[-64:], ref[-64:]) < TOL


def test_batch_of_ragged_prompts(rb, oracle_lib):
    """Independent prompts of different lengths in one launch, each with its own state."""
    Ts = [100, 64, 257, 3]
    ps = [synth.delta_prompt(50 + i, T) for i, T in enumerate(Ts)]
    st0 = synth.delta_state(60, len(Ts))
    outs, st = run_gpu(rb, ps, st0)
    for i, p in enumerate(ps):
        ref, st_ref = run_ref(p, st0[i])
        assert O.maxrel(outs[i], ref) < TOL, i
        assert O.maxrel(st[i], st_ref) < TOL, i


def test_extreme_ranges(rb, oracle_lib):
    """Strong decay (exp underflow inside a chunk), beta = 1, zero q/k rows, and v spanning
    1e-3 .. 1e3 across heads: exercises the power-of-two operand scaling."""
    T = 150
    p = synth.delta_prompt(70, T)
    p["g"][:, :8] = -40.0                       # decays to exactly zero within two tokens
    p["g"][:, 8:16] = 0.0                       # no decay at all
    p["beta"][:, 16:20] = 1.0
    p["q"][5] = 0.0
    p["k"][7] = 0.0
    scale = np.logspace(-3, 3, 32).astype(np.float32)
    p["v"] *= scale[None, :, None]
    st0 = synth.delta_state(71, 1) * scale[None, :, None, None]
    (out,), st = run_gpu(rb, [p], st0)
    ref, st_ref = run_ref(p, st0[0])
    for h in range(32):                         # per head: the scales differ by 1e6
        assert O.maxrel(out[:, h], ref[:, h]) < TOL, h
        assert O.maxrel(st[0, h], st_ref[h]) < TOL, h


def test_matches_decode_kernel(rb, oracle_lib):
    """Prefill over T tokens leaves the same state as T decode steps of the step kernel."""
    T = 96
    p = synth.delta_prompt(80, T)
    st0 = synth.delta_state(81, 1)
    (out,), st = run_gpu(rb, [p], st0)
    ds = dev(st0[0])
    d = {k: dev(v) for k, v in p.items()}
    o = torch.zeros(T, 32, 128, device="cuda")
    for t in range(T):
        rb.deltanet_step_batch([rb.delta_job(ds, d["q"][t], d["k"][t], d["v"][t], d["g"][t],
                                             d["beta"][t], o[t])])
    rb.synchronize()
    assert O.maxrel(out, host(o)) < TOL
    assert O.maxrel(st[0], host(ds)) < TOL


def test_host_entry_point(rb, oracle_lib):
    """kernel_deltanet_prefill: host q/k/v/g/beta/out, device state (the pf_ssm drop-in)."""
    import ctypes as C
    T = 77
    p = synth.delta_prompt(90, T)
    st0 = synth.delta_state(91, 1)
    ds = dev(st0[0])
    out = np.zeros((T, 32, 128), np.float32)
    f = lambda a: np.ascontiguousarray(a, np.float32).ctypes.data_as(C.c_void_p)
    rb.check(rb.lib().kernel_deltanet_prefill(ds.data_ptr(), T, f(p["q"]), f(p["k"]), f(p["v"]),
                                              f(p["g"]), f(p["beta"]), out.ctypes.data_as(C.c_void_p)),
             "kernel_deltanet_prefill")
    ref, st_ref = run_ref(p, st0[0])
    assert O.maxrel(out, ref) < TOL
    assert O.maxrel(host(ds), st_ref) < TOL


def test_config3_prompt_8192(rb, oracle_lib):
    """Config 3 length: one 8192-token prompt (128 chunks) against the sequential oracle."""
    T = 8192
    p = synth.delta_prompt(100, T)
    st0 = np.zeros((1, 32, 128, 128), np.float32)
    (out,), st = run_gpu(rb, [p], st0)
    ref, st_ref = run_ref(p, st0[0])
    assert O.maxrel(st[0], st_ref) < TOL
    assert O.maxrel(out, ref) < TOL
