"""Gated DeltaNet pre-ops (conv1d + SiLU + L2-norm + beta/g, model.c:1291-1328) and post-op
(gated RMSNorm, model.c:1333-1343) on the GPU, and the fused recurrent-layer drop-ins, against the
CPU oracle (itself equal bit for bit to the reference's pf_ssm, tests/test_oracle.py).

Tolerances (maxrel = max|a-b|/max|ref|): 1e-5 for the elementwise pre/post ops (fp32; only the
libm expf/log1pf and reduction order differ); 1e-4 for whole layers (the recurrence's bar)."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
from roaster_b200 import synth
from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu
TOL_OP = 1e-5
TOL_LAYER = 1e-4


def gpu_preop(rb, prompts):
    """prompts: list of input dicts (delta_layer_inputs). Returns per prompt (outs, conv_state)."""
    keep, jobs, outs = [], [], []
    for d in prompts:
        T = d["qkv"].shape[0]
        t = {k: dev(d[k]) for k in ("qkv", "alpha", "beta", "conv_state", "conv_w", "dt", "a")}
        o = {"q": torch.zeros(T, 16, 128, device="cuda"), "k": torch.zeros(T, 16, 128, device="cuda"),
             "v": torch.zeros(T, 32, 128, device="cuda"), "g": torch.zeros(T, 32, device="cuda"),
             "beta": torch.zeros(T, 32, device="cuda")}
        keep.append(t)
        outs.append(o)
        jobs.append((t["qkv"], t["alpha"], t["beta"], t["conv_state"], t["conv_w"], t["dt"], t["a"],
                     o["q"], o["k"], o["v"], o["g"], o["beta"], T))
    rb.deltanet_preop_batch(jobs)
    rb.synchronize()
    return [({k: host(v) for k, v in o.items()}, host(t["conv_state"])) for o, t in zip(outs, keep)]


@pytest.mark.parametrize("T", [1, 2, 3, 5, 70])
def test_preop(rb, oracle_lib, T):
    d = synth.delta_layer_inputs(20 + T, T)
    (got, conv), = gpu_preop(rb, [d])
    cs = d["conv_state"].copy()
    ref = O.delta_preop(d["qkv"], d["alpha"], d["beta"], cs, d["conv_w"], d["dt"], d["a"])
    for k in ("q", "k", "v", "g", "beta"):
        assert O.maxrel(got[k], ref[k]) < TOL_OP, k
    assert np.array_equal(conv, cs)                      # the history is a pure copy


def test_preop_ragged_batch(rb, oracle_lib):
    ds = [synth.delta_layer_inputs(30 + i, T) for i, T in enumerate([1, 4, 129, 2])]
    res = gpu_preop(rb, ds)
    for d, (got, conv) in zip(ds, res):
        cs = d["conv_state"].copy()
        ref = O.delta_preop(d["qkv"], d["alpha"], d["beta"], cs, d["conv_w"], d["dt"], d["a"])
        for k in ("q", "k", "v", "g", "beta"):
            assert O.maxrel(got[k], ref[k]) < TOL_OP, k
        assert np.array_equal(conv, cs)


def test_preop_decode_steps_in_sequence(rb, oracle_lib):
    """Five decode steps of two layers, one batch of two one-token jobs per step, queued back to
    back on the stream without a host sync between them: a decode token's history shift happens
    inside the pre-op kernel, so each step's conv must read the rows the step before wrote."""
    steps, layers = 5, 2
    ds = [synth.delta_layer_inputs(60 + l, steps) for l in range(layers)]
    dev_in = [{k: dev(d[k]) for k in ("qkv", "alpha", "beta", "conv_state", "conv_w", "dt", "a")} for d in ds]
    outs = [[{"q": torch.zeros(1, 16, 128, device="cuda"), "k": torch.zeros(1, 16, 128, device="cuda"),
              "v": torch.zeros(1, 32, 128, device="cuda"), "g": torch.zeros(1, 32, device="cuda"),
              "beta": torch.zeros(1, 32, device="cuda")} for _ in range(layers)] for _ in range(steps)]
    for s in range(steps):
        jobs = []
        for l in range(layers):
            t, o = dev_in[l], outs[s][l]
            jobs.append((t["qkv"][s:s + 1], t["alpha"][s:s + 1], t["beta"][s:s + 1], t["conv_state"], t["conv_w"],
                         t["dt"], t["a"], o["q"], o["k"], o["v"], o["g"], o["beta"], 1))
        rb.deltanet_preop_batch(jobs)
    rb.synchronize()
    for l, d in enumerate(ds):
        cs = d["conv_state"].copy()
        for s in range(steps):
            ref = O.delta_preop(d["qkv"][s:s + 1], d["alpha"][s:s + 1], d["beta"][s:s + 1], cs, d["conv_w"],
                                d["dt"], d["a"])
            for k in ("q", "k", "v", "g", "beta"):
                assert O.maxrel(host(outs[s][l][k]), ref[k]) < TOL_OP, (s, l, k)
        assert np.array_equal(host(dev_in[l]["conv_state"]), cs)


@pytest.mark.parametrize("T", [1, 70])
def test_postop(rb, oracle_lib, T):
    rng = np.random.default_rng(40 + T)
    x = rng.standard_normal((T, 32, 128)).astype(np.float32) * 3
    z = rng.standard_normal((T, 4096)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    dx, dz, dw = dev(x), dev(z), dev(w)
    rb.deltanet_postop_batch([(dx, dz, dw, T)])
    ref = O.delta_postop(x, z, w)
    assert O.maxrel(host(dx), ref.reshape(T, 32, 128)) < TOL_OP


def _layer_args(d):
    return (d["qkv"], d["z"], d["alpha"], d["beta"], d["conv_w"], d["dt"], d["a"], d["ssm_norm"])


def _fp(a):
    return np.ascontiguousarray(a, np.float32).ctypes.data_as(C.c_void_p)


def test_layer_step_drop_in(rb, oracle_lib):
    """kernel_deltanet_layer_step over 6 consecutive decode tokens (host in/out, device state)."""
    steps = 6
    d = synth.delta_layer_inputs(50, steps)
    st0 = synth.delta_state(51, 1)[0]
    ds, dcs = dev(st0), dev(d["conv_state"])
    dw, ddt, da, dn = dev(d["conv_w"]), dev(d["dt"]), dev(d["a"]), dev(d["ssm_norm"])
    outs = np.zeros((steps, 4096), np.float32)
    for t in range(steps):
        o = np.zeros(4096, np.float32)
        rc = rb.lib().kernel_deltanet_layer_step(ds.data_ptr(), dcs.data_ptr(), dw.data_ptr(), ddt.data_ptr(),
                                                 da.data_ptr(), dn.data_ptr(), _fp(d["qkv"][t]), _fp(d["z"][t]),
                                                 _fp(d["alpha"][t]), _fp(d["beta"][t]), o.ctypes.data_as(C.c_void_p))
        rb.check(rc, "kernel_deltanet_layer_step")
        outs[t] = o
    s_ref, c_ref = st0.copy(), d["conv_state"].copy()
    impl = "ref" if O.have_ref() else "port"
    ref = O.delta_layer(s_ref, c_ref, *_layer_args(d), impl=impl)
    assert O.maxrel(outs, ref.reshape(steps, 4096)) < TOL_LAYER
    assert O.maxrel(host(ds), s_ref) < TOL_LAYER
    assert np.array_equal(host(dcs), c_ref)


@pytest.mark.parametrize("T", [200, 1030])
def test_layer_prefill_drop_in(rb, oracle_lib, T):
    """kernel_deltanet_layer_prefill: pf_ssm's whole layer body over one prompt."""
    d = synth.delta_layer_inputs(60 + T, T)
    st0 = synth.delta_state(61, 1)[0]
    ds, dcs = dev(st0), dev(d["conv_state"])
    dw, ddt, da, dn = dev(d["conv_w"]), dev(d["dt"]), dev(d["a"]), dev(d["ssm_norm"])
    out = np.zeros((T, 4096), np.float32)
    rc = rb.lib().kernel_deltanet_layer_prefill(ds.data_ptr(), dcs.data_ptr(), dw.data_ptr(), ddt.data_ptr(),
                                                da.data_ptr(), dn.data_ptr(), T, _fp(d["qkv"]), _fp(d["z"]),
                                                _fp(d["alpha"]), _fp(d["beta"]), out.ctypes.data_as(C.c_void_p))
    rb.check(rc, "kernel_deltanet_layer_prefill")
    s_ref, c_ref = st0.copy(), d["conv_state"].copy()
    impl = "ref" if (O.have_ref() and T <= 256) else "port"
    ref = O.delta_layer(s_ref, c_ref, *_layer_args(d), impl=impl)
    assert O.maxrel(out, ref.reshape(T, 4096)) < TOL_LAYER
    assert O.maxrel(host(ds), s_ref) < TOL_LAYER
    assert np.array_equal(host(dcs), c_ref)
