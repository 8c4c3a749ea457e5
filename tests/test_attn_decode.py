"""Gated GQA decode attention (libroaster_b200) vs the CPU oracle (restating model.c:801-861).
Tolerance: maxrel <= 2e-3 on the gated outputs (f16 tensor-core operands, fp32 accumulation).
The appended K is compared within f16 rounding of the oracle's fp32 value; V bit-exact."""
import numpy as np
import pytest
import torch

import oracle as O
from roaster_b200 import synth
from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu
TOL = 2e-3


def make_slot(d, capacity=None, interleaved=False):
    L = d["length"]
    cap = capacity or L + 1
    kc = torch.zeros(cap, 2, 256, dtype=torch.float16, device="cuda")
    vc = torch.zeros(cap, 2, 256, dtype=torch.float16, device="cuda")
    if L:
        kc[:L] = dev(d["k_cache"])
        vc[:L] = dev(d["v_cache"])
    s = {"kc": kc, "vc": vc, "out": torch.zeros(16, 256, device="cuda"),
         "k_new": dev(d["k_new"]), "v_new": dev(d["v_new"]), "q_norm": dev(d["q_norm"]),
         "k_norm": dev(d["k_norm"])}
    if interleaved:
        qg = dev(np.concatenate([d["q"], d["gate"]], axis=1))
        s["qg"] = qg
        s["q"], s["gate"], s["stride"] = qg, qg.data_ptr() + 256 * 4, 512
    else:
        s["q"], s["gate"], s["stride"] = dev(d["q"]), dev(d["gate"]), 256
    return s


def job(R, s, d):
    return R.attn_job(s["q"], s["gate"], s["k_new"], s["v_new"], s["q_norm"], s["k_norm"], s["kc"],
                      s["vc"], d["length"], d["position"], s["out"], qg_stride=s["stride"])


def check_slot(s, d):
    ref, ka, va = O.attn_decode(d["q"], d["gate"], d["k_new"], d["v_new"], d["q_norm"],
                                d["k_norm"], d["k_cache"], d["v_cache"], d["length"], d["position"])
    out = host(s["out"])
    assert np.isfinite(out).all()
    assert O.maxrel(out, ref) <= TOL, O.maxrel(out, ref)
    L = d["length"]
    kapp = host(s["kc"][L]).astype(np.float32)
    assert np.abs(kapp - ka).max() <= 2e-3 * max(1.0, np.abs(ka).max())
    assert np.array_equal(host(s["vc"][L]), va.astype(np.float16))
    # cached rows untouched
    if L:
        assert np.array_equal(host(s["kc"][:L]), d["k_cache"])


def test_config0(rb, oracle_lib):
    d = synth.attn_decode_inputs(seed=0, length=512)
    s = make_slot(d)
    rb.attn_decode_batch([job(rb, s, d)])
    rb.synchronize()
    check_slot(s, d)


@pytest.mark.parametrize("length", [0, 1, 15, 16, 17, 63, 64, 65, 300, 2049, 9000])
def test_lengths(rb, oracle_lib, length):
    d = synth.attn_decode_inputs(seed=100 + length, length=length)
    s = make_slot(d, capacity=length + 7)
    rb.attn_decode_batch([job(rb, s, d)])
    rb.synchronize()
    check_slot(s, d)


def test_large_position_rope(rb, oracle_lib):
    d = synth.attn_decode_inputs(seed=5, length=100, position=262143)
    s = make_slot(d)
    rb.attn_decode_batch([job(rb, s, d)])
    rb.synchronize()
    check_slot(s, d)


def test_interleaved_projection_layout(rb, oracle_lib):
    d = synth.attn_decode_inputs(seed=6, length=777)
    s = make_slot(d, interleaved=True)
    rb.attn_decode_batch([job(rb, s, d)])
    rb.synchronize()
    check_slot(s, d)


def test_batch_of_ragged_slots(rb, oracle_lib):
    lens = [1, 500, 4097, 33, 12000, 0, 2048, 70]
    ds = [synth.attn_decode_inputs(seed=200 + i, length=L) for i, L in enumerate(lens)]
    ss = [make_slot(d) for d in ds]
    rb.attn_decode_batch([job(rb, s, d) for s, d in zip(ss, ds)])
    rb.synchronize()
    for s, d in zip(ss, ds):
        check_slot(s, d)


def test_more_slots_than_one_launch(rb, oracle_lib):
    n = 70                                     # > 64 jobs per launch
    ds = [synth.attn_decode_inputs(seed=300 + i, length=16 + 9 * i) for i in range(n)]
    ss = [make_slot(d) for d in ds]
    rb.attn_decode_batch([job(rb, s, d) for s, d in zip(ss, ds)])
    rb.synchronize()
    for i in (0, 33, 63, 64, 69):
        check_slot(ss[i], ds[i])


def test_repeated_calls_reset_counters(rb, oracle_lib):
    d = synth.attn_decode_inputs(seed=8, length=1500)
    s = make_slot(d)
    for _ in range(3):
        s["out"].zero_()
        rb.attn_decode_batch([job(rb, s, d)])
        rb.synchronize()
        check_slot(s, d)


def test_host_dropin_consecutive_steps(rb, oracle_lib):
    """kernel_attn_decode with model.c's host buffers over 3 consecutive steps: each step appends
    and the next attends to the appended (f16) row."""
    lib = rb.lib()
    d = synth.attn_decode_inputs(seed=9, length=300)
    cap = 310
    kc = torch.zeros(cap, 2, 256, dtype=torch.float16, device="cuda")
    vc = torch.zeros(cap, 2, 256, dtype=torch.float16, device="cuda")
    kc[:300] = dev(d["k_cache"])
    vc[:300] = dev(d["v_cache"])
    rng = np.random.default_rng(10)
    for step in range(3):
        L = 300 + step
        qg = rng.standard_normal((16, 512)).astype(np.float32)
        kn = rng.standard_normal((2, 256)).astype(np.float32)
        vn = rng.standard_normal((2, 256)).astype(np.float32)
        out = np.zeros((16, 256), np.float32)
        rc = lib.kernel_attn_decode(qg.ctypes.data, kn.ctypes.data, vn.ctypes.data,
                                    d["q_norm"].ctypes.data, d["k_norm"].ctypes.data,
                                    kc.data_ptr(), vc.data_ptr(), cap, L, L, out.ctypes.data)
        assert rc == 0, rb.last_error()
        window_k, window_v = host(kc[:L]), host(vc[:L])
        ref, _, _ = O.attn_decode(qg[:, :256], qg[:, 256:], kn, vn, d["q_norm"], d["k_norm"],
                                  window_k, window_v, L, L)
        assert O.maxrel(out, ref) <= TOL


def test_window_full_is_rejected(rb):
    d = synth.attn_decode_inputs(seed=1, length=32)
    s = make_slot(d, capacity=32)               # no room for the new token
    with pytest.raises(RuntimeError):
        rb.attn_decode_batch([job(rb, s, d)])


def test_split_partials_and_merge(rb, oracle_lib):
    """Long-context mode: one slot's window in three slices (as on three GPUs), partial records
    per slice, then the merge. Equals the single-device decode; each slice's record equals the
    oracle's partial over that slice."""
    L = 3000
    d = synth.attn_decode_inputs(seed=12, length=L)
    full = make_slot(d, capacity=L + 1)
    bounds = [(0, 1000), (1000, 2000), (2000, 3000)]
    jobs = []
    for i, (a, b) in enumerate(bounds):
        last = i == len(bounds) - 1
        jobs.append(rb.attn_job(full["q"], full["gate"], full["k_new"], full["v_new"],
                                full["q_norm"], full["k_norm"],
                                full["kc"].data_ptr() + a * 1024, full["vc"].data_ptr() + a * 1024,
                                b - a, d["position"], 0, append=last,
                                capacity=(b - a + 1) if last else (b - a)))
    partials = torch.zeros(3, 2, rb.ATTN_PARTIAL_FLOATS, device="cuda")
    rb.attn_decode_partial_batch(jobs, partials)
    rb.synchronize()
    P = host(partials)
    for i, (a, b) in enumerate(bounds[:2]):
        m, l, o = O.attn_decode_partial(d["q"], d["q_norm"], d["k_cache"], d["v_cache"], a, b,
                                        d["position"])
        for kvh in range(2):
            rec = P[i, kvh]
            hs = slice(8 * kvh, 8 * kvh + 8)
            assert np.allclose(rec[:8], m[hs] * np.log2(np.e), atol=2e-3)
            assert O.maxrel(rec[16:].reshape(8, 256), o[hs]) <= TOL
    rb.attn_merge_partials(partials, 3, [full["gate"]], [full["out"]])
    rb.synchronize()
    check_slot(full, d)
