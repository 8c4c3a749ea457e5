"""Host-buffer batch entry points (kernel_attn_decode_batch_host, kernel_deltanet_step_batch_host)
at batch sizes that take the chunked, multi-threaded staging (16 or more jobs): outputs and
caches / states must equal, bit for bit, those of the device-pointer batches run on the same
inputs, and match the oracle (restating model.c:801-861 and 272-323) within the tolerances of
the decode tests (2e-3 attention, 1e-5 one DeltaNet step)."""
import numpy as np
import pytest
import torch

import oracle as O
from roaster_b200 import synth
from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu


def test_attention_host_batch_matches_device_batch(rb, oracle_lib):
    N = 20
    ds = [synth.attn_decode_inputs(seed=300 + i, length=64 + 53 * i, position=64 + 53 * i) for i in range(N)]
    caches = []
    for d in ds:
        L = d["length"]
        kc = torch.zeros(L + 4, 2, 256, dtype=torch.float16, device="cuda")
        vc = torch.zeros_like(kc)
        kc[:L] = dev(d["k_cache"])
        vc[:L] = dev(d["v_cache"])
        caches.append((kc, vc))
    caches2 = [(k.clone(), v.clone()) for k, v in caches]
    # host path: numpy buffers
    hin = [{k: np.ascontiguousarray(d[k]) for k in ("q", "gate", "k_new", "v_new", "q_norm", "k_norm")} for d in ds]
    hout = [np.zeros((16, 256), np.float32) for _ in range(N)]
    jobs = [rb.attn_job(h["q"].ctypes.data, h["gate"].ctypes.data, h["k_new"].ctypes.data, h["v_new"].ctypes.data,
                        h["q_norm"].ctypes.data, h["k_norm"].ctypes.data, kc, vc, d["length"], d["position"],
                        o.ctypes.data)
            for h, o, (kc, vc), d in zip(hin, hout, caches, ds)]
    rb.attn_decode_batch_host(jobs)
    # device path on copies of the same caches
    dins = [{k: dev(h[k]) for k in h} for h in hin]
    douts = [torch.zeros(16, 256, device="cuda") for _ in range(N)]
    djobs = [rb.attn_job(x["q"], x["gate"], x["k_new"], x["v_new"], x["q_norm"], x["k_norm"], kc, vc, d["length"],
                         d["position"], o)
             for x, o, (kc, vc), d in zip(dins, douts, caches2, ds)]
    rb.attn_decode_batch(djobs)
    rb.synchronize()
    for i, d in enumerate(ds):
        assert np.array_equal(hout[i], host(douts[i]))
        L = d["length"]
        assert torch.equal(caches[i][0][L], caches2[i][0][L]) and torch.equal(caches[i][1][L], caches2[i][1][L])
        ref, _, _ = O.attn_decode(d["q"], d["gate"], d["k_new"], d["v_new"], d["q_norm"], d["k_norm"],
                                  d["k_cache"], d["v_cache"], L, d["position"])
        assert O.maxrel(hout[i], ref) <= 2e-3


def test_deltanet_host_batch_matches_device_batch(rb, oracle_lib):
    N = 40
    st0 = synth.delta_state(400, N)
    seq = synth.delta_sequence(401, 1, N)
    hs = {k: np.ascontiguousarray(v[0]) for k, v in seq.items()}        # [N][...]
    dst_h, dst_d = dev(st0), dev(st0)
    hout = np.zeros((N, 32, 128), np.float32)
    jobs = [rb.delta_job(dst_h[l], hs["q"][l].ctypes.data, hs["k"][l].ctypes.data, hs["v"][l].ctypes.data,
                         hs["g"][l].ctypes.data, hs["beta"][l].ctypes.data, hout[l].ctypes.data) for l in range(N)]
    rb.deltanet_step_batch_host(jobs)
    dseq = {k: dev(v) for k, v in hs.items()}
    dout = torch.zeros(N, 32, 128, device="cuda")
    rb.deltanet_step_batch([rb.delta_job(dst_d[l], dseq["q"][l], dseq["k"][l], dseq["v"][l], dseq["g"][l],
                                         dseq["beta"][l], dout[l]) for l in range(N)])
    rb.synchronize()
    assert np.array_equal(hout, host(dout))
    assert torch.equal(dst_h, dst_d)
    for l in (0, 17, 39):
        st = st0[l].copy()
        ref = O.delta_step(st, hs["q"][l], hs["k"][l], hs["v"][l], hs["g"][l], hs["beta"][l])
        assert O.maxrel(hout[l], ref) < 1e-5
        assert O.maxrel(host(dst_h)[l], st) < 1e-5
