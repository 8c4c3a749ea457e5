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


def test_registered_host_buffers_run_in_place(rb, oracle_lib):
    """With the host buffers registered (kernel_cuda_host_register), both host-batch entry points
    move the buffers' contiguous runs with the copy engine directly (no staging memcpy); the
    results equal, bit for bit, the device-pointer batches on the same inputs, over two calls in
    a row, and unregistering falls back to the staging path with the same results. The attention
    gates here are a buffer of their own, so they copy in beside the decode kernel; the 120
    DeltaNet jobs copy in and out in pipelined chunks."""
    import ctypes as C
    lib = rb.lib()
    N, L = 12, 900
    ds = [synth.attn_decode_inputs(seed=500 + i, length=L + 37 * i) for i in range(N)]
    NL = 120                                  # enough DeltaNet jobs for the pipelined (chunked) copies
    st0 = synth.delta_state(501, NL)
    seq = synth.delta_sequence(502, 1, NL)
    # one allocation for every host input and output, registered once
    sizes = {"q": N * 4096, "gate": N * 4096, "kn": N * 512, "vn": N * 512, "norms": 512, "out": N * 4096,
             "dq": NL * 2048, "dk": NL * 2048, "dv": NL * 4096, "dg": NL * 32, "db": NL * 32, "dout": NL * 4096}
    host_buf = np.zeros(sum(sizes.values()), np.float32)
    H, o = {}, 0
    for k, n in sizes.items():
        H[k] = host_buf[o:o + n]
        o += n
    H["q"] = H["q"].reshape(N, 16, 256)
    H["gate"] = H["gate"].reshape(N, 16, 256)
    H["kn"] = H["kn"].reshape(N, 2, 256)
    H["vn"] = H["vn"].reshape(N, 2, 256)
    H["out"] = H["out"].reshape(N, 16, 256)
    for i, d in enumerate(ds):
        H["q"][i], H["gate"][i], H["kn"][i], H["vn"][i] = d["q"], d["gate"], d["k_new"], d["v_new"]
    H["norms"][:256], H["norms"][256:] = ds[0]["q_norm"], ds[0]["k_norm"]
    for k, src in (("dq", "q"), ("dk", "k"), ("dv", "v"), ("dg", "g"), ("db", "beta")):
        H[k][...] = seq[src][0].reshape(-1)
    H["dq"], H["dk"] = H["dq"].reshape(NL, 16, 128), H["dk"].reshape(NL, 16, 128)
    H["dv"], H["dout"] = H["dv"].reshape(NL, 32, 128), H["dout"].reshape(NL, 32, 128)
    H["dg"], H["db"] = H["dg"].reshape(NL, 32), H["db"].reshape(NL, 32)

    def caches():
        out = []
        for d in ds:
            Ld = d["length"]
            kc = torch.zeros(Ld + 4, 2, 256, dtype=torch.float16, device="cuda")
            vc = torch.zeros_like(kc)
            kc[:Ld] = dev(d["k_cache"])
            vc[:Ld] = dev(d["v_cache"])
            out.append((kc, vc))
        return out

    def run_host(cs, st):
        outs = []
        for step in range(2):
            jobs = [rb.attn_job(H["q"][i].ctypes.data, H["gate"][i].ctypes.data, H["kn"][i].ctypes.data,
                                H["vn"][i].ctypes.data, H["norms"].ctypes.data, H["norms"][256:].ctypes.data,
                                cs[i][0], cs[i][1], d["length"] + step, d["length"] + step, H["out"][i].ctypes.data)
                    for i, d in enumerate(ds)]
            rb.attn_decode_batch_host(jobs)
            rb.deltanet_step_batch_host([rb.delta_job(st[l], H["dq"][l].ctypes.data, H["dk"][l].ctypes.data,
                                                      H["dv"][l].ctypes.data, H["dg"][l].ctypes.data,
                                                      H["db"][l].ctypes.data, H["dout"][l].ctypes.data)
                                         for l in range(NL)])
            outs.append((H["out"].copy(), H["dout"].copy()))
        return outs

    # device-pointer reference
    cs_d, st_d = caches(), dev(st0)
    dq = {k: dev(np.ascontiguousarray(H[k])) for k in ("q", "gate", "kn", "vn", "norms", "dq", "dk", "dv", "dg", "db")}
    ref_outs = []
    for step in range(2):
        ao = torch.zeros(N, 16, 256, device="cuda")
        do = torch.zeros(NL, 32, 128, device="cuda")
        rb.attn_decode_batch([rb.attn_job(dq["q"][i], dq["gate"][i], dq["kn"][i], dq["vn"][i], dq["norms"][:256],
                                          dq["norms"][256:], cs_d[i][0], cs_d[i][1], d["length"] + step,
                                          d["length"] + step, ao[i]) for i, d in enumerate(ds)])
        rb.deltanet_step_batch([rb.delta_job(st_d[l], dq["dq"][l], dq["dk"][l], dq["dv"][l], dq["dg"][l],
                                             dq["db"][l], do[l]) for l in range(NL)])
        ref_outs.append((host(ao), host(do)))

    assert lib.kernel_cuda_host_register(C.c_void_p(host_buf.ctypes.data), host_buf.nbytes) == 0, rb.last_error()
    try:
        cs_r, st_r = caches(), dev(st0)
        got = run_host(cs_r, st_r)
    finally:
        assert lib.kernel_cuda_host_unregister(C.c_void_p(host_buf.ctypes.data)) == 0, rb.last_error()
    cs_s, st_s = caches(), dev(st0)
    staged = run_host(cs_s, st_s)
    for step in range(2):
        for a, b, c in zip(got[step], staged[step], ref_outs[step]):
            assert np.array_equal(a, c) and np.array_equal(b, c)
    assert torch.equal(st_r, st_d) and torch.equal(st_s, st_d)
    for i, d in enumerate(ds):
        Ld = d["length"]
        assert torch.equal(cs_r[i][0][:Ld + 2], cs_d[i][0][:Ld + 2])
        assert torch.equal(cs_r[i][1][:Ld + 2], cs_d[i][1][:Ld + 2])
    ref, _, _ = O.attn_decode(ds[0]["q"], ds[0]["gate"], ds[0]["k_new"], ds[0]["v_new"], ds[0]["q_norm"],
                              ds[0]["k_norm"], ds[0]["k_cache"], ds[0]["v_cache"], ds[0]["length"], ds[0]["length"])
    assert O.maxrel(got[0][0][0], ref) <= 2e-3


def test_registered_interleaved_q_gate(rb, oracle_lib):
    """The reference's projection layout: each head's q row followed by its gate row
    (qg_stride 512, model.c:801-805), registered. The gates share the q rows' run, so the whole
    block copies in before the decode kernel; the output equals the device-pointer batch on the
    same values bit for bit."""
    import ctypes as C
    lib = rb.lib()
    N = 6
    ds = [synth.attn_decode_inputs(seed=700 + i, length=500 + 91 * i) for i in range(N)]
    host_buf = np.zeros(N * 8192 + 512 + N * 4096 + N * 1024, np.float32)   # every buffer registered
    qg = host_buf[:N * 8192].reshape(N, 16, 512)
    norms = host_buf[N * 8192:N * 8192 + 512]
    out = host_buf[N * 8192 + 512:N * 12288 + 512].reshape(N, 16, 256)
    kv_new = host_buf[N * 12288 + 512:].reshape(N, 2, 2, 256)
    for i, d in enumerate(ds):
        qg[i, :, :256], qg[i, :, 256:] = d["q"], d["gate"]
        kv_new[i, 0], kv_new[i, 1] = d["k_new"], d["v_new"]
    norms[:256], norms[256:] = ds[0]["q_norm"], ds[0]["k_norm"]

    def caches():
        res = []
        for d in ds:
            kc = torch.zeros(d["length"] + 2, 2, 256, dtype=torch.float16, device="cuda")
            vc = torch.zeros_like(kc)
            kc[:d["length"]] = dev(d["k_cache"])
            vc[:d["length"]] = dev(d["v_cache"])
            res.append((kc, vc))
        return res

    cs_d = caches()
    dqg, dn, dkv = dev(qg), dev(norms), dev(kv_new)
    ao = torch.zeros(N, 16, 256, device="cuda")
    rb.attn_decode_batch([rb.attn_job(dqg[i], dqg[i, 0, 256:], dkv[i, 0], dkv[i, 1], dn[:256], dn[256:],
                                      cs_d[i][0], cs_d[i][1], d["length"], d["length"], ao[i], qg_stride=512)
                          for i, d in enumerate(ds)])
    ref = host(ao)
    assert lib.kernel_cuda_host_register(C.c_void_p(host_buf.ctypes.data), host_buf.nbytes) == 0, rb.last_error()
    try:
        cs_r = caches()
        jobs = [rb.attn_job(qg[i].ctypes.data, qg[i, 0, 256:].ctypes.data, kv_new[i, 0].ctypes.data,
                            kv_new[i, 1].ctypes.data, norms.ctypes.data, norms[256:].ctypes.data, cs_r[i][0],
                            cs_r[i][1], d["length"], d["length"], out[i].ctypes.data, qg_stride=512)
                for i, d in enumerate(ds)]
        rb.attn_decode_batch_host(jobs)
    finally:
        assert lib.kernel_cuda_host_unregister(C.c_void_p(host_buf.ctypes.data)) == 0, rb.last_error()
    assert np.array_equal(out, ref)
    for i, d in enumerate(ds):
        assert torch.equal(cs_r[i][0][:d["length"] + 1], cs_d[i][0][:d["length"] + 1])
