"""The fused split-KV combine (kernel_attn_decode_partial_push + kernel_attn_merge_wait) on one
GPU, with the ranks emulated: every emulated rank's push kernel runs first, then each home
rank's merge, all in stream order, so every tag a merge waits on is already set when it starts
(no kernel waits on another kernel running beside it). Against the oracle's decode over the
whole window (model.c:825-856), maxrel 2e-3, over two consecutive steps (the two parity halves
of the receive buffers). Plus the bounded wait: a merge whose tags never arrive reports a
timeout through kernel_cuda_synchronize and leaves the context usable."""
import numpy as np
import pytest
import torch

import oracle as O
from roaster_b200 import splitkv, synth
from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu
TOL = 2e-3


@pytest.mark.parametrize("world,n_slots,L", [(2, 4, 3000), (3, 5, 2500), (4, 6, 4100)])
def test_push_and_merge_two_steps(rb, oracle_lib, world, n_slots, L):
    rng = np.random.default_rng(50 + world)
    qn = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    dqn, dkw = dev(qn), dev(kw)
    K = [rng.standard_normal((L + 2, 2, 256)).astype(np.float16) for _ in range(n_slots)]
    V = [rng.standard_normal((L + 2, 2, 256)).astype(np.float16) for _ in range(n_slots)]
    kcs = [dev(k) for k in K]
    vcs = [dev(v) for v in V]
    recv = [torch.zeros(splitkv.recv_floats(n_slots, world, r), device="cuda") for r in range(world)]
    tags = [torch.zeros(splitkv.tag_words(n_slots, world, r), dtype=torch.int32, device="cuda")
            for r in range(world)]
    rb_ = [x.data_ptr() for x in recv]
    tb_ = [x.data_ptr() for x in tags]
    for step in range(2):
        epoch = step + 1
        Ls = L + step                                # the window grows by the appended token
        vec = [{k: rng.standard_normal(s).astype(np.float32)
                for k, s in (("q", (16, 256)), ("gate", (16, 256)), ("k_new", (2, 256)), ("v_new", (2, 256)))}
               for _ in range(n_slots)]
        dv = [{k: dev(x) for k, x in v.items()} for v in vec]
        for r in range(world):
            lo, hi = splitkv.slice_bounds(Ls, world, r)
            app = splitkv.appends(world, r)
            jobs = [rb.attn_job(d["q"], d["gate"], d["k_new"], d["v_new"], dqn, dkw,
                                kc.data_ptr() + lo * 1024, vc.data_ptr() + lo * 1024, hi - lo, Ls, 0,
                                append=app, capacity=hi - lo + (1 if app else 0))
                    for d, kc, vc in zip(dv, kcs, vcs)]
            dst, tg = splitkv.push_targets(n_slots, world, r, epoch, rb_, tb_)
            rb.attn_decode_partial_push(jobs, dst, tg, epoch)
        out = torch.zeros(n_slots, 16, 256, device="cuda")
        for h in range(world):
            mine = splitkv.home_slots(n_slots, world, h)
            rv, tv = splitkv.merge_view(n_slots, world, h, epoch, rb_[h], tb_[h])
            rb.attn_merge_wait(rv, tv, world, [dv[s]["gate"] for s in mine], [out[s] for s in mine], epoch)
        rb.synchronize()
        got = host(out)
        for s in range(n_slots):
            hk, hv = host(kcs[s]), host(vcs[s])
            ref, ka, va = O.attn_decode(vec[s]["q"], vec[s]["gate"], vec[s]["k_new"], vec[s]["v_new"], qn, kw,
                                        hk[:Ls], hv[:Ls], Ls, Ls)
            assert O.maxrel(got[s], ref) <= TOL, (world, step, s, O.maxrel(got[s], ref))
            assert np.array_equal(hv[Ls], va.astype(np.float16))


def test_merge_wait_times_out_and_context_survives(rb, oracle_lib):
    """Tags that nothing sets: the bounded wait gives up (about a second), the error word reports
    it, the output is not written, and a real decode runs correctly afterwards."""
    n_slots, world = 4, 2
    n = splitkv.home_count(n_slots, world, 0)
    recv = torch.zeros(splitkv.recv_floats(n_slots, world, 0), device="cuda")
    tags = torch.zeros(splitkv.tag_words(n_slots, world, 0), dtype=torch.int32, device="cuda")
    gates = [torch.zeros(16, 256, device="cuda") for _ in range(n)]
    outs = [torch.full((16, 256), 7.0, device="cuda") for _ in range(n)]
    rv, tv = splitkv.merge_view(n_slots, world, 0, 1, recv.data_ptr(), tags.data_ptr())
    rb.attn_merge_wait(rv, tv, 2, gates, outs, 1)
    with pytest.raises(RuntimeError, match="timed out"):
        rb.synchronize()
    assert (host(outs[0]) == 7.0).all()
    d = synth.attn_decode_inputs(seed=3, length=700)
    kc = torch.zeros(701, 2, 256, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    kc[:700] = dev(d["k_cache"])
    vc[:700] = dev(d["v_cache"])
    out = torch.zeros(16, 256, device="cuda")
    rb.attn_decode_batch([rb.attn_job(dev(d["q"]), dev(d["gate"]), dev(d["k_new"]), dev(d["v_new"]),
                                      dev(d["q_norm"]), dev(d["k_norm"]), kc, vc, 700, 700, out)])
    rb.synchronize()
    ref, _, _ = O.attn_decode(d["q"], d["gate"], d["k_new"], d["v_new"], d["q_norm"], d["k_norm"],
                              d["k_cache"], d["v_cache"], 700, 700)
    assert O.maxrel(host(out), ref) <= TOL
