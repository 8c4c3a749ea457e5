"""The allocation-free decode entry point, kernel_attn_decode_batch_noalloc.

It is for callers that cannot allocate device memory while serving (a fixed device-memory
budget set at start-up, or code that must not enter an allocator at decode time): its scratch is
a static device array instead of library-allocated memory. This file is collected last so that a
failure here stops a `-x` run only after every other test has run; it must pass on its own in a
fresh process as well as after the other tests.

Check: two decode steps in a row through the new entry point give the same outputs and cache
appends as the allocating entry point kernel_attn_decode_batch on identical copies of the
caches, within the attention tolerance the other tests use (maxrel 2e-3).
"""
import numpy as np
import pytest
import torch

import oracle as O
from roaster_b200 import synth
from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _slots(lens, extra):
    out = []
    for i, L in enumerate(lens):
        d = synth.attn_decode_inputs(seed=700 + i, length=L)
        kc = torch.zeros(L + extra, 2, 256, dtype=torch.float16, device="cuda")
        vc = torch.zeros_like(kc)
        if L:
            kc[:L] = dev(d["k_cache"])
            vc[:L] = dev(d["v_cache"])
        out.append({"d": d, "kc": kc, "vc": vc})
    return out


def _jobs(rb, slots, tensors, outs, step):
    jobs = []
    for s, t, o in zip(slots, tensors, outs):
        L = s["d"]["length"] + step
        jobs.append(rb.attn_job(t["q"][step], t["gate"][step], t["kn"][step], t["vn"][step],
                                t["qn"], t["kw"], s["kc"], s["vc"], L, L, o))
    return jobs


def test_noalloc_matches_allocating_entry_point_two_calls(rb):
    lens = [1, 500, 4097, 33, 12000, 0, 2048, 70, 30000]
    a_slots = _slots(lens, extra=4)
    b_slots = [{"d": s["d"], "kc": s["kc"].clone(), "vc": s["vc"].clone()} for s in a_slots]
    rng = np.random.default_rng(77)
    tensors = []
    for s in a_slots:
        d = s["d"]
        tensors.append({"q": dev(rng.standard_normal((2, 16, 256)).astype(np.float32)),
                        "gate": dev(rng.standard_normal((2, 16, 256)).astype(np.float32)),
                        "kn": dev(rng.standard_normal((2, 2, 256)).astype(np.float32)),
                        "vn": dev(rng.standard_normal((2, 2, 256)).astype(np.float32)),
                        "qn": dev(d["q_norm"]), "kw": dev(d["k_norm"])})
    n = len(lens)
    for step in range(2):                               # two calls in a row
        out_a = torch.zeros(n, 16, 256, device="cuda")
        out_b = torch.zeros(n, 16, 256, device="cuda")
        rb.attn_decode_batch(_jobs(rb, a_slots, tensors, out_a, step))
        rb.attn_decode_batch_noalloc(_jobs(rb, b_slots, tensors, out_b, step))
        rb.synchronize()
        a, b = host(out_a), host(out_b)
        assert np.isfinite(b).all()
        assert O.maxrel(b, a) <= TOL, (step, O.maxrel(b, a))
        for sa, sb in zip(a_slots, b_slots):
            L = sa["d"]["length"] + step
            assert np.array_equal(host(sa["kc"][: L + 1]), host(sb["kc"][: L + 1]))
            assert np.array_equal(host(sa["vc"][: L + 1]), host(sb["vc"][: L + 1]))


def test_noalloc_rejects_more_than_64_slots(rb):
    lens = [16] * 65
    slots = _slots(lens, extra=2)
    t = {"q": torch.zeros(1, 16, 256, device="cuda"), "gate": torch.zeros(1, 16, 256, device="cuda"),
         "kn": torch.zeros(1, 2, 256, device="cuda"), "vn": torch.zeros(1, 2, 256, device="cuda"),
         "qn": torch.ones(256, device="cuda"), "kw": torch.ones(256, device="cuda")}
    out = torch.zeros(65, 16, 256, device="cuda")
    with pytest.raises(RuntimeError, match="64"):
        rb.attn_decode_batch_noalloc(_jobs(rb, slots, [t] * 65, out, 0))
