"""Failure handling without a GPU fault: a kernel whose bounded wait can never complete gives
up, records the timeout in the device error word and returns; the error surfaces on the host and
the context keeps serving real work afterwards."""
import numpy as np
import pytest
import torch

import oracle as O
from roaster_b200 import synth
from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu


def _decode_once(rb):
    d = synth.attn_decode_inputs(seed=0, length=512, position=512)
    kc = torch.zeros(600, 2, 256, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    kc[:512] = dev(d["k_cache"])
    vc[:512] = dev(d["v_cache"])
    q, g, kn, vn = dev(d["q"]), dev(d["gate"]), dev(d["k_new"]), dev(d["v_new"])
    qn, knw = dev(d["q_norm"]), dev(d["k_norm"])
    out = torch.zeros(16, 256, device="cuda")
    rb.attn_decode_batch([rb.attn_job(q, g, kn, vn, qn, knw, kc, vc, 512, 512, out)])
    rb.synchronize()
    ref, _, _ = O.attn_decode(d["q"], d["gate"], d["k_new"], d["v_new"], d["q_norm"], d["k_norm"],
                              d["k_cache"], d["v_cache"], 512, 512)
    return O.maxrel(host(out), ref)


def test_bounded_wait_times_out_and_context_survives(rb, oracle_lib):
    assert _decode_once(rb) < 2e-3
    bits = rb.lib().kernel_cuda_wait_probe(2_000_000)        # ~1 ms at B200 clocks
    assert bits == 1, bits                                    # kErrWaitTimeout, nothing else
    rb.synchronize()                                          # the word was cleared
    assert _decode_once(rb) < 2e-3                            # the context still works


def test_wait_probe_rejects_bad_budget(rb):
    assert rb.lib().kernel_cuda_wait_probe(0) == -1
    assert "budget" in rb.last_error()
