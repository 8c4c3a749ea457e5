"""Generate the golden fixtures in this folder from the REFERENCE'S OWN CPU CODE.

Run in a container that has the reference sources (oracle/Makefile compiles them into
oracle/_ref/libroaster_ref.so):   python tests/golden/make_golden.py

Inputs are regenerated from seeds by roaster_b200.synth; each fixture stores a SHA-256 of its
inputs so a change in the generator is caught instead of silently comparing different data.
Outputs are stored in full (float32) except where noted.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from roaster_b200 import synth  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def decode_case():
    d = synth.attn_decode_inputs(seed=0, length=512)
    return d, digest(d["q"], d["gate"], d["k_new"], d["v_new"], d["q_norm"], d["k_norm"],
                     d["k_cache"], d["v_cache"])


def delta_case():
    state = synth.delta_state(seed=11, layers=1)[0]
    seq = synth.delta_sequence(seed=12, steps=16, layers=1)
    return state, seq, digest(state, *[seq[k] for k in ("q", "k", "v", "g", "beta")])


def prefill_case():
    d = synth.prefill_inputs(seed=21, T=12, kbase=50)
    return d, digest(d["q"], d["gate"], d["k"], d["v"], d["q_norm"], d["k_norm"], d["k_cache"],
                     d["v_cache"])


def main():
    oracle.build()
    assert oracle.have_ref(), "reference build missing: the golden vectors must come from it"
    d, dg = decode_case()
    out, ka, va = oracle.attn_decode(d["q"], d["gate"], d["k_new"], d["v_new"], d["q_norm"],
                                     d["k_norm"], d["k_cache"], d["v_cache"], 512, 512, impl="ref")
    np.savez(os.path.join(HERE, "attn_decode_cfg0.npz"), out=out, k_app=ka, v_app=va,
             digest=np.array(dg))

    state, seq, dg = delta_case()
    st = state.copy()
    outs = []
    for t in range(16):
        outs.append(oracle.delta_step(st, seq["q"][t, 0], seq["k"][t, 0], seq["v"][t, 0],
                                      seq["g"][t, 0], seq["beta"][t, 0], impl="ref"))
    np.savez(os.path.join(HERE, "delta_16steps.npz"), out_last=outs[-1], out_first=outs[0],
             state_heads_0_31=st[[0, 31]], state_sum=np.array(st.astype(np.float64).sum()),
             state_abs_sum=np.array(np.abs(st.astype(np.float64)).sum()), digest=np.array(dg))

    d, dg = prefill_case()
    out, ka, va = oracle.attn_prefill(d["q"], d["gate"], d["k"], d["v"], d["q_norm"], d["k_norm"],
                                      d["k_cache"], d["v_cache"], 50, 300, impl="ref")
    np.savez(os.path.join(HERE, "attn_prefill_t12.npz"), out=out, k_app=ka, v_app=va,
             digest=np.array(dg))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
