"""Device attention window (KernelKvWindow) against the reference's own kvwindow.c + kvspill.c
(compiled from its sources into oracle/_ref and driven through a Model rig): the same random
sequences of appends (kvw_ensure_room first, as forward_impl and prefill_chunk do), evictions,
restores, rollbacks to earlier snapshots and context changes, with the window state and every
K/V row compared after each operation. Rows are f16 values, so the device window (f16) and the
reference (fp32) must agree exactly, across spills to a file and to host memory."""
import ctypes as C
import os

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


class DevWindow:
    def __init__(self, rb, layers, ctx, slide, keep, pin, path):
        self.rb, self.L = rb, rb.lib()
        self.h = self.L.kernel_kvw_create(layers, ctx, int(slide), keep, pin, path.encode())
        assert self.h, rb.last_error()
        self.layers = layers

    def append(self, k, v):
        n = k.shape[1]
        if self.L.kernel_kvw_ensure_room(self.h, n) != 0:
            return -1
        at = self.L.kernel_kvw_len(self.h)
        for a in range(self.layers):
            for src, ptr in ((k[a], self.L.kernel_kvw_k(self.h, a)), (v[a], self.L.kernel_kvw_v(self.h, a))):
                h16 = np.ascontiguousarray(src.astype(np.float16))
                dst = ptr + at * 512 * 2
                self.rb.check(self.L.kernel_cuda_upload(C.c_void_p(dst), h16.ctypes.data_as(C.c_void_p), h16.nbytes),
                              "upload")
        return self.L.kernel_kvw_appended(self.h, n)

    def evict(self, n):
        return self.L.kernel_kvw_evict(self.h, n)

    def restore(self, n):
        return self.L.kernel_kvw_restore(self.h, n)

    def rollback(self, p0, s0):
        return self.L.kernel_kvw_rollback(self.h, p0, s0)

    def set_context(self, ctx):
        return self.L.kernel_kvw_set_context(self.h, ctx)

    def state(self):
        return {k: int(getattr(self.L, "kernel_kvw_" + ("spilled" if k == "spilled" else k))(self.h))
                for k in ("len", "spilled", "head", "max_chunk", "position", "context")}

    def read(self, a):
        n = self.L.kernel_kvw_len(self.h)
        out = []
        for ptr in (self.L.kernel_kvw_k(self.h, a), self.L.kernel_kvw_v(self.h, a)):
            h16 = np.zeros((n, 512), np.float16)
            if n:
                self.rb.check(self.L.kernel_cuda_download(h16.ctypes.data_as(C.c_void_p), C.c_void_p(ptr), h16.nbytes),
                              "download")
            out.append(h16.astype(np.float32))
        return out

    def close(self):
        self.L.kernel_kvw_destroy(self.h)


def _compare(ref, dev, what):
    rs, ds = ref.state(), dev.state()
    assert rs == ds, (what, rs, ds)
    for a in (0, 4, ref.layers - 1):
        rk, rv = ref.read(a)
        dk, dv = dev.read(a)
        assert np.array_equal(rk, dk), (what, a, "K")
        assert np.array_equal(rv, dv), (what, a, "V")


def _run(rb, tmp_path, seed, ctx, slide, keep, pin, use_file, steps, script=None):
    """Random operations (or the given `script` of (op, arg) pairs) on both windows."""
    if not O.have_ref():
        pytest.skip("reference build (oracle/_ref) not present")
    rng = np.random.default_rng(seed)
    ref = O.RefWindow(ctx, slide, keep, pin, str(tmp_path / f"ref{seed}.kv"))
    dev = DevWindow(rb, ref.layers, ctx, slide, keep, pin, str(tmp_path / f"dev{seed}.kv") if use_file else "")
    snaps = []
    seen = {"spilled": 0, "failed": 0}
    ops = script if script is not None else [None] * steps
    try:
        for step, planned in enumerate(ops):
            if planned is None:
                op = rng.choice(["append", "append", "append", "evict", "restore", "rollback", "context"],
                                p=[0.3, 0.15, 0.1, 0.1, 0.12, 0.13, 0.1])
                arg = None
            else:
                op, arg = planned
            if op == "append":
                n = arg if arg is not None else int(rng.integers(1, max(2, ctx // 3)))
                k = rng.standard_normal((ref.layers, n, 512)).astype(np.float16).astype(np.float32)
                v = rng.standard_normal((ref.layers, n, 512)).astype(np.float16).astype(np.float32)
                r1, r2 = ref.append(k, v), dev.append(k, v)
                snaps.append((ref.state()["position"], ref.state()["spilled"]))
            elif op == "evict":
                n = arg if arg is not None else int(rng.integers(0, 20))
                r1, r2 = ref.evict(n), dev.evict(n)
            elif op == "restore":
                n = arg if arg is not None else int(rng.integers(0, 20))
                r1, r2 = ref.restore(n), dev.restore(n)
            elif op == "rollback":
                if not snaps:
                    continue
                p0, s0 = snaps[arg if arg is not None else int(rng.integers(0, len(snaps)))]
                r1, r2 = ref.rollback(p0, s0), dev.rollback(p0, s0)
                snaps = [s for s in snaps if s[0] <= p0]
            else:
                new = arg if arg is not None else int(rng.integers(max(8, ctx // 4), 2 * ctx))
                r1, r2 = ref.set_context(new), dev.set_context(new)
            assert (r1 == 0) == (r2 == 0), (step, op, r1, r2)
            _compare(ref, dev, (step, op))
            seen["spilled"] = max(seen["spilled"], ref.state()["spilled"])
            seen["failed"] += r1 != 0
    finally:
        ref.close()
        dev.close()
    return seen


@pytest.mark.parametrize("seed,keep,pin,use_file", [(1, 16, 0, True), (2, 0, 0, False), (3, 8, 40, True),
                                                    (4, 64, 0, False)])
def test_sliding_window_matches_reference(rb, tmp_path, seed, keep, pin, use_file):
    seen = _run(rb, tmp_path, seed, ctx=160, slide=True, keep=keep, pin=pin, use_file=use_file, steps=60)
    assert seen["spilled"] > 0                  # the window slid and used the store


def test_without_sliding(rb, tmp_path):
    """Sliding off: a full window rejects appends; evictions still go to the store."""
    _run(rb, tmp_path, 5, ctx=96, slide=False, keep=16, pin=0, use_file=True, steps=40)


def test_long_window_large_moves(rb, tmp_path):
    """A 20k-token window: a slide evicts ~5k rows and moves a ~10k-row tail by less than a move
    block (scratch-staged), restores of a few tokens shift the whole tail, a large eviction moves
    it in direct blocks, then rollback, growth (refill from the store) and shrinking."""
    script = [("append", 15000), ("append", 8000), ("restore", 3), ("append", 400), ("evict", 9000),
              ("restore", 2500), ("append", 6000), ("rollback", 2), ("context", 30000), ("context", 12000),
              ("append", 5000)]
    seen = _run(rb, tmp_path, 6, ctx=20000, slide=True, keep=64, pin=0, use_file=True, steps=0, script=script)
    assert seen["spilled"] > 5000
