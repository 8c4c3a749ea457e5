"""The state file ("RSTA" v2, reference src/state.c:7-81) with the KV windows and DeltaNet
states resident on the device: the writer and reader below are state.c's model_state_save /
model_state_load with their KV memcpys replaced by kernel_cuda_download_f16_f32 /
kernel_cuda_upload_f32_f16 and their state memcpys by kernel_cuda_download / kernel_cuda_upload
(the edit state.c needs once its buffers live on the device). Checked against the reference's
own model_state_load and model_state_save (oracle/_ref, state.c compiled from its sources): a
file written from device
state loads in the reference bit for bit, a file the reference writes restores the device state
bit for bit, and decoding continues from a restored state exactly as from the original."""
import os
import struct

import numpy as np
import pytest
import torch

import oracle as O
from roaster_b200 import synth
from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu
MAGIC, VERSION = 0x41545352, 2


def _write(lib, path, ctx, position, layers, kv, states, conv):
    with open(path, "wb") as f:
        f.write(struct.pack("<IIIIQQ", MAGIC, VERSION, len(layers), 0, ctx, position))
        for l, att in enumerate(layers):
            if att:
                kc, vc, n = kv[l]
                f.write(struct.pack("<Q", n))
                for t in (kc, vc):
                    buf = np.zeros(n * 512, np.float32)
                    assert lib.kernel_cuda_download_f16_f32(buf.ctypes.data, t.data_ptr(), n * 512) == 0
                    f.write(buf.tobytes())
            else:
                buf = np.zeros(32 * 128 * 128, np.float32)
                assert lib.kernel_cuda_download(buf.ctypes.data, states[l].data_ptr(), buf.nbytes) == 0
                f.write(buf.tobytes())
                f.write(np.ascontiguousarray(conv[l], np.float32).tobytes())


def _read(lib, path, layers, kv, states, conv):
    with open(path, "rb") as f:
        magic, version, nl, _, ctx, position = struct.unpack("<IIIIQQ", f.read(32))
        assert (magic, version, nl) == (MAGIC, VERSION, len(layers))
        lens = set()
        for l, att in enumerate(layers):
            if att:
                (n,) = struct.unpack("<Q", f.read(8))
                kc, vc, _ = kv[l]
                assert n <= kc.shape[0]
                for t in (kc, vc):
                    buf = np.frombuffer(f.read(n * 512 * 4), np.float32).copy()
                    assert lib.kernel_cuda_upload_f32_f16(t.data_ptr(), buf.ctypes.data, n * 512) == 0
                kv[l] = (kc, vc, n)
                lens.add(n)
            else:
                buf = np.frombuffer(f.read(32 * 128 * 128 * 4), np.float32).copy()
                assert lib.kernel_cuda_upload(states[l].data_ptr(), buf.ctypes.data, buf.nbytes) == 0
                conv[l] = np.frombuffer(f.read(3 * 8192 * 4), np.float32).reshape(3, 8192).copy()
    assert lens == {position}                      # no spill store: the window holds every token
    return position


def _device_model(ctx, L, seed, layers):
    rng = np.random.default_rng(seed)
    kv, states, conv = {}, {}, {}
    for l, att in enumerate(layers):
        if att:
            kc = torch.zeros(ctx, 2, 256, dtype=torch.float16, device="cuda")
            vc = torch.zeros_like(kc)
            kc[:L] = dev(rng.standard_normal((L, 2, 256)).astype(np.float16))
            vc[:L] = dev(rng.standard_normal((L, 2, 256)).astype(np.float16))
            kv[l] = (kc, vc, L)
        else:
            states[l] = dev((0.02 * rng.standard_normal((32, 128, 128))).astype(np.float32))
            conv[l] = rng.standard_normal((3, 8192)).astype(np.float32)
    return kv, states, conv


def _step(rb, kv, states, inputs, layers):
    """One decode token on every attention layer (appending) and every DeltaNet layer."""
    d, dn = inputs
    att = [l for l, a in enumerate(layers) if a]
    out = torch.zeros(len(att), 16, 256, device="cuda")
    rb.attn_decode_batch([rb.attn_job(d["q"], d["gate"], d["k_new"], d["v_new"], d["q_norm"], d["k_norm"],
                                      kv[l][0], kv[l][1], kv[l][2], kv[l][2], out[i]) for i, l in enumerate(att)])
    rec = [l for l, a in enumerate(layers) if not a]
    dout = torch.zeros(len(rec), 32, 128, device="cuda")
    rb.deltanet_step_batch([rb.delta_job(states[l], dn["q"][0], dn["k"][0], dn["v"][0], dn["g"][0], dn["beta"][0],
                                         dout[i]) for i, l in enumerate(rec)])
    rb.synchronize()
    for l in att:
        kv[l] = (kv[l][0], kv[l][1], kv[l][2] + 1)
    return host(out), host(dout)


def _inputs(seed):
    d = synth.attn_decode_inputs(seed=seed, length=0)
    dn = synth.delta_step_inputs(np.random.default_rng(seed + 1), 1)
    return ({k: dev(d[k]) for k in ("q", "gate", "k_new", "v_new", "q_norm", "k_norm")},
            {k: dev(v) for k, v in dn.items()})


def test_device_state_round_trips_through_the_reference_format(rb, oracle_lib, tmp_path):
    lib = rb.lib()
    ctx, L = 300, 257
    ref = O.RefState(ctx)
    layers = [ref.is_attention(l) for l in range(ref.layers)]
    kv, states, conv = _device_model(ctx, L, 31, layers)
    _step(rb, kv, states, _inputs(32), layers)              # device-computed content in the state
    pos = L + 1

    # device -> file -> the reference's own loader
    a = str(tmp_path / "a.rsta")
    _write(lib, a, ctx, pos, layers, kv, states, conv)
    assert ref.load(a) == 0 and ref.position() == pos
    for l, att in enumerate(layers):
        if att:
            k, v = ref.kv(l)
            assert ref.length(l) == pos
            assert np.array_equal(k[:pos], host(kv[l][0][:pos]).reshape(pos, 512).astype(np.float32))
            assert np.array_equal(v[:pos], host(kv[l][1][:pos]).reshape(pos, 512).astype(np.float32))
        else:
            st, cv = ref.ssm(l)
            assert np.array_equal(st, host(states[l])) and np.array_equal(cv, conv[l])

    # the reference's own writer -> file -> fresh device buffers
    b = str(tmp_path / "b.rsta")
    assert ref.save(b) == 0
    assert os.path.getsize(a) == os.path.getsize(b)
    kv2, states2, conv2 = _device_model(ctx, 0, 99, layers)
    assert _read(lib, b, layers, kv2, states2, conv2) == pos
    for l, att in enumerate(layers):
        if att:
            assert kv2[l][2] == pos
            assert torch.equal(kv2[l][0][:pos], kv[l][0][:pos]) and torch.equal(kv2[l][1][:pos], kv[l][1][:pos])
        else:
            assert torch.equal(states2[l], states[l]) and np.array_equal(conv2[l], conv[l])
    ref.close()

    # decoding continues from the restored state exactly as from the original
    nxt = _inputs(40)
    o1, d1 = _step(rb, kv, states, nxt, layers)
    o2, d2 = _step(rb, kv2, states2, nxt, layers)
    assert np.array_equal(o1, o2) and np.array_equal(d1, d2)


def test_f16_transfers_round_to_nearest_even(rb):
    """kernel_cuda_upload_f32_f16 rounds like numpy's float16 conversion (round to nearest even,
    overflow to inf) and kernel_cuda_download_f16_f32 widens exactly, over more than one staged
    piece (5M values)."""
    lib = rb.lib()
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(5_000_000) * np.exp(rng.uniform(-20, 12, 5_000_000))).astype(np.float32)
    d = torch.empty(x.size, dtype=torch.float16, device="cuda")
    assert lib.kernel_cuda_upload_f32_f16(d.data_ptr(), x.ctypes.data, x.size) == 0
    assert np.array_equal(host(d).view(np.uint16), x.astype(np.float16).view(np.uint16))
    back = np.zeros(x.size, np.float32)
    assert lib.kernel_cuda_download_f16_f32(back.ctypes.data, d.data_ptr(), x.size) == 0
    assert np.array_equal(back, x.astype(np.float16).astype(np.float32))
