#!/usr/bin/env python
"""Hybrid-attention decode benchmark on B200.

One step = one decode token for every one of the 64 slots: per slot one gated-attention layer
(16 q / 2 kv heads, d 256, q/k RMSNorm, partial RoPE, sigmoid gate) over an f16 KV window of
L ~ U[1k, 32k] tokens that grows by the appended token each step, plus 3 Gated DeltaNet layers
(32 x 128 x 128 fp32 state each). The 64 slots are sharded across the N GPUs (longest windows
first onto the least-loaded GPU, equal slot counts) with no communication: strong scaling, the
configuration as stated. A secondary object keeps 64 slots per GPU (weak scaling) at N > 1.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

The device-timed `value` runs both kernels on resident inputs (CUDA events on the launching
stream, max over ranks). `e2e` runs the same step through the host-buffer C-ABI entry points
(inputs copied host->device and outputs device->host inside the timed region). `parity` checks
one more step of the same batch (a sample of slots, after the timed region) against the
reference's own CPU code. `cpu_baseline` and `--impl reference` time the reference's own CPU code
(compiled from its sources into oracle/_ref) on this host's cores. Inputs are seeded synthetic
data (no dataset exists for the path); the KV windows (2.2 GB) and states (0.4 GB) exceed the
126 MB L2, so no flush is needed between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SLOTS = 64                      # config 2's slots (global)
DN_LAYERS = 3
METRIC = "hybrid-attn decode tok/s (config 2: 64 slots sharded over the GPUs, 1 gated-attn + 3 DeltaNet layers)"
# DRAM bytes per launch / algorithmic bytes for the decode-attention kernel, from one ncu capture
# of a 64-slot launch with windows U[1024, 4096] (dram__bytes_read 336.07 MB + write 6.81 MB for
# 338.31 MB algorithmic). Traffic grows with the KV positions streamed, so the ratio scales to
# the full launch.
ATTN_TRAFFIC_RATIO = (336.069888e6 + 6.806784e6) / 338309120
CPU_BUDGET_S = 90.0             # bound on the reference arm's timed CPU work


def args_parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the parity check of the timed batch")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-3 prefill measurement")
    ap.add_argument("--prefill-steps", type=int, default=5)
    ap.add_argument("--no-long", action="store_true", help="skip the config-4 long-context decode")
    ap.add_argument("--long-steps", type=int, default=30)
    ap.add_argument("--long-window", type=int, default=262144)
    ap.add_argument("--no-proj", action="store_true", help="skip the k-quant projection measurement")
    ap.add_argument("--proj-steps", type=int, default=20)
    ap.add_argument("--step-rounds", type=int, default=10, help="timed rounds of the batched-step measurement")
    ap.add_argument("--no-shards", action="store_true", help="skip the per-GPU shard sweep at N=1")
    ap.add_argument("--no-recurrent", action="store_true", help="skip the config-1 recurrent decode (rank 0)")
    ap.add_argument("--recurrent-steps", type=int, default=RECUR_STEPS)
    ap.add_argument("--kv-lo", type=int, default=1024, help="smallest slot window (config 2: 1024)")
    ap.add_argument("--kv-hi", type=int, default=32768, help="largest slot window (config 2: 32768)")
    ap.add_argument("--cpu-json", help=argparse.SUPPRESS)       # internal: CPU leg in a subprocess
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def slot_lengths(seed: int = 1000, lo: int = 1024, hi: int = 32768, n: int = SLOTS):
    from roaster_b200 import synth
    return [int(x) for x in synth.slot_lengths(seed, n, lo, hi)]


def assign_slots(lens, world: int):
    """Shard the slots over `world` GPUs: equal slot counts (the DeltaNet work per slot is fixed),
    windows longest first onto the GPU with the least attention work so far. Returns each rank's
    slot indices in ascending order."""
    per = -(-len(lens) // world)
    load, cnt, out = [0] * world, [0] * world, [[] for _ in range(world)]
    for s in sorted(range(len(lens)), key=lambda i: (-lens[i], i)):
        r = min((r for r in range(world) if cnt[r] < per), key=lambda r: (load[r], r))
        out[r].append(s)
        cnt[r] += 1
        load[r] += lens[s]
    return [sorted(x) for x in out]


def config2_desc(world: int, a) -> dict:
    """The `config` object of the config-2 line; both arms print the same one."""
    return {"workload": "config 2: batched hybrid-layer decode, 64 slots sharded over the GPUs",
            "global_slots": SLOTS, "slots_per_gpu": -(-SLOTS // world),
            "kv_len": f"U[{a.kv_lo}, {a.kv_hi}] per slot (seed 1000), +1 per step",
            "deltanet_layers_per_slot": DN_LAYERS,
            "parallelism": f"slot-sharded x{world} (balanced by window length, no collective)",
            "l2": "inputs (>2.5 GB at N=1) exceed L2; no flush needed"}


# ------------------------------------------------------------------------------ CPU legs (subprocess)

def cpu_reference(lens, steps: int, warmup: int, threads: int, budget_s: float) -> dict:
    """Time the reference's own CPU path (oracle/_ref): one step = every slot once, in turn as the
    reference's step lock serves them (slots.c:864-891): its full_attention over the slot's
    window (the four projection matvecs it also runs are timed separately and subtracted) + 3
    recurrent_delta_step calls; windows grow by one token per step as on the GPU. Runs the
    warm-up steps, then timed steps until `steps` or `budget_s` of CPU work."""
    import ctypes as C

    import numpy as np

    import oracle
    lib = oracle.ref_lib()
    rng = np.random.default_rng(5)
    cap = max(lens) + steps + warmup + 2
    qn = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    fp = C.POINTER(C.c_float)
    ctx = lib.ref_decode_ctx_new(cap, qn.ctypes.data_as(fp), kn.ctypes.data_as(fp))
    if not ctx:
        raise RuntimeError("reference rig allocation failed")
    kw = np.ctypeslib.as_array(lib.ref_decode_ctx_k(ctx), shape=(cap * 512,))
    vw = np.ctypeslib.as_array(lib.ref_decode_ctx_v(ctx), shape=(cap * 512,))
    kw[:] = rng.standard_normal(cap * 512, dtype=np.float32).astype(np.float16).astype(np.float32)
    vw[:] = rng.standard_normal(cap * 512, dtype=np.float32).astype(np.float16).astype(np.float32)
    state = (0.02 * rng.standard_normal((DN_LAYERS, 32, 128, 128), dtype=np.float32)).astype(np.float32)
    from roaster_b200 import synth
    dn = synth.delta_step_inputs(rng, DN_LAYERS)
    out = np.zeros((32, 128), np.float32)
    args = [np.ascontiguousarray(dn[k]) for k in ("q", "k", "v", "g", "beta")]
    # projection matvecs full_attention runs (W_q 8192x2048, W_k, W_v 512x2048, W_o 2048x4096)
    pt = []
    for _ in range(5):
        t0 = time.perf_counter()
        lib.ref_decode_ctx_projections(ctx)
        pt.append(time.perf_counter() - t0)
    proj = statistics.median(pt)

    def one_step(i):
        tot = 0.0
        for L0 in lens:
            L = L0 + i
            t0 = time.perf_counter()
            if lib.ref_decode_ctx_step(ctx, L, L) != 0:
                raise RuntimeError("reference full_attention failed")
            for l in range(DN_LAYERS):
                lib.ref_delta_step(state[l].ctypes.data_as(fp),
                                   *[a[l].ctypes.data_as(fp) for a in args], out.ctypes.data_as(fp))
            tot += max(time.perf_counter() - t0 - proj, 1e-9)
        return tot

    est = None
    for i in range(warmup):
        est = one_step(i)
    n_timed = steps
    if est is not None:
        n_timed = max(1, min(steps, int(budget_s / max(est, 1e-9))))
    total, done = 0.0, 0
    for i in range(n_timed):
        total += one_step(warmup + i)
        done += 1
        if est is None and total * (i + 2) / (i + 1) > budget_s:
            break
    lib.ref_decode_ctx_free(ctx)
    return {"tok_s": len(lens) * done / total, "seconds": total, "steps": done, "slots": len(lens),
            "threads": threads, "projection_ms_subtracted": proj * 1e3}


def cpu_parity(path: str) -> dict:
    """Check a sample of one config-2 step of the GPU batch (saved by the GPU arm) against the
    reference's own CPU code: full_attention's math per slot (oracle impl "ref") on the same f16
    window, and recurrent_delta_step on the saved states."""
    import numpy as np

    import oracle as O
    z = np.load(path)
    impl = "ref" if O.have_ref() else "port"
    attn, st_err, out_err = [], [], []
    for i in range(int(z["n"])):
        L = int(z[f"len{i}"])
        ref, ka, va = O.attn_decode(z[f"q{i}"], z[f"gate{i}"], z[f"kn{i}"], z[f"vn{i}"], z["qn"], z["kw"],
                                    z[f"kc{i}"], z[f"vc{i}"], L, L, impl=impl)
        attn.append(O.maxrel(z[f"out{i}"], ref))
        for l in range(DN_LAYERS):
            st = np.ascontiguousarray(z[f"st{i}"][l])
            o = O.delta_step(st, *[np.ascontiguousarray(z[f"d{k}{i}"][l]) for k in ("q", "k", "v", "g", "beta")],
                             impl=impl)
            st_err.append(O.maxrel(z[f"st_after{i}"][l], st))
            out_err.append(O.maxrel(z[f"dout{i}"][l], o))
    return {"impl": impl, "attn_maxrel": max(attn), "state_maxrel": max(st_err), "deltanet_out_maxrel": max(out_err),
            "slots": [int(z[f"len{i}"]) for i in range(int(z["n"]))]}


PREFILL_CHUNK = 256             # the reference's PF_MAX_T (model.c:1401)


def cpu_prefill(threads: int) -> dict:
    """The reference's own prefill path for ONE config-3 prompt of 8192 tokens on the host:
    pf_attention (model.c:1536-1602) chunk by chunk, 256 tokens each, and the delta_head
    recurrence of pf_ssm (model.c:1644-1658) over all 8192 tokens for one DeltaNet layer.
    Attention: a chunk's attention work is proportional to the keys its rows attend to
    (start + 128.5 on average), while its projections and per-token prep do not depend on the
    start. So the first and the last chunk are timed, their difference gives the time per
    attended key, and the 32 chunks' attention time is that rate times the keys they attend to
    (sum over chunks of start + 128.5). The result is extrapolated x8 to the configuration's 8
    prompts (stated in the sample)."""
    import ctypes as C

    import numpy as np

    import oracle
    from roaster_b200 import synth
    lib = oracle.ref_lib()
    T = 8192
    rng = np.random.default_rng(6)
    qn = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    fp = C.POINTER(C.c_float)
    ctx = lib.ref_prefill_ctx_new(T, qn.ctypes.data_as(fp), kn.ctypes.data_as(fp))
    if not ctx:
        raise RuntimeError("reference prefill rig allocation failed")
    kw = np.ctypeslib.as_array(lib.ref_prefill_ctx_k(ctx), shape=(T * 512,))
    vw = np.ctypeslib.as_array(lib.ref_prefill_ctx_v(ctx), shape=(T * 512,))
    kw[:] = rng.standard_normal(T * 512, dtype=np.float32)
    vw[:] = rng.standard_normal(T * 512, dtype=np.float32)
    C_ = PREFILL_CHUNK
    nchunks = T // C_

    def timed(fn):
        t0 = time.perf_counter()
        if fn() != 0:
            raise RuntimeError("reference prefill call failed")
        return time.perf_counter() - t0

    timed(lambda: lib.ref_prefill_ctx_chunk(ctx, C_, 0, 0))                   # warm-up
    last_kb = T - C_
    first = statistics.median([timed(lambda: lib.ref_prefill_ctx_chunk(ctx, C_, 0, 0)) for _ in range(3)])
    last = statistics.median([timed(lambda: lib.ref_prefill_ctx_chunk(ctx, C_, last_kb, last_kb))
                              for _ in range(2)])
    proj = statistics.median([timed(lambda: lib.ref_prefill_ctx_projections(ctx, C_)) for _ in range(2)])
    per_key = (last - first) / last_kb                 # seconds per attended key of a chunk
    keys = sum(c * C_ + (C_ + 1) / 2 for c in range(nchunks))
    attn_s = per_key * keys
    lib.ref_prefill_ctx_free(ctx)
    del kw, vw
    p = synth.delta_prompt(7, T)
    st = np.zeros((32, 128, 128), np.float32)
    out = np.zeros((T, 32, 128), np.float32)
    t0 = time.perf_counter()
    lib.ref_delta_prefill(st.ctypes.data_as(fp), T, *[np.ascontiguousarray(p[k]).ctypes.data_as(fp)
                                                       for k in ("q", "k", "v", "g", "beta")],
                          out.ctypes.data_as(fp))
    dn_s = time.perf_counter() - t0
    return {"attn_s_per_prompt": attn_s, "deltanet_s_per_prompt": dn_s, "first_chunk_s": first,
            "last_chunk_s": last, "projections_s_per_chunk": proj, "threads": threads}


def cpu_long(window: int, slots: int, threads: int) -> dict:
    """The reference's own decode for config 4: one slot-step of full_attention over a window of
    `window` cached tokens (projection matvecs subtracted) + 3 recurrent_delta_step, timed twice;
    a step serves all `slots` slots in turn (the reference's step lock)."""
    import ctypes as C

    import numpy as np

    import oracle
    lib = oracle.ref_lib()
    rng = np.random.default_rng(8)
    cap = window + 4
    qn = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    fp = C.POINTER(C.c_float)
    ctx = lib.ref_decode_ctx_new(cap, qn.ctypes.data_as(fp), kn.ctypes.data_as(fp))
    if not ctx:
        raise RuntimeError("reference rig allocation failed")
    kw = np.ctypeslib.as_array(lib.ref_decode_ctx_k(ctx), shape=(cap * 512,))
    vw = np.ctypeslib.as_array(lib.ref_decode_ctx_v(ctx), shape=(cap * 512,))
    kw[:] = rng.standard_normal(cap * 512, dtype=np.float32)
    vw[:] = rng.standard_normal(cap * 512, dtype=np.float32)
    from roaster_b200 import synth
    dn = synth.delta_step_inputs(rng, DN_LAYERS)
    state = (0.02 * rng.standard_normal((DN_LAYERS, 32, 128, 128), dtype=np.float32)).astype(np.float32)
    out = np.zeros((32, 128), np.float32)
    args = [np.ascontiguousarray(dn[k]) for k in ("q", "k", "v", "g", "beta")]
    proj = statistics.median([(lambda t0: (lib.ref_decode_ctx_projections(ctx), time.perf_counter() - t0)[1])(
        time.perf_counter()) for _ in range(3)])
    ts = []
    for i in range(3):
        t0 = time.perf_counter()
        if lib.ref_decode_ctx_step(ctx, window + i, window + i) != 0:
            raise RuntimeError("reference full_attention failed")
        for l in range(DN_LAYERS):
            lib.ref_delta_step(state[l].ctypes.data_as(fp), *[x[l].ctypes.data_as(fp) for x in args],
                               out.ctypes.data_as(fp))
        ts.append(time.perf_counter() - t0 - proj)
    lib.ref_decode_ctx_free(ctx)
    slot_s = statistics.median(ts[1:])
    return {"slot_step_s": slot_s, "tok_s": 1.0 / slot_s, "slots": slots, "threads": threads,
            "projection_ms_subtracted": proj * 1e3}


RECUR_LAYERS = 30               # config 1: one slot, 30 Gated DeltaNet layers
RECUR_STEPS = 1024              # ... stepped 1024 times in sequence


def cpu_recurrent(threads: int, steps: int) -> dict:
    """The reference's own config-1 decode: per step, recurrent_delta_step (kernels.c, through
    oracle/_ref) for each of the 30 layers of one slot, `steps` timed steps after one warm-up
    step. The step's cost does not depend on the values, so one seeded input set serves every
    step; the states evolve."""
    import ctypes as C

    import numpy as np

    import oracle
    from roaster_b200 import synth
    lib = oracle.ref_lib()
    rng = np.random.default_rng(11)
    dn = synth.delta_step_inputs(rng, RECUR_LAYERS)
    state = (0.02 * rng.standard_normal((RECUR_LAYERS, 32, 128, 128), dtype=np.float32)).astype(np.float32)
    out = np.zeros((32, 128), np.float32)
    fp = C.POINTER(C.c_float)
    args = [np.ascontiguousarray(dn[k]) for k in ("q", "k", "v", "g", "beta")]
    ts = []
    for _ in range(steps + 1):
        t0 = time.perf_counter()
        for l in range(RECUR_LAYERS):
            lib.ref_delta_step(state[l].ctypes.data_as(fp), *[x[l].ctypes.data_as(fp) for x in args],
                               out.ctypes.data_as(fp))
        ts.append(time.perf_counter() - t0)
    step_s = statistics.median(ts[1:])
    return {"step_s": step_s, "tok_s": 1.0 / step_s, "steps": steps, "threads": threads}


def cpu_parity1(path: str) -> dict:
    """Config-1 parity: the sampled layers' whole sequences (saved by the GPU arm) through the
    reference's recurrence (oracle impl "ref": delta_head as pf_ssm runs it, one token at a
    time) from the same initial states; final states and every step's outputs compared."""
    import numpy as np

    import oracle as O
    z = np.load(path)
    impl = "ref" if O.have_ref() else "port"
    st_err, out_err = [], []
    for i in range(int(z["n"])):
        st = np.ascontiguousarray(z[f"st0_{i}"])
        o = O.delta_prefill(st, *[z[f"{k}{i}"] for k in ("q", "k", "v", "g", "beta")], impl=impl)
        st_err.append(O.maxrel(z[f"st_end{i}"], st))
        out_err.append(O.maxrel(z[f"out{i}"], o))
    return {"impl": impl, "state_maxrel": max(st_err), "out_maxrel": max(out_err),
            "layers": [int(x) for x in z["layers"]], "steps": int(z["steps"])}


def cpu_leg(task: str, threads: int | None = None, timeout: int = 1800, native: bool = False, **kw):
    """Run one CPU task in a fresh process (its OpenMP runtime never meets torch's)."""
    threads = threads or os.cpu_count() or 1
    env = dict(os.environ, OMP_NUM_THREADS=str(threads), CUDA_VISIBLE_DEVICES="",
               ROASTER_REF_NATIVE="1" if native else "0")
    spec = json.dumps(dict(kw, task=task, threads=threads))
    out = subprocess.run([sys.executable, os.path.abspath(__file__), "--cpu-json", spec],
                         capture_output=True, text=True, env=env, timeout=timeout)
    if out.returncode != 0:
        raise RuntimeError(f"CPU leg '{task}' failed (rc {out.returncode}): " + out.stderr[-1500:])
    return json.loads(out.stdout.strip().splitlines()[-1])


def cpu_leg_ref(task: str, **kw):
    """The reference CPU leg with the reference's own flags (-march of the GPU host) when that
    build exists and runs here, else the portable build; says which in `build`."""
    import oracle
    if oracle.native_ref_available():
        try:
            r = cpu_leg(task, native=True, **kw)
            r["build"] = f"reference sources, -O3 -march={oracle.native_ref_march()} -fopenmp"
            return r
        except Exception as e:  # e.g. the host CPU lacks an instruction of that -march
            note = f"-march build failed here ({str(e)[:120]}); "
    else:
        note = ""
    r = cpu_leg(task, native=False, **kw)
    r["build"] = note + "reference sources, -O3 -mavx2 -mfma -mf16c -fopenmp (portable)"
    return r


def cpu_main(spec: dict) -> dict:
    t = spec["task"]
    if t == "decode":
        return cpu_reference(spec["lens"], spec["steps"], spec["warmup"], spec["threads"], spec["budget_s"])
    if t == "parity":
        return cpu_parity(spec["path"])
    if t == "prefill":
        return cpu_prefill(spec["threads"])
    if t == "long":
        return cpu_long(spec["window"], spec["slots"], spec["threads"])
    if t == "recurrent":
        return cpu_recurrent(spec["threads"], spec["steps"])
    if t == "parity1":
        return cpu_parity1(spec["path"])
    raise ValueError(t)


# ------------------------------------------------------------------------------ clocks

class ClockSampler:
    FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        import tempfile
        self.path = os.path.join(tempfile.gettempdir(), f"roaster_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), "--query-gpu=" + ",".join(self.FIELDS),
                 "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                c = [x.strip() for x in line.split(",")]
                if len(c) < 9:
                    continue
                try:
                    sm.append(float(c[1]))
                    mx.append(float(c[2]))
                except ValueError:
                    continue
                for n, v in zip(names, c[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.remove(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------ prefill (config 3)

PREFILL_PROMPTS = 8
PREFILL_T = 8192
DN_PREFILL_KERNELS = "deltanet_prefill_kernel"
DN_PREFILL_NOTE = ("each product runs as three f16 MMAs (hi*hi + hi*lo + lo*hi) to keep the fp32 state "
                   "within 1e-4")


def run_prefill(R, torch, dev, stream, steps: int, rank: int):
    """Config 3: 8 prompts x 8192 tokens.
    Attention: bf16 Q/K/V/gate ~ N(0,1), causal gated attention (prep + tcgen05 kernel) into empty
    windows. DeltaNet: one layer's chunked prefill over the same positions, config-1 input
    distributions, from a zero state. Each part device-timed per step; returns
    (attention ms, DeltaNet ms, launches)."""
    from roaster_b200 import synth
    import torch.nn.functional as F
    keep, jobs, djobs = [], [], []
    for p in range(PREFILL_PROMPTS):
        s0 = 100 * (rank + 1) + 16 * p
        q = synth.device_normal(torch, (PREFILL_T, 16, 256), s0, dev, torch.bfloat16)
        g = synth.device_normal(torch, (PREFILL_T, 16, 256), s0 + 1, dev, torch.bfloat16)
        k = synth.device_normal(torch, (PREFILL_T, 2, 256), s0 + 2, dev, torch.bfloat16)
        v = synth.device_normal(torch, (PREFILL_T, 2, 256), s0 + 3, dev, torch.bfloat16)
        qn = 1 + 0.1 * synth.device_normal(torch, (256,), s0 + 5, dev, torch.float32)
        kn = 1 + 0.1 * synth.device_normal(torch, (256,), s0 + 6, dev, torch.float32)
        kc = torch.zeros(PREFILL_T, 2, 256, dtype=torch.float16, device=dev)
        vc = torch.zeros_like(kc)
        out = torch.empty(PREFILL_T, 16, 256, device=dev)
        keep.append((q, g, k, v, qn, kn, kc, vc, out))
        jobs.append(R.KernelAttnPrefillJob(q.data_ptr(), g.data_ptr(), 256, 4096, k.data_ptr(),
                                           v.data_ptr(), qn.data_ptr(), kn.data_ptr(), kc.data_ptr(),
                                           vc.data_ptr(), PREFILL_T, 0, 0, PREFILL_T, out.data_ptr(),
                                           1))
        # DeltaNet layer: q, k L2-normalised per head, v ~ N(0,1), beta = sigmoid(N(0,1)),
        # g = -exp(N(-1, 0.5)) * softplus(N(0,1))
        dq = F.normalize(synth.device_normal(torch, (PREFILL_T, 16, 128), s0 + 7, dev, torch.float32), dim=-1)
        dk = F.normalize(synth.device_normal(torch, (PREFILL_T, 16, 128), s0 + 8, dev, torch.float32), dim=-1)
        dv = synth.device_normal(torch, (PREFILL_T, 32, 128), s0 + 9, dev, torch.float32)
        db = torch.sigmoid(synth.device_normal(torch, (PREFILL_T, 32), s0 + 10, dev, torch.float32))
        dg = -torch.exp(synth.device_normal(torch, (PREFILL_T, 32), s0 + 11, dev, torch.float32, 0.5) - 1.0) \
            * F.softplus(synth.device_normal(torch, (PREFILL_T, 32), s0 + 12, dev, torch.float32))
        dst = torch.zeros(32, 128, 128, device=dev)
        dout = torch.empty(PREFILL_T, 32, 128, device=dev)
        keep.append((dq, dk, dv, db, dg, dst, dout))
        djobs.append(R.delta_prefill_job(dst, dq, dk, dv, dg, db, dout, PREFILL_T))
    arr = (R.KernelAttnPrefillJob * len(jobs))(*jobs)
    darr = (R.KernelDeltaPrefillJob * len(djobs))(*djobs)
    lib = R.lib()
    for _ in range(2):
        if lib.kernel_attn_prefill_batch(arr, len(jobs)) != 0 or \
                lib.kernel_deltanet_prefill_batch(darr, len(djobs)) != 0:
            raise RuntimeError(R.last_error())
    R.synchronize()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    n0 = R.launch_count()
    ta = td = 0.0
    for _ in range(steps):
        ev[0].record(stream)
        lib.kernel_attn_prefill_batch(arr, len(jobs))
        ev[1].record(stream)
        lib.kernel_deltanet_prefill_batch(darr, len(djobs))
        ev[2].record(stream)
        torch.cuda.synchronize()
        ta += ev[0].elapsed_time(ev[1])
        td += ev[1].elapsed_time(ev[2])
    R.synchronize()
    launches = R.launch_count() - n0
    del keep
    return ta / steps, td / steps, launches


# ------------------------------------------------------------------------------ projections (section 8f row 3)

# One decode token's projections of the 40-layer hybrid stack (kernel_matvec_quant_batch's jobs):
# 10 full-attention layers (q+gate 8192x2048 Q4_K, k 512x2048 Q4_K, v 512x2048 Q6_K,
# o 2048x4096 Q6_K) and 30 DeltaNet layers (qkv 8192x2048 Q4_K, z 4096x2048 Q4_K, alpha and beta
# 32x2048 Q4_K, ssm_out 2048x4096 Q6_K).
PROJ_ATT = [(False, 8192, 2048), (False, 512, 2048), (True, 512, 2048), (True, 2048, 4096)]
PROJ_DN = [(False, 8192, 2048), (False, 4096, 2048), (False, 32, 2048), (False, 32, 2048), (True, 2048, 4096)]
PROJ_SHAPES = PROJ_ATT * 10 + PROJ_DN * 30


def proj_bytes(shapes) -> int:
    return sum(r * (c // 256) * (210 if q6 else 144) for q6, r, c in shapes)


def run_projections(R, torch, dev, stream, steps: int, rank: int):
    """All projections of the stack for one token in one kernel_cuda_matvec_quant_batch call:
    random k-quant blocks (uniform bytes) and N(0,1) activations. The weights (811 MB) exceed L2,
    so each step streams them from HBM. Returns (ms per step, launches)."""
    keep, jobs = [], []
    gen = torch.Generator(device=dev)
    gen.manual_seed(7000 + rank)
    for q6, r, c in PROJ_SHAPES:
        m = torch.randint(0, 256, (r * (c // 256) * (210 if q6 else 144),), dtype=torch.uint8, device=dev,
                          generator=gen)
        x = torch.randn(c, device=dev, generator=gen)
        y = torch.empty(r, device=dev)
        keep.append((m, x, y))
        jobs.append(R.KernelCudaMatvecJob(int(q6), m.data_ptr(), x.data_ptr(), y.data_ptr(), r, c))
    arr = (R.KernelCudaMatvecJob * len(jobs))(*jobs)
    lib = R.lib()
    for _ in range(3):
        if lib.kernel_cuda_matvec_quant_batch(arr, len(jobs)) != 0:
            raise RuntimeError(R.last_error())
    R.synchronize()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = R.launch_count()
    e0.record(stream)
    for _ in range(steps):
        lib.kernel_cuda_matvec_quant_batch(arr, len(jobs))
    e1.record(stream)
    R.synchronize()
    torch.cuda.synchronize()
    launches = R.launch_count() - n0
    del keep
    return e0.elapsed_time(e1) / steps, launches


def proj_cpu_reference(seconds: float = 1.5) -> dict:
    """The reference's own CPU k-quant matvec (kernel_dot_q4_k / kernel_dot_q6_k per row under
    OpenMP, as matvec_q4_cpu / matvec_q6_cpu) on one DeltaNet layer's and one attention layer's
    projections, repeated for about `seconds`."""
    import numpy as np
    import oracle as O
    from roaster_b200 import synth
    shapes = PROJ_ATT + PROJ_DN
    mats = [(q6, synth.quant_matrix(11 + i, r, c, q6), np.random.default_rng(i).standard_normal(c).astype(np.float32),
             r, c) for i, (q6, r, c) in enumerate(shapes)]
    O.matvec_q(*mats[0][:2], mats[0][2], mats[0][3], mats[0][4], impl="ref")
    reps, t0 = 0, time.perf_counter()
    while True:
        for q6, m, x, r, c in mats:
            O.matvec_q(q6, m, x, r, c, impl="ref")
        reps += 1
        el = time.perf_counter() - t0
        if el > seconds:
            break
    nbytes = proj_bytes(shapes) * reps
    return {"GBps": nbytes / el / 1e9, "threads": os.cpu_count(), "reps": reps,
            "sample_MB": proj_bytes(shapes) / 1e6}


PREFILL_PROJ_T = 256      # one prefill chunk (the reference's MM_MAX_T, kernels.c:1837)


def proj_flops(shapes, T: int) -> float:
    return 2.0 * T * sum(r * c for _, r, c in shapes)


def run_prefill_projections(R, torch, dev, stream, steps: int, rank: int):
    """One 256-token prefill chunk through every projection of the stack in one
    kernel_cuda_matmul_quant_batch call (190 jobs; the projections of a layer that read the same
    input share one X, as in the reference's batched prefill). Random k-quant blocks, N(0,1)
    activations. Returns (ms per step, launches)."""
    T = PREFILL_PROJ_T
    keep, jobs = [], []
    gen = torch.Generator(device=dev)
    gen.manual_seed(7100 + rank)
    layers = [PROJ_ATT] * 10 + [PROJ_DN] * 30
    for shapes in layers:
        xs = {}
        for q6, r, c in shapes:
            if c not in xs or c == 4096:        # the o / ssm_out projections read their own input
                xs[c] = torch.randn(T, c, device=dev, generator=gen)
            m = torch.randint(0, 256, (r * (c // 256) * (210 if q6 else 144),), dtype=torch.uint8, device=dev,
                              generator=gen)
            y = torch.empty(T, r, device=dev)
            keep.append((m, xs[c], y))
            jobs.append(R.KernelCudaMatmulJob(int(q6), m.data_ptr(), xs[c].data_ptr(), y.data_ptr(), r, c, T))
    arr = (R.KernelCudaMatmulJob * len(jobs))(*jobs)
    lib = R.lib()
    for _ in range(3):
        if lib.kernel_cuda_matmul_quant_batch(arr, len(jobs)) != 0:
            raise RuntimeError(R.last_error())
    R.synchronize()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = R.launch_count()
    e0.record(stream)
    for _ in range(steps):
        lib.kernel_cuda_matmul_quant_batch(arr, len(jobs))
    e1.record(stream)
    R.synchronize()
    torch.cuda.synchronize()
    launches = R.launch_count() - n0
    del keep
    return e0.elapsed_time(e1) / steps, launches


# ------------------------------------------------------------------- cross-slot batched step (section 8f row 4)

STEP_SLOTS = 64           # config 2's slots per GPU


def run_batched_step(R, torch, dev, stream, steps: int, rank: int, slots: int = STEP_SLOTS):
    """`slots` native slot threads (libslot_threads.so) step one token each through the step group,
    layer by layer: per layer one kernel_step_group_matvec with that layer's projections (site =
    layer; the projections of a layer that read the same input share it, as in the model). The
    group merges the slots' jobs on each shared matrix into one `slots`-token product.
    Compared with the per-slot form of the reference's step lock: one
    kernel_cuda_matvec_quant_batch per slot carrying all 190 of its projections, slots one after
    another. Returns a dict of timings."""
    import ctypes as C
    import time
    from roaster_b200 import build as B
    drv = C.CDLL(B.SLOT_LIB)
    drv.slot_threads_run.restype = C.c_int
    drv.slot_threads_run.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_int), C.c_int, C.c_int,
                                     C.POINTER(C.c_int), C.POINTER(R.KernelCudaMatvecJob), C.c_int]
    gen = torch.Generator(device=dev)
    gen.manual_seed(7200 + rank)
    mats = [torch.randint(0, 256, (r * (c // 256) * (210 if q6 else 144),), dtype=torch.uint8, device=dev,
                          generator=gen) for q6, r, c in PROJ_SHAPES]
    layers = [PROJ_ATT] * 10 + [PROJ_DN] * 30
    per_site = [len(shapes) for shapes in layers]
    total = len(PROJ_SHAPES)
    # a layer's projections that read the same input share it (q/k/v; qkv/z/alpha/beta), the
    # output projection (o / ssm_out, 4096 columns) reads its own: one 2048 and one 4096 vector
    xcols = sum(sum({c for _, _, c in shapes}) for shapes in layers)
    yrows = sum(r for _, r, _ in PROJ_SHAPES)
    X = torch.randn(slots, xcols, device=dev, generator=gen)
    Y = torch.zeros(slots, yrows + 4 * total, device=dev)
    jobs = (R.KernelCudaMatvecJob * (slots * total))()
    for i in range(slots):
        xo = yo = 0
        j = 0
        for shapes in layers:
            xoff = {}
            for c in sorted({c for _, _, c in shapes}):
                xoff[c] = xo
                xo += c
            for q6, r, c in shapes:
                jobs[i * total + j] = R.KernelCudaMatvecJob(int(q6), mats[j].data_ptr(), X[i, xoff[c]:].data_ptr(),
                                                            Y[i, yo:].data_ptr(), r, c)
                yo += (r + 3) // 4 * 4          # 16-byte aligned outputs
                j += 1
    ps = (C.c_int * len(per_site))(*per_site)
    g = R.StepGroup(slots, straggler_us=2000, call_timeout_ms=20000)
    ids_l = [g.join() for _ in range(slots)]
    ids = (C.c_int * slots)(*ids_l)
    lib = R.lib()

    def group_rounds(n):
        if drv.slot_threads_run(C.c_void_p(g._h), slots, ids, n, len(per_site), ps, jobs, total) != 0:
            raise RuntimeError("step group: " + R.last_error())

    group_rounds(3)          # warm-up: plain launches, then each layer's call recorded
    R.synchronize()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = R.launch_count()
    st0 = g.stats()
    t0 = time.perf_counter()
    e0.record(stream)
    group_rounds(steps)
    e1.record(stream)
    R.synchronize()
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) * 1e3 / steps
    gms = e0.elapsed_time(e1) / steps
    launches = R.launch_count() - n0
    st1 = g.stats()
    for m in ids_l:
        g.leave(m)
    g.close()

    # the per-slot form: one call per slot, slots in turn
    per = [C.cast(C.addressof(jobs) + i * total * C.sizeof(R.KernelCudaMatvecJob), C.POINTER(R.KernelCudaMatvecJob))
           for i in range(slots)]
    for i in range(slots):
        lib.kernel_cuda_matvec_quant_batch(per[i], total)
    R.synchronize()
    torch.cuda.synchronize()
    psteps = max(1, steps // 2)
    e0.record(stream)
    for _ in range(psteps):
        for i in range(slots):
            if lib.kernel_cuda_matvec_quant_batch(per[i], total) != 0:
                raise RuntimeError(R.last_error())
    e1.record(stream)
    R.synchronize()
    torch.cuda.synchronize()
    sms = e0.elapsed_time(e1) / psteps
    del mats, X, Y
    return {"group_ms": gms, "group_wall_ms": wall, "serial_ms": sms, "launches": launches,
            "rounds": st1["rounds"] - st0["rounds"], "calls": st1["calls"] - st0["calls"],
            "products": st1["products"] - st0["products"], "max_round": st1["max_round"],
            "replayed": st1["replayed"] - st0["replayed"]}


def prefill_proj_cpu_reference(seconds: float = 2.0) -> dict:
    """The reference's own CPU prefill matmul (matmul_quant_cpu under OpenMP) on one attention
    layer's and one DeltaNet layer's projections for a 256-token chunk, repeated for about
    `seconds`."""
    import numpy as np
    import oracle as O
    from roaster_b200 import synth
    shapes = PROJ_ATT + PROJ_DN
    T = PREFILL_PROJ_T
    mats = [(q6, synth.quant_matrix(21 + i, r, c, q6),
             np.random.default_rng(i).standard_normal((T, c)).astype(np.float32), r, c)
            for i, (q6, r, c) in enumerate(shapes)]
    reps, t0 = 0, time.perf_counter()
    while True:
        for q6, m, X, r, c in mats:
            O.matmul_q(q6, m, X, r, c, impl="ref")
        reps += 1
        el = time.perf_counter() - t0
        if el > seconds:
            break
    return {"TFLOPs": proj_flops(shapes, T) * reps / el / 1e12, "threads": os.cpu_count(), "reps": reps}


# ------------------------------------------------------------------------------ long context (config 4)

LONG_SLOTS = 16


def run_long_context(R, torch, dist, dev, stream, world: int, rank: int, window: int, steps: int,
                     warmup: int = 3, mode: str = "push"):
    """Config 4: 16 slots x `window` f16 KV positions, each window split into contiguous slices
    across the ranks; the rank holding the newest slice appends. Plus 3 DeltaNet layers per slot
    on the slot's home rank (slot % world). Strong scaling: the job is fixed, ranks split it.
    The per-(slot, kv head) softmax partials (8.3 KB each) are combined on the slot's home rank:
      mode "push":   the partial kernel stores them straight into the home rank's memory (peer
                     stores over NVLink, buffers opened through CUDA IPC) with a tag per record;
                     the home rank's merge kernel waits on the tags; no collective in the step;
      mode "gather": an NCCL all-gather of every rank's partials, then every rank merges all
                     slots (kernel_attn_merge_partials)."""
    import ctypes as C

    from roaster_b200 import splitkv, synth
    lo, hi = splitkv.slice_bounds(window, world, rank)
    app = splitkv.appends(world, rank)
    local = hi - lo
    cap = local + (steps + warmup + 8 if app else 0)
    kpool = synth.device_normal(torch, (LONG_SLOTS * cap, 2, 256), 500 + rank, dev, torch.float16)
    vpool = synth.device_normal(torch, (LONG_SLOTS * cap, 2, 256), 600 + rank, dev, torch.float16)
    g = torch.Generator(device=dev)
    g.manual_seed(700)                           # identical q / gate / new token on every rank
    q = torch.randn(LONG_SLOTS, 16, 256, generator=g, device=dev)
    gate = torch.randn(LONG_SLOTS, 16, 256, generator=g, device=dev)
    kn = torch.randn(LONG_SLOTS, 2, 256, generator=g, device=dev)
    vn = torch.randn(LONG_SLOTS, 2, 256, generator=g, device=dev)
    qn = 1 + 0.1 * torch.randn(256, generator=g, device=dev)
    kw = 1 + 0.1 * torch.randn(256, generator=g, device=dev)
    out = torch.empty(LONG_SLOTS, 16, 256, device=dev)
    home = splitkv.home_slots(LONG_SLOTS, world, rank)
    nh = max(1, len(home))
    states = synth.device_normal(torch, (nh, DN_LAYERS, 32, 128, 128), 800 + rank, dev, torch.float32, std=0.02)
    dq = torch.nn.functional.normalize(torch.randn(nh, DN_LAYERS, 16, 128, device=dev), dim=-1)
    dk = torch.nn.functional.normalize(torch.randn(nh, DN_LAYERS, 16, 128, device=dev), dim=-1)
    dv = torch.randn(nh, DN_LAYERS, 32, 128, device=dev)
    db = torch.sigmoid(torch.randn(nh, DN_LAYERS, 32, device=dev))
    dg = -torch.rand(nh, DN_LAYERS, 32, device=dev)
    dout = torch.empty(nh, DN_LAYERS, 32, 128, device=dev)
    es = kpool.element_size()
    jobs = [R.attn_job(q[s], gate[s], kn[s], vn[s], qn, kw,
                       kpool.data_ptr() + s * cap * 512 * es, vpool.data_ptr() + s * cap * 512 * es,
                       local, window, out[s], append=app, capacity=cap) for s in range(LONG_SLOTS)]
    arr = (R.KernelAttnDecodeJob * LONG_SLOTS)(*jobs)
    dj = [R.delta_job(states[i, l], dq[i, l], dk[i, l], dv[i, l], dg[i, l], db[i, l], dout[i, l])
          for i in range(len(home)) for l in range(DN_LAYERS)]
    darr = (R.KernelDeltaStepJob * max(1, len(dj)))(*dj) if dj else None
    lib = R.lib()
    vp = C.c_void_p
    opened, owned = [], []
    if world > 1 and mode == "push":
        # The push form's merge waits on kernels of the other ranks: every rank must be on a GPU
        # of its own (two ranks sharing one would wait on each other within one GPU).
        ids = [None] * world
        dist.all_gather_object(ids, str(torch.cuda.get_device_properties(dev).uuid))
        if len(set(ids)) != world:
            mode = "gather"
    if world > 1 and mode == "push":
        nbytes = splitkv.recv_floats(LONG_SLOTS, world, rank) * 4
        tbytes = splitkv.tag_words(LONG_SLOTS, world, rank) * 4
        recv, tags = lib.kernel_cuda_alloc(nbytes), lib.kernel_cuda_alloc(tbytes)   # zeroed
        if not recv or not tags:
            raise RuntimeError(R.last_error())
        owned = [recv, tags]
        mine = (R.ipc_handle(recv), R.ipc_handle(tags))
        allh = [None] * world
        dist.all_gather_object(allh, mine)
        rbases, tbases = [], []
        for r in range(world):
            if r == rank:
                rbases.append(recv)
                tbases.append(tags)
            else:
                a_, b_ = R.ipc_open(allh[r][0]), R.ipc_open(allh[r][1])
                opened += [a_, b_]
                rbases.append(a_)
                tbases.append(b_)
        targets = []
        for par in (0, 1):            # push addresses of both parity halves (epoch parity)
            d_, t_ = splitkv.push_targets(LONG_SLOTS, world, rank, par, rbases, tbases)
            targets.append(((vp * LONG_SLOTS)(*d_), (vp * LONG_SLOTS)(*t_),
                            splitkv.merge_view(LONG_SLOTS, world, rank, par, recv, tags)))
        gates_h = (vp * nh)(*[gate[s].data_ptr() for s in home])
        outs_h = (vp * nh)(*[out[s].data_ptr() for s in home])
    else:
        part = torch.empty(LONG_SLOTS, 2, splitkv.PARTIAL_FLOATS, device=dev)
        gathered = torch.empty(world, LONG_SLOTS, 2, splitkv.PARTIAL_FLOATS, device=dev)
        gates_p = (vp * LONG_SLOTS)(*[gate[s].data_ptr() for s in range(LONG_SLOTS)])
        outs_p = (vp * LONG_SLOTS)(*[out[s].data_ptr() for s in range(LONG_SLOTS)])
    pos = [window]
    epoch = [0]

    def one():
        for s in range(LONG_SLOTS):
            arr[s].position = pos[0]
        epoch[0] += 1
        if world == 1:
            rc = lib.kernel_attn_decode_batch(arr, LONG_SLOTS)
        elif mode == "push":
            dst_a, tag_a, (rv, tv) = targets[epoch[0] & 1]

            def push_fn():
                if lib.kernel_attn_decode_partial_push(arr, LONG_SLOTS, dst_a, tag_a, epoch[0]) != 0:
                    raise RuntimeError(R.last_error())

            def merge_fn():
                if home and lib.kernel_attn_merge_wait(vp(rv), vp(tv), world, len(home), gates_h, 256, outs_h,
                                                       epoch[0]) != 0:
                    raise RuntimeError(R.last_error())

            splitkv.push_step(push_fn, merge_fn)
            rc = 0
        else:
            def partial_fn():
                if lib.kernel_attn_decode_partial_batch(arr, LONG_SLOTS, vp(part.data_ptr())) != 0:
                    raise RuntimeError(R.last_error())
                return part

            def gather_fn(local_part):
                dist.all_gather_into_tensor(gathered, local_part)
                return gathered

            def merge_fn(gt, w):
                if lib.kernel_attn_merge_partials(vp(gt.data_ptr()), w, LONG_SLOTS, gates_p, 256, outs_p) != 0:
                    raise RuntimeError(R.last_error())

            splitkv.step(world, partial_fn, gather_fn, merge_fn)
            rc = 0
        if darr is not None:
            rc |= lib.kernel_deltanet_step_batch(darr, len(dj))
        if rc != 0:
            raise RuntimeError(R.last_error())
        if app:
            for s in range(LONG_SLOTS):
                arr[s].length += 1
        pos[0] += 1

    for _ in range(warmup):
        one()
    R.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = R.launch_count()
    e0.record(stream)
    for _ in range(steps):
        one()
    e1.record(stream)
    torch.cuda.synchronize()
    R.synchronize()
    ms = e0.elapsed_time(e1) / steps
    launches = R.launch_count() - n0
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    ms = float(t.item())
    for ptr in opened:
        R.ipc_close(ptr)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
    for ptr in owned:
        lib.kernel_cuda_free(vp(ptr))
    kv_bytes = LONG_SLOTS * local * 2048
    dn_bytes = len(home) * DN_LAYERS * (2 * 32 * 128 * 128 * 4)
    hbm, _, src = peaks()
    gbs = (kv_bytes + dn_bytes) / (ms / 1e3) / 1e9
    del kpool, vpool
    return {"metric": "long-context decode tok/s (config 4: 16 slots x 262144 f16 KV + 3 DeltaNet layers)",
            "value": round(LONG_SLOTS / (ms / 1e3), 1), "unit": "tok/s", "ms_per_step": round(ms, 4),
            "steps": steps, "scaling": "strong", "window": window,
            "kv_split": (f"{world} contiguous slices per slot; " +
                         ("one GPU, no split" if world == 1 else
                          "partials pushed into the home GPU's memory by the partial kernel (peer stores, "
                          "tagged), merged there; no collective" if mode == "push" else
                          "NCCL all-gather of softmax partials, every GPU merges every slot")),
            "kv_bytes_per_gpu_per_step": kv_bytes + dn_bytes,
            "roofline": {"bound": "hbm", "kernel": "attn_decode_kernel (+ deltanet_step_kernel)",
                         "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s", "frac": round(gbs / hbm, 4),
                         "peak_source": f"{src} hbm_gbs (a copy: read + write; this step only reads KV)",
                         "scope": "per GPU, the whole step (max over ranks)"},
            "gpu_launches": int(launches)}


# ------------------------------------------------------------------------------ config 2 (GPU arm)

def run_recurrent(R, torch, dev, stream, steps: int, warmup: int, parity: bool) -> dict:
    """Config 1: one slot's 30 Gated DeltaNet layers stepped `steps` times in sequence (after
    `warmup` untimed steps), one kernel_deltanet_step_batch of 30 jobs (one per layer) per step,
    each step's inputs drawn with config 1's distributions. The 30 states (63 MB) would stay in
    the 126 MB L2, so a 256 MB device write precedes every timed step and each step is timed
    alone (CUDA events on the launching stream). With `parity`, layers 0 and 29 are saved for
    the CPU check against the reference's recurrence over the whole sequence."""
    import numpy as np

    from roaster_b200 import synth
    L, n = RECUR_LAYERS, steps + warmup
    g = torch.Generator(device=dev)
    g.manual_seed(9100)
    rn = lambda *s: torch.randn(*s, generator=g, device=dev)  # noqa: E731
    nz = torch.nn.functional.normalize
    q = nz(rn(n, L, 16, 128), dim=-1).contiguous()
    k = nz(rn(n, L, 16, 128), dim=-1).contiguous()
    v = rn(n, L, 32, 128)
    beta = torch.sigmoid(rn(n, L, 32))
    gl = (-torch.exp(-1 + 0.5 * rn(n, L, 32)) * torch.nn.functional.softplus(rn(n, L, 32))).contiguous()
    states = synth.device_normal(torch, (L, 32, 128, 128), 9101, dev, torch.float32, std=0.02)
    pick = [0, L - 1]
    st0 = states[pick].cpu().numpy() if parity else None
    out = torch.empty(n, L, 32, 128, device=dev)
    # job arrays from raw addresses (30 x (steps + warmup) jobs)
    qa, ka, va, ga, ba, oa, sa = (t.data_ptr() for t in (q, k, v, gl, beta, out, states))
    arrs = []
    for s in range(n):
        jobs = [R.delta_job(sa + l * 32 * 128 * 128 * 4, qa + (s * L + l) * 2048 * 4, ka + (s * L + l) * 2048 * 4,
                            va + (s * L + l) * 4096 * 4, ga + (s * L + l) * 32 * 4, ba + (s * L + l) * 32 * 4,
                            oa + (s * L + l) * 4096 * 4) for l in range(L)]
        arrs.append((R.KernelDeltaStepJob * L)(*jobs))
    lib = R.lib()
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)          # 256 MB > L2
    for s in range(warmup):
        if lib.kernel_deltanet_step_batch(arrs[s], L) != 0:
            raise RuntimeError(R.last_error())
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    launches0 = R.launch_count()
    for i in range(steps):
        flush.zero_()
        evs[i][0].record(stream)
        rc = lib.kernel_deltanet_step_batch(arrs[warmup + i], L)
        evs[i][1].record(stream)
        if rc != 0:
            raise RuntimeError(R.last_error())
    torch.cuda.synchronize()
    launches = R.launch_count() - launches0
    R.synchronize()
    ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    res = {"ms": ms, "launches": launches}
    if parity:
        z = {"n": np.int64(len(pick)), "layers": np.array(pick), "steps": np.int64(n)}
        for i, l in enumerate(pick):
            z[f"st0_{i}"] = st0[i]
            z[f"st_end{i}"] = states[l].cpu().numpy()
            for nm, t in (("q", q), ("k", k), ("v", v), ("g", gl), ("beta", beta), ("out", out)):
                z[f"{nm}{i}"] = np.ascontiguousarray(t[:, l].cpu().numpy())
        fd, path = tempfile.mkstemp(suffix=".npz", prefix="roaster_parity1_")
        os.close(fd)
        np.savez(path, **z)
        res["parity_file"] = path
    del q, k, v, beta, gl, states, out, flush
    return res


def run_layer_block(R, torch, dev, stream, steps: int, warmup: int) -> dict:
    """Config 1 with the recurrent-layer block around the recurrence (model.c:1291-1343 without
    the projections): per step, one kernel_deltanet_preop_batch (conv1d + SiLU + L2-norm + beta/g
    and the history shift, 30 jobs), one kernel_deltanet_step_batch and one
    kernel_deltanet_postop_batch (gated RMSNorm), timed like run_recurrent (a 256 MB device write
    before every step, each step timed alone), so the difference from the recurrence alone is what
    the pre/post-op launches cost per decode step."""
    from roaster_b200 import synth
    L = RECUR_LAYERS
    d = synth.delta_layer_inputs(9200, 1)
    rep = lambda x: torch.from_numpy(x).to(dev).expand(L, *x.shape).contiguous()  # noqa: E731
    qkv, z, alpha, beta = (rep(d[k]) for k in ("qkv", "z", "alpha", "beta"))
    conv_w, dt, av, norm_w = (rep(d[k]) for k in ("conv_w", "dt", "a", "ssm_norm"))
    conv_state = rep(d["conv_state"])
    states = synth.device_normal(torch, (L, 32, 128, 128), 9201, dev, torch.float32, std=0.02)
    q = torch.empty(L, 16, 128, device=dev)
    k = torch.empty(L, 16, 128, device=dev)
    v = torch.empty(L, 32, 128, device=dev)
    g = torch.empty(L, 32, device=dev)
    b = torch.empty(L, 32, device=dev)
    out = torch.empty(L, 32, 128, device=dev)
    P = lambda t, l: t[l].data_ptr()  # noqa: E731
    pre = (R.KernelDeltaPreopJob * L)(*[R.KernelDeltaPreopJob(
        P(qkv, l), P(alpha, l), P(beta, l), P(conv_state, l), P(conv_w, l), P(dt, l), P(av, l),
        P(q, l), P(k, l), P(v, l), P(g, l), P(b, l), 1) for l in range(L)])
    stp = (R.KernelDeltaStepJob * L)(*[R.delta_job(P(states, l), P(q, l), P(k, l), P(v, l), P(g, l), P(b, l),
                                                   P(out, l)) for l in range(L)])
    post = (R.KernelDeltaPostopJob * L)(*[R.KernelDeltaPostopJob(P(out, l), P(z, l), P(norm_w, l), 1)
                                          for l in range(L)])
    lib = R.lib()

    def step():
        if (lib.kernel_deltanet_preop_batch(pre, L) != 0 or lib.kernel_deltanet_step_batch(stp, L) != 0
                or lib.kernel_deltanet_postop_batch(post, L) != 0):
            raise RuntimeError(R.last_error())

    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)          # 256 MB > L2
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    launches0 = R.launch_count()
    for i in range(steps):
        flush.zero_()
        evs[i][0].record(stream)
        step()
        evs[i][1].record(stream)
    torch.cuda.synchronize()
    launches = R.launch_count() - launches0
    R.synchronize()
    if not bool(torch.isfinite(out).all()):
        raise RuntimeError("layer block: non-finite outputs")
    ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    del qkv, z, alpha, beta, conv_w, dt, av, norm_w, conv_state, states, q, k, v, g, b, out, flush
    return {"ms": ms, "launches": launches}


def attn_step_bytes(n: int, mean_L: float) -> float:
    """Algorithmic bytes of one decode-attention launch over n slots of mean window mean_L:
    the f16 K/V rows (2 kv heads x K,V x 256 x 2 B per position), the appended row, q/gate/out."""
    return n * (mean_L * 2048 + 2048 + 3 * 16 * 256 * 4 + 2 * 2 * 256 * 4)


def dn_step_bytes(n_states: int) -> float:
    """Algorithmic bytes of one DeltaNet step launch: state read + write, inputs and outputs."""
    return n_states * (2 * 32 * 128 * 128 * 4 + (2 * 16 + 2 * 32) * 128 * 4 + 2 * 32 * 4)


def run_config2(R, torch, dev, stream, lens, K: int, W: int, seed: int, world: int, barrier,
                clocks=None, e2e: bool = False, parity: bool = False):
    """Time K steps (after W warm-up steps) of the config-2 decode over this GPU's slots `lens`:
    one kernel_attn_decode_batch + one kernel_deltanet_step_batch per step, windows growing by
    one token per step. Optionally: the same steps through the host-buffer entry points (e2e),
    and one more step whose inputs and outputs for a sample of slots are saved for the CPU
    parity check. Returns per-rank figures (the caller takes the max over ranks)."""
    import numpy as np

    from roaster_b200 import synth
    n = len(lens)
    grow = K + W + 8
    caps = [L + grow for L in lens]
    offs = np.concatenate([[0], np.cumsum(caps)]).astype(np.int64)
    # KV windows of all slots in one pool (per slot [cap][2][256] f16, 1 KB per position)
    kpool = synth.device_normal(torch, (int(offs[-1]), 2, 256), seed, dev, torch.float16)
    vpool = synth.device_normal(torch, (int(offs[-1]), 2, 256), seed + 1, dev, torch.float16)
    states = synth.device_normal(torch, (n, DN_LAYERS, 32, 128, 128), seed + 2, dev, torch.float32, std=0.02)
    NP = 4                                            # rotating pools of per-step inputs
    g = torch.Generator(device=dev)
    g.manual_seed(seed + 3)
    rn = lambda *s: torch.randn(*s, generator=g, device=dev)  # noqa: E731
    q, gate = rn(NP, n, 16, 256), rn(NP, n, 16, 256)
    kn, vn = rn(NP, n, 2, 256), rn(NP, n, 2, 256)
    qn = 1 + 0.1 * rn(256)
    kw = 1 + 0.1 * rn(256)
    dq = torch.nn.functional.normalize(rn(NP, n, DN_LAYERS, 16, 128), dim=-1)
    dk = torch.nn.functional.normalize(rn(NP, n, DN_LAYERS, 16, 128), dim=-1)
    dv = rn(NP, n, DN_LAYERS, 32, 128)
    dbeta = torch.sigmoid(rn(NP, n, DN_LAYERS, 32))
    dgl = -torch.exp(-1 + 0.5 * rn(NP, n, DN_LAYERS, 32)) * torch.nn.functional.softplus(
        rn(NP, n, DN_LAYERS, 32))
    aout = torch.empty(n, 16, 256, device=dev)
    dout = torch.empty(n, DN_LAYERS, 32, 128, device=dev)
    es = kpool.element_size()
    kaddr = [kpool.data_ptr() + int(offs[s]) * 512 * es for s in range(n)]
    vaddr = [vpool.data_ptr() + int(offs[s]) * 512 * es for s in range(n)]

    attn_arrs, dn_arrs = [], []
    for pi in range(NP):
        jobs = [R.attn_job(q[pi, s], gate[pi, s], kn[pi, s], vn[pi, s], qn, kw, kaddr[s], vaddr[s],
                           lens[s], lens[s], aout[s], capacity=caps[s]) for s in range(n)]
        attn_arrs.append((R.KernelAttnDecodeJob * n)(*jobs))
        dj = [R.delta_job(states[s, l], dq[pi, s, l], dk[pi, s, l], dv[pi, s, l], dgl[pi, s, l],
                          dbeta[pi, s, l], dout[s, l]) for s in range(n) for l in range(DN_LAYERS)]
        dn_arrs.append((R.KernelDeltaStepJob * len(dj))(*dj))
    lib = R.lib()
    cur = list(lens)

    def step(i, ev=None):
        arr = attn_arrs[i % NP]
        for s in range(n):
            arr[s].length = cur[s]
            arr[s].position = cur[s]
        if ev:
            ev[0].record(stream)
        rc = lib.kernel_attn_decode_batch(arr, n)
        if ev:
            ev[1].record(stream)
        rc |= lib.kernel_deltanet_step_batch(dn_arrs[i % NP], n * DN_LAYERS)
        if ev:
            ev[2].record(stream)
        if rc != 0:
            raise RuntimeError(R.last_error())
        for s in range(n):
            cur[s] += 1

    for i in range(W):
        step(i)
    R.synchronize()
    torch.cuda.synchronize()
    barrier()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if clocks:
        clocks.start()
        time.sleep(0.3)
    launches0 = R.launch_count()
    lens_at_start = list(cur)
    t_start.record(stream)
    for i in range(K):
        step(W + i, evs[i])
    t_end.record(stream)
    torch.cuda.synchronize()
    launches = R.launch_count() - launches0
    clk = clocks.stop() if clocks else None
    R.synchronize()
    res = {"ms": t_start.elapsed_time(t_end),
           "attn_ms": statistics.mean(e[0].elapsed_time(e[1]) for e in evs),
           "dn_ms": statistics.mean(e[1].elapsed_time(e[2]) for e in evs),
           "launches": launches, "clocks": clk,
           "mean_L": statistics.mean(lens_at_start) + (K - 1) / 2, "n": n}

    # ---------------------------------------------------------------- parity sample (untimed)
    if parity:
        order = sorted(range(n), key=lambda s: lens[s])
        pick = sorted({order[0], order[-1], order[len(order) // 2], *order[:: max(1, n // 4)]})[:6]
        pi = (W + K) % NP
        z = {"n": np.int64(len(pick)), "qn": qn.cpu().numpy(), "kw": kw.cpu().numpy()}
        for j, s in enumerate(pick):
            L = cur[s]
            z[f"len{j}"] = np.int64(L)
            z[f"kc{j}"] = kpool[int(offs[s]):int(offs[s]) + L].cpu().numpy()
            z[f"vc{j}"] = vpool[int(offs[s]):int(offs[s]) + L].cpu().numpy()
            z[f"q{j}"], z[f"gate{j}"] = q[pi, s].cpu().numpy(), gate[pi, s].cpu().numpy()
            z[f"kn{j}"], z[f"vn{j}"] = kn[pi, s].cpu().numpy(), vn[pi, s].cpu().numpy()
            z[f"st{j}"] = states[s].cpu().numpy()
            for nm, t in (("q", dq), ("k", dk), ("v", dv), ("g", dgl), ("beta", dbeta)):
                z[f"d{nm}{j}"] = t[pi, s].cpu().numpy()
        step(W + K)                                   # the same two launches as a timed step
        R.synchronize()
        for j, s in enumerate(pick):
            z[f"out{j}"] = aout[s].cpu().numpy()
            z[f"dout{j}"] = dout[s].cpu().numpy()
            z[f"st_after{j}"] = states[s].cpu().numpy()
        fd, path = tempfile.mkstemp(suffix=".npz", prefix="roaster_parity_")
        os.close(fd)
        np.savez(path, **z)
        res["parity_file"] = path

    # ---------------------------------------------------------------- end to end (host buffers)
    if e2e:
        # All host inputs and outputs in one allocation, so the caller registers one range
        # (kernel_cuda_host_register) once, outside the timed region, as a serving host would
        # its long-lived step buffers.
        shapes = {"q": (NP, n, 16, 256), "gate": (NP, n, 16, 256), "kn": (NP, n, 2, 256), "vn": (NP, n, 2, 256),
                  "qn": (256,), "kw": (256,), "dq": (NP, n, DN_LAYERS, 16, 128), "dk": (NP, n, DN_LAYERS, 16, 128),
                  "dv": (NP, n, DN_LAYERS, 32, 128), "dg": (NP, n, DN_LAYERS, 32), "db": (NP, n, DN_LAYERS, 32),
                  "ao": (n, 16, 256), "do": (n, DN_LAYERS, 32, 128)}
        sizes = {k: int(np.prod(v)) for k, v in shapes.items()}
        host = np.zeros(sum(sizes.values()), np.float32)
        H, o_ = {}, 0
        for k, shp in shapes.items():
            H[k] = host[o_:o_ + sizes[k]].reshape(shp)
            o_ += sizes[k]
        for k, t in (("q", q), ("gate", gate), ("kn", kn), ("vn", vn), ("qn", qn), ("kw", kw), ("dq", dq),
                     ("dk", dk), ("dv", dv), ("dg", dgl), ("db", dbeta)):
            H[k][...] = t.cpu().numpy()
        ha, hd = [], []
        for pi in range(NP):
            jobs = [R.attn_job(H["q"][pi, s].ctypes.data, H["gate"][pi, s].ctypes.data, H["kn"][pi, s].ctypes.data,
                               H["vn"][pi, s].ctypes.data, H["qn"].ctypes.data, H["kw"].ctypes.data, kaddr[s],
                               vaddr[s], 0, 0, H["ao"][s].ctypes.data, capacity=caps[s]) for s in range(n)]
            ha.append((R.KernelAttnDecodeJob * n)(*jobs))
            dj = [R.delta_job(states[s, l], H["dq"][pi, s, l].ctypes.data, H["dk"][pi, s, l].ctypes.data,
                              H["dv"][pi, s, l].ctypes.data, H["dg"][pi, s, l].ctypes.data,
                              H["db"][pi, s, l].ctypes.data, H["do"][s, l].ctypes.data)
                  for s in range(n) for l in range(DN_LAYERS)]
            hd.append((R.KernelDeltaStepJob * len(dj))(*dj))
        KE = max(1, min(K, 200))

        def estep(i):
            arr = ha[i % NP]
            for s in range(n):
                arr[s].length = cur[s]
                arr[s].position = cur[s]
            rc = lib.kernel_attn_decode_batch_host(arr, n)
            rc |= lib.kernel_deltanet_step_batch_host(hd[i % NP], n * DN_LAYERS)
            if rc != 0:
                raise RuntimeError(R.last_error())
            for s in range(n):
                cur[s] += 1

        def timed_e2e():
            # windows were sized for K+W+8 appends: wind them back and append again (KE <= K)
            for s in range(n):
                cur[s] = lens[s]
            for i in range(2):
                estep(i)
            barrier()
            t0 = time.perf_counter()
            for i in range(KE):
                estep(i)
            return time.perf_counter() - t0

        if lib.kernel_cuda_host_register(host.ctypes.data, host.nbytes) != 0:
            raise RuntimeError(R.last_error())
        try:
            res["e2e_s"] = timed_e2e()
        finally:
            lib.kernel_cuda_host_unregister(host.ctypes.data)
        res["e2e_staged_s"] = timed_e2e()
        res["e2e_steps"] = KE
        res["h2d"] = n * (4096 * 2 + 512 * 2 + 256 * 2) * 4 + n * DN_LAYERS * (2 * 2048 + 4096 + 64) * 4
        res["d2h"] = n * 4096 * 4 + n * DN_LAYERS * 4096 * 4
    del kpool, vpool, states
    return res



# ------------------------------------------------------------------------------ GPU arm

def run_ours(a):
    # NCCL prints its banner to stdout; keep stdout for the one JSON line
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
    import torch
    import torch.distributed as dist

    import roaster_b200 as R

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    R.init(local)
    stream = torch.cuda.current_stream()
    R.set_stream(stream)

    def barrier():
        if world > 1:
            dist.barrier()

    def allmax(vals):
        t = torch.tensor([float(v) for v in vals], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(x) for x in t.tolist()]

    K, W = a.steps, a.warmup
    hbm, _, src = peaks()
    glens = slot_lengths(1000, a.kv_lo, a.kv_hi)
    mine = assign_slots(glens, world)[rank]
    lens = [glens[s] for s in mine]
    clocks = ClockSampler(local if not os.environ.get("CUDA_VISIBLE_DEVICES") else
                          int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local]))
    want_parity = rank == 0 and not a.no_parity and not a.no_cpu_baseline
    c2 = run_config2(R, torch, dev, stream, lens, K, W, 11, world, barrier, clocks=clocks,
                     e2e=not a.no_e2e, parity=want_parity)
    ms, attn_avg, dn_avg = allmax([c2["ms"], c2["attn_ms"], c2["dn_ms"]])
    ms_step = ms / K
    value = SLOTS / (ms_step / 1e3)
    # algorithmic bytes per launch on the slowest rank's shard are not the same for every rank:
    # report rank 0's kernels against rank 0's own time
    attn_bytes = attn_step_bytes(c2["n"], c2["mean_L"])
    dn_bytes = dn_step_bytes(c2["n"] * DN_LAYERS)
    attn_gbs = attn_bytes / (c2["attn_ms"] / 1e3) / 1e9
    dn_gbs = dn_bytes / (c2["dn_ms"] / 1e3) / 1e9
    e2e = None
    if not a.no_e2e:
        el, els = allmax([c2["e2e_s"], c2["e2e_staged_s"]])
        e2e = {"value": round(SLOTS * c2["e2e_steps"] / el, 1), "unit": "tok/s",
               "h2d_bytes_per_step": c2["h2d"] * world, "d2h_bytes_per_step": c2["d2h"] * world,
               "steps": c2["e2e_steps"],
               "api": "kernel_attn_decode_batch_host + kernel_deltanet_step_batch_host",
               "host_buffers": "one numpy allocation registered once with kernel_cuda_host_register (outside "
                               "the timed region): each call's buffers move as a few large copy-engine "
                               "copies (their contiguous runs), no staging memcpy",
               "staged": {"value": round(SLOTS * c2["e2e_steps"] / els, 1), "unit": "tok/s",
                          "what": "the same calls with the buffers unregistered: pinned staging copies"}}

    # per-GPU efficiency of the shards the strong split gives each GPU at N = 2, 4, 8 (one GPU)
    shards = None
    if world == 1 and not a.no_shards:
        shards = {}
        for nr in (2, 4, 8):
            sl = [glens[s] for s in assign_slots(glens, nr)[0]]
            r = run_config2(R, torch, dev, stream, sl, min(K, 100), 3, 21, 1, barrier)
            ab = attn_step_bytes(r["n"], r["mean_L"])
            db = dn_step_bytes(r["n"] * DN_LAYERS)
            shards[f"{r['n']}_slots"] = {
                "as_rank0_of": nr, "ms_per_step": round(r["ms"] / min(K, 100), 4),
                "attn_ms": round(r["attn_ms"], 4), "attn_frac": round(ab / (r["attn_ms"] / 1e3) / 1e9 / hbm, 4),
                "deltanet_ms": round(r["dn_ms"], 4), "deltanet_frac": round(db / (r["dn_ms"] / 1e3) / 1e9 / hbm, 4),
                "step_frac": round((ab + db) / (r["ms"] / min(K, 100) / 1e3) / 1e9 / hbm, 4)}

    # 64 slots per GPU (weak scaling), the form measured before the strong split
    weak = None
    if world > 1:
        wl = slot_lengths(1000 + rank, a.kv_lo, a.kv_hi)
        KW = min(K, 100)
        r = run_config2(R, torch, dev, stream, wl, KW, 3, 31 + rank, world, barrier)
        wms, wattn = allmax([r["ms"], r["attn_ms"]])
        weak = {"metric": "config-2 decode with 64 slots per GPU (weak scaling)",
                "value": round(SLOTS * world / (wms / KW / 1e3), 1), "unit": "tok/s",
                "ms_per_step": round(wms / KW, 4), "steps": KW, "scaling": "weak",
                "attn_frac_rank0": round(attn_step_bytes(r["n"], r["mean_L"]) / (r["attn_ms"] / 1e3) / 1e9 / hbm, 4)}

    parity = None
    if want_parity:
        try:
            parity = cpu_leg("parity", path=c2["parity_file"], timeout=900)
            parity["pass"] = parity["attn_maxrel"] <= 2e-3 and parity["state_maxrel"] <= 1e-4 \
                and parity["deltanet_out_maxrel"] <= 1e-4
            parity["what"] = ("one more step of the timed batch (rank 0's shard, same launches), sampled "
                              "slots vs the reference's own CPU code; bars 2e-3 attention, 1e-4 DeltaNet")
        except Exception as e:  # reported, not fatal
            parity = {"pass": None, "error": str(e)[:300]}
        finally:
            try:
                os.remove(c2["parity_file"])
            except OSError:
                pass

    prefill = None
    if not a.no_prefill:
        ams, dms, pl = run_prefill(R, torch, dev, stream, a.prefill_steps, rank)
        ams, dms = allmax([ams, dms])
        pms = ams + dms
        _, tflops, srcp = peaks()
        flop = 2.0 * PREFILL_T * PREFILL_T * 256 * 16 * PREFILL_PROMPTS     # causal QK^T + PV
        achieved = flop / (ams / 1e3) / 1e12
        # chunked DeltaNet: per (chunk, value head) 10 C^2 d + 6 C d^2 flops (C = 64, d = 128)
        dflop = (10.0 * 64 * 64 * 128 + 6.0 * 64 * 128 * 128) * (PREFILL_T // 64) * 32 * PREFILL_PROMPTS
        dach = dflop / (dms / 1e3) / 1e12
        ntok = PREFILL_PROMPTS * PREFILL_T * world
        prefill = {"metric": "prefill tok/s (config 3: 8 prompts x 8192; causal gated attention, bf16 in, "
                             "+ one chunked Gated DeltaNet layer)",
                   "value": round(ntok / (pms / 1e3), 1),
                   "unit": "tok/s", "ms_per_step": round(pms, 4), "steps": a.prefill_steps,
                   "gpu_launches": int(pl),
                   "attention": {"ms_per_step": round(ams, 4), "tok_s": round(ntok / (ams / 1e3), 1),
                                 "roofline": {"bound": "tensor",
                                              "kernel": "prefill_attn_kernel (+ prefill_prep_kernel)",
                                              "achieved": round(achieved, 1), "peak": tflops, "unit": "TFLOP/s",
                                              "frac": round(achieved / tflops, 4),
                                              "peak_source": f"{srcp} bf16_tflops (burst; f16 operands run at the same rate)",
                                              "algorithmic_flop_per_step": flop}},
                   "deltanet": {"ms_per_step": round(dms, 4), "tok_s": round(ntok / (dms / 1e3), 1),
                                "roofline": {"bound": "tensor", "kernel": DN_PREFILL_KERNELS,
                                             "achieved": round(dach, 1), "peak": tflops, "unit": "TFLOP/s",
                                             "frac": round(dach / tflops, 4),
                                             "peak_source": f"{srcp} bf16_tflops (burst)",
                                             "algorithmic_flop_per_step": dflop,
                                             "note": DN_PREFILL_NOTE}}}
        if rank == 0 and world == 1 and not a.no_cpu_baseline:
            try:
                c = cpu_leg_ref("prefill", timeout=1200)
                per_prompt = c["attn_s_per_prompt"] + c["deltanet_s_per_prompt"]
                prefill["cpu_baseline"] = {
                    "value": round(PREFILL_T / per_prompt, 2), "unit": "tok/s", "cores": c["threads"],
                    "kind": "reference", "build": c["build"],
                    "attention_s_per_prompt": round(c["attn_s_per_prompt"], 3),
                    "deltanet_s_per_prompt": round(c["deltanet_s_per_prompt"], 3),
                    "sample": "ONE 8192-token prompt (the other 7 are the same work: x8 extrapolated, tok/s "
                              "unchanged): pf_attention in 256-token chunks, first and last chunk timed, "
                              "their difference giving the time per attended key (projections and prep "
                              "cancel), times the keys the 32 chunks attend to; delta_head over all 8192 "
                              "tokens for one DeltaNet layer"}
            except Exception as e:  # reported, not fatal
                prefill["cpu_baseline"] = {"value": None, "sample": f"failed: {e}"[:300]}

    proj = None
    if not a.no_proj:
        pms, plaunch = run_projections(R, torch, dev, stream, a.proj_steps, rank)
        (pms,) = allmax([pms])
        pbytes = proj_bytes(PROJ_SHAPES)
        hbm_p, _, src_p = peaks()
        gbs = pbytes / (pms / 1e3) / 1e9
        proj = {"metric": "decode projections GB/s (one token through the 40-layer stack's Q4_K/Q6_K "
                          "attention + DeltaNet projections, one kernel_cuda_matvec_quant_batch call)",
                "value": round(gbs * world, 1), "unit": "GB/s", "ms_per_step": round(pms, 4),
                "steps": a.proj_steps, "gpu_launches": int(plaunch), "jobs": len(PROJ_SHAPES),
                "weight_bytes_per_step": pbytes,
                "data": "synthetic: uniform random k-quant blocks, N(0,1) activations",
                "roofline": {"bound": "hbm", "kernel": "quant_matvec_staged_kernel",
                             "achieved": round(gbs, 1), "peak": hbm_p, "unit": "GB/s",
                             "frac": round(gbs / hbm_p, 4),
                             "peak_source": f"{src_p} hbm_gbs (burst)",
                             "algorithmic_bytes_per_launch": pbytes,
                             "l2": "weights (811 MB) exceed L2; no flush needed"}}
        if rank == 0 and world == 1 and not a.no_cpu_baseline:
            try:
                c = proj_cpu_reference()
                proj["cpu_baseline"] = {"value": round(c["GBps"], 2), "unit": "GB/s", "cores": c["threads"],
                                        "kind": "reference",
                                        "sample": f"{c['reps']} x one attention + one DeltaNet layer's projections "
                                                  f"({c['sample_MB']:.1f} MB), the reference's kernel_dot_q4_k / "
                                                  f"kernel_dot_q6_k per row under OpenMP"}
            except Exception as e:  # reported, not fatal
                proj["cpu_baseline"] = {"value": None, "sample": f"failed: {e}"[:300]}

    pproj = None
    if not a.no_proj:
        pms, plaunch = run_prefill_projections(R, torch, dev, stream, a.proj_steps, rank)
        (pms,) = allmax([pms])
        pflop = proj_flops(PROJ_SHAPES, PREFILL_PROJ_T)
        _, tens_p, src_p = peaks()
        tfs = pflop / (pms / 1e3) / 1e12
        pproj = {"metric": "prefill projections TFLOP/s (one 256-token chunk through the 40-layer stack's "
                           "Q4_K/Q6_K attention + DeltaNet projections, one kernel_cuda_matmul_quant_batch call)",
                 "value": round(tfs * world, 2), "unit": "TFLOP/s", "ms_per_step": round(pms, 4),
                 "tokens_per_s": round(PREFILL_PROJ_T / (pms / 1e3) * world, 1),
                 "steps": a.proj_steps, "gpu_launches": int(plaunch), "jobs": len(PROJ_SHAPES),
                 "algorithmic_flop_per_step": pflop,
                 "data": "synthetic: uniform random k-quant blocks, N(0,1) activations",
                 "roofline": {"bound": "tensor", "kernel": "quant_mm_tc_kernel",
                              "achieved": round(tfs, 2), "peak": tens_p, "unit": "TFLOP/s",
                              "frac": round(tfs / tens_p, 4),
                              "peak_source": f"{src_p} bf16_tflops (burst)",
                              "note": "tcgen05 (A from tensor memory, M = N = 128); each product runs as 2 "
                                      "f16 MMAs (activation hi + lo; Q6_K 4: the scale split in two exact "
                                      "halves), plus the Q4_K min term"}}
        if rank == 0 and world == 1 and not a.no_cpu_baseline:
            try:
                c = prefill_proj_cpu_reference()
                pproj["cpu_baseline"] = {"value": round(c["TFLOPs"], 4), "unit": "TFLOP/s", "cores": c["threads"],
                                         "kind": "reference",
                                         "sample": f"{c['reps']} x one attention + one DeltaNet layer's projections "
                                                   f"for 256 tokens, the reference's matmul_quant_cpu under OpenMP"}
            except Exception as e:  # reported, not fatal
                pproj["cpu_baseline"] = {"value": None, "sample": f"failed: {e}"[:300]}

    bstep = None
    if not a.no_proj:
        r = run_batched_step(R, torch, dev, stream, a.step_rounds, rank)
        gms, sms = allmax([r["group_ms"], r["serial_ms"]])
        flop = proj_flops(PROJ_SHAPES, STEP_SLOTS)
        _, tens_p, src_p = peaks()
        tfs = flop / (gms / 1e3) / 1e12
        bstep = {"metric": "batched decode step tok/s (64 slot threads, one token each through the 40-layer "
                           "stack's Q4_K/Q6_K projections via the step group, one combined call per layer)",
                 "value": round(STEP_SLOTS / (gms / 1e3) * world, 1), "unit": "tok/s",
                 "ms_per_step": round(gms, 4), "wall_ms_per_step": round(r["group_wall_ms"], 4),
                 "steps": a.step_rounds, "gpu_launches": int(r["launches"]), "slots": STEP_SLOTS,
                 "rounds": r["rounds"], "combined_calls": r["calls"], "merged_products": r["products"],
                 "replayed_calls": r["replayed"],
                 "max_round": r["max_round"],
                 "per_slot_form": {"ms_per_step": round(sms, 4),
                                   "value": round(STEP_SLOTS / (sms / 1e3) * world, 1), "unit": "tok/s",
                                   "what": "one kernel_cuda_matvec_quant_batch per slot (all 190 of its "
                                           "projections), slots in turn, as under the reference's step lock"},
                 "data": "synthetic: uniform random k-quant blocks, N(0,1) activations; native pthreads "
                         "(libslot_threads.so) as the slot threads",
                 "roofline": {"bound": "tensor", "kernel": "quant_mm_tc_kernel",
                              "achieved": round(tfs, 2), "peak": tens_p, "unit": "TFLOP/s",
                              "frac": round(tfs / tens_p, 4), "peak_source": f"{src_p} bf16_tflops (burst)",
                              "algorithmic_flop_per_step": flop}}

    long_ctx = None
    if not a.no_long:
        long_ctx = run_long_context(R, torch, dist, dev, stream, world, rank, a.long_window, a.long_steps)
        if world > 1:
            gl = run_long_context(R, torch, dist, dev, stream, world, rank, a.long_window, a.long_steps,
                                  mode="gather")
            long_ctx["nccl_gather_form"] = {k: gl[k] for k in ("value", "ms_per_step", "kv_split")}
        if rank == 0 and world == 1 and not a.no_cpu_baseline:
            try:
                c = cpu_leg_ref("long", window=a.long_window, slots=LONG_SLOTS, timeout=1200)
                long_ctx["cpu_baseline"] = {
                    "value": round(c["tok_s"], 3), "unit": "tok/s", "cores": c["threads"], "kind": "reference",
                    "build": c["build"],
                    "sample": f"2 timed slot-steps of full_attention over {a.long_window} cached tokens (projection "
                              f"matvecs subtracted) + 3 recurrent_delta_step; the reference serves the "
                              f"{LONG_SLOTS} slots in turn, so tok/s = 1 / slot-step time"}
            except Exception as e:  # reported, not fatal
                long_ctx["cpu_baseline"] = {"value": None, "sample": f"failed: {e}"[:300]}

    recur = None
    if not a.no_recurrent and rank == 0:
        # config 1 is one slot: it does not shard; rank 0 runs it on its GPU
        r1 = run_recurrent(R, torch, dev, stream, a.recurrent_steps, 3, not a.no_parity)
        rbytes = RECUR_LAYERS * (32 * 128 * 128 * 4 * 2 + (2 * 2048 + 4096 + 64) * 4 + 4096 * 4)
        hbm_r, _, src_r = peaks()
        gbs_r = rbytes / (r1["ms"] * 1e-3) / 1e9
        recur = {"metric": "recurrent decode tok/s (config 1: 1 slot, 30 Gated DeltaNet layers, sequential steps)",
                 "value": round(1e3 / r1["ms"], 1), "unit": "tok/s", "ms_per_step": round(r1["ms"], 5),
                 "steps": a.recurrent_steps, "warmup": 3, "gpu_launches": int(r1["launches"]),
                 "config": {"workload": "config 1", "layers": RECUR_LAYERS, "slots": 1,
                            "launch": "one kernel_deltanet_step_batch of 30 jobs per step",
                            "l2": "states 63 MB < L2: a 256 MB device write before every timed step, each "
                                  "step timed alone"},
                 "roofline": {"bound": "hbm", "kernel": "deltanet_step_kernel", "achieved": round(gbs_r, 1),
                              "peak": hbm_r, "unit": "GB/s", "frac": round(gbs_r / hbm_r, 4),
                              "peak_source": f"{src_r} hbm_gbs",
                              "algorithmic_bytes_per_step": rbytes,
                              "scope": "state read + write, inputs and outputs of the 30 layers per step"},
                 "scope": "rank 0 only (one slot does not shard)"}
        try:
            lb = run_layer_block(R, torch, dev, stream, a.recurrent_steps, 3)
            recur["layer_block"] = {
                "ms_per_step": round(lb["ms"], 5), "value": round(1e3 / lb["ms"], 1), "unit": "tok/s",
                "extra_ms_vs_recurrence": round(lb["ms"] - r1["ms"], 5),
                "gpu_launches_per_step": round(lb["launches"] / a.recurrent_steps, 2),
                "what": "per step the 30 layers' pre-ops (conv1d + SiLU + L2-norm + beta/g, history shift), "
                        "the recurrence and the gated-RMSNorm post-op: kernel_deltanet_preop_batch + "
                        "kernel_deltanet_step_batch + kernel_deltanet_postop_batch, timed as the recurrence "
                        "alone is (L2 flushed before each step)"}
        except Exception as e:  # reported, not fatal
            recur["layer_block"] = {"ms_per_step": None, "what": f"failed: {e}"[:300]}
        if "parity_file" in r1:
            try:
                pr = cpu_leg("parity1", path=r1["parity_file"], timeout=900)
                recur["parity"] = dict(pr, tolerance=1e-4, **{"pass": max(pr["state_maxrel"], pr["out_maxrel"]) <= 1e-4},
                                       what="layers 0 and 29 over every step (warm-up + timed) from the same "
                                            "initial states, against the reference's recurrence")
            except Exception as e:  # reported, not fatal
                recur["parity"] = {"pass": None, "what": f"failed: {e}"[:300]}
            finally:
                os.unlink(r1["parity_file"])
        if world == 1 and not a.no_cpu_baseline:
            try:
                c = cpu_leg_ref("recurrent", steps=20, timeout=900)
                recur["cpu_baseline"] = {"value": round(c["tok_s"], 3), "unit": "tok/s", "cores": c["threads"],
                                         "kind": "reference", "build": c["build"],
                                         "sample": "20 timed steps (after 1 warm-up) of recurrent_delta_step over "
                                                   "the 30 layers of one slot"}
            except Exception as e:  # reported, not fatal
                recur["cpu_baseline"] = {"value": None, "sample": f"failed: {e}"[:300]}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        try:
            r = cpu_leg_ref("decode", lens=glens, steps=1, warmup=0, budget_s=CPU_BUDGET_S)
            r1 = cpu_leg_ref("decode", lens=glens[:8], steps=1, warmup=0, budget_s=CPU_BUDGET_S, threads=1)
            cpu = {"value": round(r["tok_s"], 3), "unit": "tok/s", "cores": r["threads"],
                   "kind": "reference", "build": r["build"],
                   "sample": f"{r['steps']} step of all {r['slots']} slots (every slot once, windows of this run), "
                             f"reference full_attention minus its projection matvecs "
                             f"({r['projection_ms_subtracted']:.2f} ms) + 3 recurrent_delta_step, "
                             f"OpenMP {r['threads']} threads, slots serialised as in slots.c",
                   "one_thread": {"value": round(r1["tok_s"], 3), "unit": "tok/s", "cores": 1,
                                  "sample": "the same, 1 OpenMP thread, the first 8 slots of the step"}}
        except Exception as e:  # reported, not fatal
            cpu = {"value": None, "unit": "tok/s", "cores": None, "kind": "reference",
                   "sample": f"failed: {e}"[:300]}

    if rank == 0:
        traffic = None if ATTN_TRAFFIC_RATIO is None else round(ATTN_TRAFFIC_RATIO * attn_bytes)
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16 KV / fp32 state",
            "data": "synthetic (seeded N(0,1) KV and inputs; no dataset exists for this path)",
            "config": dict(config2_desc(world, a), mean_kv_len_rank0=round(c2["mean_L"], 1),
                           slots_rank0=c2["n"]),
            "roofline": {"bound": "hbm", "kernel": "attn_decode_kernel",
                         "achieved": round(attn_gbs, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(attn_gbs / hbm, 4), "traffic": traffic,
                         "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured" else src,
                         "algorithmic_bytes_per_launch": round(attn_bytes),
                         "scope": "rank 0's launch against rank 0's own kernel time"},
            "kernels": {
                "attn_decode_kernel": {"ms": round(c2["attn_ms"], 4), "GB/s": round(attn_gbs, 1),
                                       "frac": round(attn_gbs / hbm, 4), "bytes": round(attn_bytes)},
                "deltanet_step_kernel": {"ms": round(c2["dn_ms"], 4), "GB/s": round(dn_gbs, 1),
                                         "frac": round(dn_gbs / hbm, 4), "bytes": round(dn_bytes)},
                "max_over_ranks_ms": {"attn": round(attn_avg, 4), "deltanet": round(dn_avg, 4)}},
            "parity": parity, "e2e": e2e, "cpu_baseline": cpu, "clocks": c2["clocks"],
            "gpu_launches": int(c2["launches"]),
            "shards": shards, "weak_64_per_gpu": weak,
            "prefill": prefill, "long_context": long_ctx, "projections": proj, "prefill_projections": pproj,
            "batched_step": bstep, "recurrent": recur,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(a):
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", 1))
    glens = slot_lengths(1000, a.kv_lo, a.kv_hi)
    r = cpu_leg_ref("decode", lens=glens, steps=max(1, a.steps), warmup=max(0, min(a.warmup, 2)),
                    budget_s=CPU_BUDGET_S, timeout=3600)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(r["tok_s"], 3), "unit": "tok/s",
        "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": round(1e3 * r["seconds"] / r["steps"], 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32 (reference CPU path)",
        "data": "synthetic (seeded)",
        "config": config2_desc(world, a),
        "cpu_baseline": {"value": round(r["tok_s"], 3), "unit": "tok/s", "cores": r["threads"],
                         "kind": "reference", "build": r["build"],
                         "sample": f"{r['steps']} timed steps of the {a.steps} requested (bounded to "
                                   f"{CPU_BUDGET_S:.0f} s of CPU work; min(2, W) warm-up steps), each step = all "
                                   f"{r['slots']} slots once, windows +1 per step as on the GPU: reference "
                                   f"full_attention minus its projection matvecs + 3 recurrent_delta_step; "
                                   f"OpenMP {r['threads']} threads; slots served in turn (slots.c step lock)"},
        "e2e": {"value": round(r["tok_s"], 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    a = args_parse()
    if a.cpu_json:
        print(json.dumps(cpu_main(json.loads(a.cpu_json))))
        return
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
