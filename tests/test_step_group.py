"""Cross-slot batched step (kernel_step_group_*): the batched counterpart of the reference's
per-token step lock (src/slots.c:77-105 FairLock, 864-880 step_forward).

CPU tests drive the rendezvous with host threads and placeholder jobs whose null pointers every
batch entry point rejects on the host (-1, no device work, on any machine); they check how calls
combine into rounds and batches through the group's counters. GPU tests run real slots through
the group and compare with the same slots run one call per slot, as the reference's step lock
does: attention (gated GQA decode, model.c:801-861) within 2e-3 like its oracle tests, the
DeltaNet step and the projections (kernels.c:405-431, 553-578) within 1e-5."""
import threading
import time

import numpy as np
import pytest

import roaster_b200 as R


def _run(n, fn):
    """Run fn(i) on n threads; return the results, re-raising the first failure."""
    res, err = [None] * n, []

    def body(i):
        try:
            res[i] = fn(i)
        except BaseException as e:   # noqa: BLE001 - surfaced below
            err.append(e)

    ts = [threading.Thread(target=body, args=(i,)) for i in range(n)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(60)
    assert not any(t.is_alive() for t in ts), "a member thread did not finish"
    if err:
        raise err[0]
    return res


def _mv(matrix, rows=64):
    return R.KernelCudaMatvecJob(0, matrix, 0, 0, rows, 256)   # null vector/output: rejected


def test_rounds_combine_every_call():
    """All members of a round meet at each call; one batch per call carries every member's job,
    and projections on a shared matrix are planned as one multi-token product."""
    M, ROUNDS = 4, 3
    g = R.StepGroup(M, straggler_us=5_000_000)
    ids = [g.join() for _ in range(M)]
    sizes = []

    def member(i):
        m = ids[i]
        for _ in range(ROUNDS):
            sizes.append(g.begin(m))
            assert g.attn(m, 0, R.KernelAttnDecodeJob()) == -1         # placeholder job
            assert g.delta(m, 1, R.KernelDeltaStepJob()) == -1
            assert g.matvec(m, 2, [_mv(0x1000), _mv(0x2000), _mv(0x3000 + 0x100 * i)]) == -1
            assert g.end(m) == 0

    _run(M, member)
    st = g.stats()
    assert sizes == [M] * (M * ROUNDS)
    assert st["rounds"] == ROUNDS and st["max_round"] == M
    assert st["calls"] == 3 * ROUNDS
    assert st["jobs"] == ROUNDS * (M + M + 3 * M)
    assert st["products"] == 2 * ROUNDS            # the two shared matrices, once per round
    assert st["merged_jobs"] == 2 * M * ROUNDS     # private matrices stay single-token
    assert st["errors"] == 3 * ROUNDS
    for m in ids:
        assert g.leave(m) == 0
    assert g.stats()["members"] == 0
    g.close()


def test_straggler_takes_next_round():
    """A round forms after the straggler limit with the members that have begun."""
    g = R.StepGroup(3, straggler_us=300_000)
    a, b, c = g.join(), g.join(), g.join()
    got = {}

    def member(i):
        m = (a, b, c)[i]
        if m == c:
            time.sleep(1.5)
        got[m] = g.begin(m)
        assert g.attn(m, 7, R.KernelAttnDecodeJob()) == -1
        assert g.end(m) == 0
        if m != c:
            assert g.leave(m) == 0

    _run(3, member)
    assert got[a] == 2 and got[b] == 2 and got[c] == 1
    st = g.stats()
    assert st["rounds"] == 2 and st["calls"] == 2 and st["jobs"] == 3
    g.close()


def test_mismatched_call_sites_fail_the_round():
    g = R.StepGroup(2, straggler_us=5_000_000, call_timeout_ms=5000)
    ids = [g.join(), g.join()]
    out = {}

    def member(i):
        m = ids[i]
        assert g.begin(m) == 2
        if i == 1:
            time.sleep(0.1)                  # member 0 opens site 0 first
        out[(i, "first")] = g.attn(m, i, R.KernelAttnDecodeJob())
        out[(i, "second")] = g.delta(m, 5, R.KernelDeltaStepJob())
        assert g.end(m) == 0

    _run(2, member)
    assert out[(0, "first")] == -1 and out[(1, "first")] == -1
    assert out[(0, "second")] == -1 and out[(1, "second")] == -1
    st = g.stats()
    assert st["calls"] == 0 and st["errors"] == 1

    # the next round is clean again: its calls run (and fail only on the placeholder jobs)
    def again(i):
        assert g.begin(ids[i]) == 2
        assert g.delta(ids[i], 5, R.KernelDeltaStepJob()) == -1
        assert g.end(ids[i]) == 0

    _run(2, again)
    assert g.stats()["calls"] == 1
    g.close()


def test_call_timeout_is_bounded():
    """A member that never reaches a call fails it for the others after the call timeout."""
    g = R.StepGroup(2, straggler_us=5_000_000, call_timeout_ms=200)
    a, b = g.join(), g.join()
    t = {}

    def member(i):
        m = (a, b)[i]
        assert g.begin(m) == 2
        if i == 0:
            t0 = time.monotonic()
            t["rc"] = g.attn(m, 0, R.KernelAttnDecodeJob())
            t["dt"] = time.monotonic() - t0
            t["msg"] = R.last_error()
        else:
            time.sleep(0.6)
        assert g.end(m) == 0

    _run(2, member)
    assert t["rc"] == -1 and 0.15 < t["dt"] < 5.0
    st = g.stats()
    assert st["calls"] == 0 and st["errors"] == 1
    g.close()


def test_member_ending_early_releases_the_call():
    """A member that ends its step early (its slot failed) does not hold up the others: the
    open call runs as soon as every member still in the round has reached it."""
    g = R.StepGroup(3, straggler_us=5_000_000, call_timeout_ms=20000)
    ids = [g.join() for _ in range(3)]

    def member(i):
        m = ids[i]
        assert g.begin(m) == 3
        if i == 2:
            time.sleep(0.2)
            assert g.end(m) == 0
            return None
        t0 = time.monotonic()
        rc = g.attn(m, 3, R.KernelAttnDecodeJob())
        assert g.end(m) == 0
        return rc, time.monotonic() - t0

    res = _run(3, member)
    for rc, dt in res[:2]:
        assert rc == -1 and dt < 10.0
    st = g.stats()
    assert st["calls"] == 1 and st["jobs"] == 2
    g.close()


def test_membership_rules():
    g = R.StepGroup(2)
    a, b = g.join(), g.join()
    with pytest.raises(RuntimeError):
        g.join()                                           # full
    assert g.attn(a, 0, R.KernelAttnDecodeJob()) == -1    # not in a round
    assert "not in a round" in R.last_error()
    assert g.end(a) == -1
    assert g.leave(b) == 0
    assert g.begin(a) == 1                                 # alone: the round forms at once
    assert g.begin(a) == -1                                # already begun
    assert g.leave(a) == -1                                # inside a round
    assert g.end(a) == 0
    assert g.leave(a) == 0
    assert g.leave(a) == -1
    assert R.lib().kernel_step_group_create(0, 0, 1) is None
    g.close()


def test_fifo_lock_serves_in_arrival_order():
    g = R.StepGroup(1)
    order = []
    g.lock()

    def taker(i):
        time.sleep(0.1 * i)                  # arrive in index order while the lock is held
        g.lock()
        order.append(i)
        g.unlock()

    ts = [threading.Thread(target=taker, args=(i,)) for i in range(4)]
    for t in ts:
        t.start()
    time.sleep(0.7)
    g.unlock()
    for t in ts:
        t.join(10)
    assert order == [0, 1, 2, 3]
    g.close()


def test_many_members_many_rounds():
    M, ROUNDS, CALLS = 12, 8, 5
    g = R.StepGroup(M, straggler_us=10_000_000)
    ids = [g.join() for _ in range(M)]
    rng = np.random.default_rng(0)
    delays = rng.uniform(0, 0.003, size=(M, ROUNDS, CALLS))

    def member(i):
        m = ids[i]
        for r in range(ROUNDS):
            assert g.begin(m) == M
            for c in range(CALLS):
                time.sleep(delays[i, r, c])
                assert g.delta(m, c, R.KernelDeltaStepJob()) == -1
            assert g.end(m) == 0

    _run(M, member)
    st = g.stats()
    assert st["rounds"] == ROUNDS and st["calls"] == ROUNDS * CALLS and st["jobs"] == ROUNDS * CALLS * M
    g.close()


def test_members_ending_at_random_points():
    """Members end their step after a random number of calls (a slot whose step failed). The
    others never wait for them: call c of a round runs once, as soon as every member still in
    the round has reached it, so a round runs max(calls made) batches carrying sum(calls made)."""
    M, ROUNDS, CALLS = 32, 20, 6
    g = R.StepGroup(M, straggler_us=10_000_000, call_timeout_ms=20000)
    ids = [g.join() for _ in range(M)]
    rng = np.random.default_rng(1)
    made = rng.integers(0, CALLS + 1, size=(ROUNDS, M))
    made[:, 0] = CALLS                      # at least one member makes every call
    jitter = rng.uniform(0, 0.002, size=(ROUNDS, M))

    def member(i):
        m = ids[i]
        for r in range(ROUNDS):
            assert g.begin(m) == M
            for c in range(int(made[r, i])):
                if c == 2:
                    time.sleep(jitter[r, i])
                assert g.delta(m, c, R.KernelDeltaStepJob()) == -1
            assert g.end(m) == 0

    _run(M, member)
    st = g.stats()
    assert st["rounds"] == ROUNDS
    assert st["calls"] == ROUNDS * CALLS
    assert st["jobs"] == int(made.sum())
    g.close()


# ----------------------------------------------------------------------------------- GPU

def _slots(torch, n, seed):
    from roaster_b200 import synth
    from tests.gpu_util import dev
    slots = []
    for i in range(n):
        d = synth.attn_decode_inputs(seed=seed + i, length=100 + 37 * i, position=100 + 37 * i)
        L = d["length"]
        kc = torch.zeros(L + 8, 2, 256, dtype=torch.float16, device="cuda")
        vc = torch.zeros_like(kc)
        kc[:L] = dev(d["k_cache"])
        vc[:L] = dev(d["v_cache"])
        st = dev(synth.delta_state(seed + 100 + i, 1)[0])
        seq = {k: dev(v[0, 0]) for k, v in synth.delta_sequence(seed + 200 + i, 1, 1).items()}
        slots.append({"d": d, "kc": kc, "vc": vc, "q": dev(d["q"]), "gate": dev(d["gate"]),
                      "k_new": dev(d["k_new"]), "v_new": dev(d["v_new"]), "q_norm": dev(d["q_norm"]),
                      "k_norm": dev(d["k_norm"]), "out": torch.zeros(16, 256, device="cuda"),
                      "state": st, "seq": seq, "dout": torch.zeros(32, 128, device="cuda")})
    return slots


def _clone(torch, slots):
    return [{k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in s.items()} for s in slots]


def _jobs(s):
    d = s["d"]
    a = R.attn_job(s["q"], s["gate"], s["k_new"], s["v_new"], s["q_norm"], s["k_norm"], s["kc"], s["vc"],
                   d["length"], d["position"], s["out"])
    q = s["seq"]
    dj = R.delta_job(s["state"], q["q"], q["k"], q["v"], q["g"], q["beta"], s["dout"])
    return a, dj


@pytest.mark.gpu
def test_group_step_matches_per_slot_step(rb, oracle_lib):
    """8 slots decode one token through the group (attention, DeltaNet, and 4 projections of
    which 3 share their weights across slots, two of those also reading the same input vector,
    like a layer's q and k); the same slots run one call per slot as under the reference's step
    lock. Same results; the shared projections ran as multi-token products."""
    import torch
    import oracle as O
    from roaster_b200 import synth
    from tests.gpu_util import dev, host
    N = 8
    base = _slots(torch, N, 11)
    ref = _clone(torch, base)
    shared = [(False, synth.quant_matrix(1, 512, 2048, False), 512, 2048),
              (True, synth.quant_matrix(2, 256, 1024, True), 256, 1024),
              (False, synth.quant_matrix(3, 256, 2048, False), 256, 2048)]
    xin = [0, 1, 0]                          # the third matrix reads the first one's input
    dshared = [(q6, dev(m), r, c) for q6, m, r, c in shared]
    priv = [dev(synth.quant_matrix(30 + i, 96, 512, False)) for i in range(N)]
    rng = np.random.default_rng(5)
    xs = [[dev(rng.standard_normal(c).astype(np.float32)) for c in (2048, 1024, 512)] for _ in range(N)]

    def mv_jobs(i, outs):
        js = [(q6, m, xs[i][xin[k]], outs[k], r, c) for k, (q6, m, r, c) in enumerate(dshared)]
        js.append((False, priv[i], xs[i][2], outs[3], 96, 512))
        return js

    g_out = [[torch.zeros(r, device="cuda") for (_, _, r, _) in dshared] + [torch.zeros(96, device="cuda")]
             for _ in range(N)]
    r_out = [[torch.zeros_like(t) for t in o] for o in g_out]
    torch.cuda.synchronize()

    # one call per slot, serialised
    for i, s in enumerate(ref):
        a, dj = _jobs(s)
        rb.attn_decode_batch([a])
        rb.deltanet_step_batch([dj])
        rb.matvec_quant_batch(mv_jobs(i, r_out[i]))
    torch.cuda.synchronize()

    g = R.StepGroup(N, straggler_us=5_000_000)
    ids = [g.join() for _ in range(N)]

    def member(i):
        m = ids[i]
        a, dj = _jobs(base[i])
        assert g.begin(m) == N
        assert g.attn(m, 0, a) == 0, R.last_error()
        assert g.delta(m, 1, dj) == 0, R.last_error()
        assert g.matvec(m, 2, mv_jobs(i, g_out[i])) == 0, R.last_error()
        assert g.end(m) == 0

    _run(N, member)
    rb.synchronize()
    st = g.stats()
    assert st["calls"] == 3 and st["jobs"] == N * 6 and st["errors"] == 0
    assert st["products"] == 3 and st["merged_jobs"] == 3 * N
    for s, r in zip(base, ref):
        assert O.maxrel(host(s["out"]), host(r["out"])) <= 2e-3
        L = s["d"]["length"]
        assert torch.equal(s["vc"][L], r["vc"][L])
        assert O.maxrel(host(s["dout"]), host(r["dout"])) <= 1e-5
        assert O.maxrel(host(s["state"]), host(r["state"])) <= 1e-5
    for i in range(N):
        for a, b in zip(g_out[i], r_out[i]):
            assert O.maxrel(host(a), host(b)) <= 1e-5
    # and against the reference's own matvec for one slot's shared projection
    for k in (0, 2):                         # both readers of the shared input block
        q6, m, r, c = shared[k]
        want = O.matvec_q(q6, m, host(xs[3][0]), r, c, impl="ref" if O.have_ref() else "port")
        assert O.maxrel(host(g_out[3][k]), want) <= 1e-5
    for m_ in ids:
        g.leave(m_)
    g.close()


@pytest.mark.gpu
def test_group_rounds_over_tokens(rb, oracle_lib):
    """Several tokens in a row: DeltaNet states advance through group rounds exactly as through
    per-slot steps (the state carries every earlier round's result)."""
    import torch
    import oracle as O
    from roaster_b200 import synth
    from tests.gpu_util import dev, host
    N, T = 6, 5
    st0 = [synth.delta_state(40 + i, 1)[0] for i in range(N)]
    seqs = [synth.delta_sequence(60 + i, T, 1) for i in range(N)]
    dst = [dev(s) for s in st0]
    dseq = [{k: dev(v[:, 0]) for k, v in s.items()} for s in seqs]
    outs = [torch.zeros(T, 32, 128, device="cuda") for _ in range(N)]
    g = R.StepGroup(N, straggler_us=5_000_000)
    ids = [g.join() for _ in range(N)]
    torch.cuda.synchronize()

    def member(i):
        m = ids[i]
        for t in range(T):
            q = dseq[i]
            assert g.begin(m) == N
            rc = g.delta(m, 0, R.delta_job(dst[i], q["q"][t], q["k"][t], q["v"][t], q["g"][t], q["beta"][t],
                                           outs[i][t]))
            assert rc == 0, R.last_error()
            assert g.end(m) == 0

    _run(N, member)
    rb.synchronize()
    assert g.stats()["rounds"] == T and g.stats()["calls"] == T
    for i in range(N):
        st = st0[i].copy()
        ref = O.delta_prefill(st, seqs[i]["q"][:, 0], seqs[i]["k"][:, 0], seqs[i]["v"][:, 0], seqs[i]["g"][:, 0],
                              seqs[i]["beta"][:, 0])
        assert O.maxrel(host(dst[i]), st) < 1e-4
        assert O.maxrel(host(outs[i]), ref) < 1e-4
    g.close()


@pytest.mark.gpu
def test_group_projections_recorded_and_replayed(rb, oracle_lib):
    """Projection calls whose job lists repeat are recorded and replayed. Each slot feeds its
    output back as its next input (buffers A and B in turn, so two job lists alternate; a second
    matrix reads the same input into C): over 6 tokens each list runs once plain, once recorded
    and once replayed, with new values every token. The final buffers match the same chain run
    one call per slot."""
    import torch
    import oracle as O
    from roaster_b200 import synth
    from tests.gpu_util import dev, host
    N, T = 8, 6
    w4 = dev(synth.quant_matrix(71, 512, 512, False))
    w6 = dev(synth.quant_matrix(72, 256, 512, True))
    rng = np.random.default_rng(9)
    x0 = [rng.standard_normal(512).astype(np.float32) for _ in range(N)]

    def buffers():
        return [{"A": dev(x0[i]), "B": torch.zeros(512, device="cuda"), "C": torch.zeros(256, device="cuda")}
                for i in range(N)]

    def jobs(b, t):
        src, dst = (b["A"], b["B"]) if t % 2 == 0 else (b["B"], b["A"])
        return [(False, w4, src, dst, 512, 512), (True, w6, src, b["C"], 256, 512)]

    ref = buffers()
    for t in range(T):
        for i in range(N):
            rb.matvec_quant_batch(jobs(ref[i], t))
    grp = buffers()
    torch.cuda.synchronize()
    g = R.StepGroup(N, straggler_us=5_000_000)
    ids = [g.join() for _ in range(N)]

    def member(i):
        for t in range(T):
            assert g.begin(ids[i]) == N
            assert g.matvec(ids[i], t % 2, jobs(grp[i], t)) == 0, R.last_error()
            assert g.end(ids[i]) == 0

    _run(N, member)
    rb.synchronize()
    st = g.stats()
    assert st["calls"] == T and st["errors"] == 0 and st["products"] == 2 * T
    assert st["replayed"] == 2                   # the third occurrence of each list
    for i in range(N):
        for k in ("A", "B", "C"):
            assert O.maxrel(host(grp[i][k]), host(ref[i][k])) <= 1e-4, (i, k)
    for m in ids:
        g.leave(m)
    g.close()


@pytest.mark.gpu
def test_group_projections_in_place_at_64_members(rb, oracle_lib):
    """64 members (the batched step's size): the merged products take the tensor-core path and
    read each member's vector and write each member's output in place (per-token row tables, no
    gather or scatter). Three rounds of the same job lists run plain, recorded and replayed;
    every round's outputs match one call per slot."""
    import torch
    import oracle as O
    from roaster_b200 import synth
    from tests.gpu_util import dev, host
    N, ROUNDS = 64, 3
    w4 = dev(synth.quant_matrix(81, 8192, 2048, False))
    w6 = dev(synth.quant_matrix(82, 512, 2048, True))
    rng = np.random.default_rng(12)
    xs = [dev(rng.standard_normal(2048).astype(np.float32)) for _ in range(N)]

    def jobs(i, outs):
        return [(False, w4, xs[i], outs[0], 8192, 2048), (True, w6, xs[i], outs[1], 512, 2048)]

    ref = [(torch.zeros(8192, device="cuda"), torch.zeros(512, device="cuda")) for _ in range(N)]
    for i in range(N):
        rb.matvec_quant_batch(jobs(i, ref[i]))
    got = [(torch.zeros(8192, device="cuda"), torch.zeros(512, device="cuda")) for _ in range(N)]
    torch.cuda.synchronize()
    g = R.StepGroup(N, straggler_us=20_000_000)
    ids = [g.join() for _ in range(N)]
    errs = []

    def member(i):
        for _ in range(ROUNDS):
            for t in got[i]:                 # the replayed round must write them again
                t.zero_()
            assert g.begin(ids[i]) == N
            assert g.matvec(ids[i], 0, jobs(i, got[i])) == 0, R.last_error()
            assert g.end(ids[i]) == 0

    _run(N, member)
    rb.synchronize()
    st = g.stats()
    assert st["calls"] == ROUNDS and st["errors"] == 0 and st["products"] == 2 * ROUNDS
    assert st["replayed"] == 1
    for i in range(N):
        for a, b in zip(got[i], ref[i]):
            errs.append(O.maxrel(host(a), host(b)))
    assert max(errs) <= 1e-5, max(errs)
    for m in ids:
        g.leave(m)
    g.close()


@pytest.mark.gpu
def test_group_recording_not_replayed_after_the_scratch_moves(rb, oracle_lib):
    """A recording points into the library's scratch. Between rounds the library's buffers are
    released (kernel_cuda_trim_scratch, under the group's lock); the next occurrence of the job list
    must be recorded again, not replayed into freed memory. Every round's outputs (zeroed before
    it) match one call per slot."""
    import torch
    import oracle as O
    from roaster_b200 import synth
    from tests.gpu_util import dev, host
    N = 8
    w4 = dev(synth.quant_matrix(91, 512, 1024, False))
    rng = np.random.default_rng(13)
    xs = [dev(rng.standard_normal(1024).astype(np.float32)) for _ in range(N)]
    ref = [torch.zeros(512, device="cuda") for _ in range(N)]
    for i in range(N):
        rb.matvec_quant_batch([(False, w4, xs[i], ref[i], 512, 1024)])
    got = [torch.zeros(512, device="cuda") for _ in range(N)]
    torch.cuda.synchronize()
    g = R.StepGroup(N, straggler_us=5_000_000)
    ids = [g.join() for _ in range(N)]

    def rounds(n):
        def member(i):
            for _ in range(n):
                got[i].zero_()
                assert g.begin(ids[i]) == N
                assert g.matvec(ids[i], 0, [(False, w4, xs[i], got[i], 512, 1024)]) == 0, R.last_error()
                assert g.end(ids[i]) == 0
        _run(N, member)
        rb.synchronize()
        for i in range(N):
            assert O.maxrel(host(got[i]), host(ref[i])) <= 1e-5

    rounds(3)                                    # plain, recorded, replayed
    assert g.stats()["replayed"] == 1
    g.lock()                                     # the library frees its scratch and staging
    rb.lib().kernel_cuda_trim_scratch()
    g.unlock()
    rb.synchronize()
    rounds(3)                                    # plain (it allocates), recorded again, replayed
    assert g.stats()["replayed"] == 2 and g.stats()["errors"] == 0
    for m in ids:
        g.leave(m)
    g.close()
