"""Split-KV long-context decode host logic over a 2-rank gloo process group (CPU).

Each rank holds one contiguous slice of the window (roaster_b200.splitkv.slice_bounds); the rank
with the newest slice appends the new token. Partials come from the CPU oracle (stand-in for
kernel_attn_decode_partial_batch), are all-gathered over gloo and merged with the same formula as
kernel_attn_merge_partials; the result must equal one decode over the whole window."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

LOG2E = 1.4426950408889634


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, L, outdir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import torch.distributed as dist

    import oracle as O
    from roaster_b200 import splitkv, synth
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    d = synth.attn_decode_inputs(seed=21, length=L)
    _, k_app, v_app = O.attn_decode(d["q"], d["gate"], d["k_new"], d["v_new"], d["q_norm"],
                                    d["k_norm"], d["k_cache"], d["v_cache"], L, L)
    lo, hi = splitkv.slice_bounds(L, world, rank)
    kc = d["k_cache"][lo:hi]
    vc = d["v_cache"][lo:hi]
    if splitkv.appends(world, rank):                 # the newest slice takes the new token
        kc = np.concatenate([kc, k_app[None].astype(np.float16)])
        vc = np.concatenate([vc, v_app[None].astype(np.float16)])

    def partial_fn():
        m, l, o = O.attn_decode_partial(d["q"], d["q_norm"], kc, vc, 0, len(kc), L)
        rec = np.zeros((1, 2, splitkv.PARTIAL_FLOATS), np.float32)
        for kvh in range(2):
            hs = slice(8 * kvh, 8 * kvh + 8)
            rec[0, kvh, :8] = m[hs] * LOG2E
            rec[0, kvh, 8:16] = l[hs]
            rec[0, kvh, 16:] = o[hs].reshape(-1)
        return rec

    def gather_fn(local):
        t = torch.from_numpy(local)
        out = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        return np.stack([x.numpy() for x in out])

    def merge_fn(g, w):
        return splitkv.merge_reference(g, d["gate"][None])

    out = splitkv.step(world, partial_fn, gather_fn, merge_fn)
    np.save(os.path.join(outdir, f"out{rank}.npy"), out)
    dist.destroy_process_group()


@pytest.mark.parametrize("L", [1000, 4099])
def test_two_rank_split_decode_equals_single_window(tmp_path, L):
    import oracle as O
    from roaster_b200 import synth
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, L, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    d = synth.attn_decode_inputs(seed=21, length=L)
    ref, _, _ = O.attn_decode(d["q"], d["gate"], d["k_new"], d["v_new"], d["q_norm"], d["k_norm"],
                              d["k_cache"], d["v_cache"], L, L)
    for r in range(2):
        got = np.load(tmp_path / f"out{r}.npy")[0]
        assert O.maxrel(got, ref) < 2e-3, O.maxrel(got, ref)


def test_slice_bounds_cover_window():
    from roaster_b200 import splitkv
    for L in (1, 7, 262144, 262147):
        for world in (1, 2, 4, 8):
            spans = [splitkv.slice_bounds(L, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == L
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert sum(splitkv.appends(world, r) for r in range(world)) == 1


def _dying_worker(rank, world, port, outdir):
    """Rank 1 dies before the partial gather; rank 0 must get an error, not hang."""
    import datetime
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        os._exit(3)                                    # a rank lost between steps
    t = torch.ones(4)
    out = [torch.zeros(4) for _ in range(world)]
    try:
        dist.all_gather(out, t)
        result = "no error"
    except Exception as e:                             # the survivor sees the failure
        result = "error: " + type(e).__name__
    with open(os.path.join(outdir, "rank0.txt"), "w") as f:
        f.write(result)
    os._exit(0)


def test_lost_rank_surfaces_as_error(tmp_path):
    import time
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    t0 = time.time()
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert time.time() - t0 < 90
    assert procs[1].exitcode == 3
    assert procs[0].exitcode == 0
    assert open(tmp_path / "rank0.txt").read().startswith("error")



def test_push_layout_covers_every_record_once():
    """The fused form's buffer layout (CPU): for every world size up to 8 and both parity
    halves, the records all ranks push land at distinct addresses inside their home rank's
    buffer, exactly at the places that rank's merge view reads, and a numpy merge over those
    views equals the merge of the gathered form."""
    from roaster_b200 import splitkv
    PF = splitkv.PARTIAL_FLOATS
    rng = np.random.default_rng(3)
    for world in range(1, 9):
        for n_slots in (1, 5, 16):
            bases = [(r + 1) << 32 for r in range(world)]           # disjoint fake address spaces
            tbases = [(r + 1) << 40 for r in range(world)]
            for epoch in (1, 2):
                seen = set()
                bufs = [np.zeros(splitkv.recv_floats(n_slots, world, r), np.float32) for r in range(world)]
                part = rng.standard_normal((world, n_slots, 2, PF)).astype(np.float32)
                part[..., :8] = rng.standard_normal((world, n_slots, 2, 8))
                part[..., 8:16] = rng.uniform(0.5, 2.0, (world, n_slots, 2, 8))
                for r in range(world):
                    dst, tags = splitkv.push_targets(n_slots, world, r, epoch, bases, tbases)
                    for s in range(n_slots):
                        h = splitkv.home_of(s, world)
                        off = dst[s] - bases[h]
                        assert off % 16 == 0 and (dst[s], tags[s]) not in seen
                        seen.add((dst[s], tags[s]))
                        fo = off // 4
                        assert 0 <= fo and fo + 2 * PF <= bufs[h].size
                        tw = (tags[s] - tbases[h]) // 4
                        assert tw % (2 * splitkv.TAGS_PER_RECORD) == 0
                        assert tw + 2 * splitkv.TAGS_PER_RECORD <= splitkv.tag_words(n_slots, world, h)
                        bufs[h][fo:fo + 2 * PF] = part[r, s].reshape(-1)
                gates = rng.standard_normal((n_slots, 16, 256)).astype(np.float32)
                want = splitkv.merge_reference(part, gates)
                for h in range(world):
                    mine = splitkv.home_slots(n_slots, world, h)
                    if not mine:
                        continue
                    rv, _ = splitkv.merge_view(n_slots, world, h, epoch, bases[h], tbases[h])
                    fo = (rv - bases[h]) // 4
                    view = bufs[h][fo:fo + world * len(mine) * 2 * PF].reshape(world, len(mine), 2, PF)
                    got = splitkv.merge_reference(view, gates[mine])
                    assert np.allclose(got, want[mine], rtol=1e-5, atol=1e-6)
