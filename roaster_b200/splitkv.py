"""Long-context decode with each slot's KV window split across GPUs (host side).

Each rank of a process group holds one contiguous slice of every slot's window (positions
``slice_bounds``); the rank holding the newest slice is the only one that appends the decoded
token. One step is:

1. every rank computes, per (slot, kv head), one softmax partial over its slice
   (``kernel_attn_decode_partial_batch``: m = max score in log2 units, l = sum of exp2(s - m),
   o = output normalised by l; the appending rank also folds in the new token);
2. one all-gather of the partial buffers (``KERNEL_ATTN_PARTIAL_FLOATS`` floats per slot and kv
   head, 8.3 KB) over NCCL;
3. every rank merges the gathered partials and applies the gate
   (``kernel_attn_merge_partials``): M = max m_i, w_i = l_i 2^(m_i - M), o = sum w_i o_i / sum w_i.

The operations are passed in, so the same host logic runs with the CUDA kernels + NCCL and, in
tests, with CPU stand-ins over gloo.

Fused form (``push_step``), with no collective call in the step: each slot has a home rank
(``home_of``). Every rank's partial kernel writes the slot's record straight into the home
rank's receive buffer (peer stores over NVLink into memory opened through CUDA IPC) and then
sets a tag word to the step's epoch; the home rank's merge kernel waits on the tags of its own
slots only, merges and gates. The receive buffer of a rank holds two halves (step parity), each
``[world][n_home][2][PARTIAL_FLOATS]`` floats, plus tags ``[2][world][n_home][2][8]`` (one per
record and query head): a rank can be
at most one step ahead of a home rank that has not merged yet, so a half is never overwritten
before it is read.
"""
from __future__ import annotations

PARTIAL_FLOATS = 8 + 8 + 8 * 256
TAGS_PER_RECORD = 8             # one release tag per query head of a pushed record


def slice_bounds(window: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous slice [lo, hi) of a window of `window` positions held by `rank`; the last rank
    takes the remainder and owns appends."""
    per = window // world
    lo = rank * per
    hi = window if rank == world - 1 else lo + per
    return lo, hi


def appends(world: int, rank: int) -> bool:
    """Whether `rank` holds the newest slice (appends the new token and scores it)."""
    return rank == world - 1


def step(world: int, partial_fn, gather_fn, merge_fn):
    """Run one split-KV decode step.

    partial_fn() -> local partial buffer [n_slots, 2, PARTIAL_FLOATS] (this rank's slices)
    gather_fn(local) -> gathered buffer [world, n_slots, 2, PARTIAL_FLOATS] (rank order)
    merge_fn(gathered, world) -> gated outputs
    """
    local = partial_fn()
    gathered = local if world == 1 else gather_fn(local)
    return merge_fn(gathered, world)


def merge_reference(gathered, gates):
    """numpy statement of the merge (for checks): gathered [P, n, 2, PF], gates [n, 16, 256]."""
    import numpy as np
    g = np.asarray(gathered, np.float64)
    P, n = g.shape[0], g.shape[1]
    out = np.zeros((n, 16, 256))
    for j in range(n):
        for kvh in range(2):
            m = g[:, j, kvh, :8]
            l = g[:, j, kvh, 8:16]
            o = g[:, j, kvh, 16:].reshape(P, 8, 256)
            M = m.max(axis=0)
            w = np.where(np.isneginf(m), 0.0, l * np.exp2(m - M))
            L = w.sum(axis=0)
            acc = (w[:, :, None] * o).sum(axis=0)
            res = np.where(L[:, None] > 0, acc / np.where(L[:, None] > 0, L[:, None], 1), 0.0)
            gate = np.asarray(gates[j], np.float64)[8 * kvh:8 * kvh + 8]
            out[j, 8 * kvh:8 * kvh + 8] = res / (1.0 + np.exp(-gate))
    return out.astype(np.float32)


# ----------------------------------------------------------------------------- fused (push) form

def home_of(slot: int, world: int) -> int:
    """Rank that merges (and owns the recurrent layers of) `slot`."""
    return slot % world


def home_slots(n_slots: int, world: int, rank: int) -> list[int]:
    """Slots whose home is `rank`, in the order of that rank's receive buffer."""
    return [s for s in range(n_slots) if home_of(s, world) == rank]


def home_count(n_slots: int, world: int, rank: int) -> int:
    """Slots whose home is `rank` (the `n` of its receive buffer)."""
    return len(home_slots(n_slots, world, rank))


def recv_floats(n_slots: int, world: int, rank: int) -> int:
    """Floats of `rank`'s receive buffer (both parity halves)."""
    return 2 * world * home_count(n_slots, world, rank) * 2 * PARTIAL_FLOATS


def tag_words(n_slots: int, world: int, rank: int) -> int:
    """Tag words of `rank`'s receive buffer (both parity halves; one per record and query head)."""
    return 2 * world * home_count(n_slots, world, rank) * 2 * TAGS_PER_RECORD


def push_targets(n_slots: int, world: int, rank: int, epoch: int, recv_bases, tag_bases):
    """Per slot, where `rank` writes its records this step: (record address, tag address) in the
    home rank's buffers (recv_bases / tag_bases: device addresses of every rank's receive buffer
    and tags, this rank's own included), in the half of the step's parity."""
    half = epoch & 1
    dst, tags = [], []
    for s in range(n_slots):
        h = home_of(s, world)
        nh = home_count(n_slots, world, h)
        i = home_slots(n_slots, world, h).index(s)
        rec = ((half * world + rank) * nh + i) * 2
        dst.append(recv_bases[h] + rec * PARTIAL_FLOATS * 4)
        tags.append(tag_bases[h] + rec * TAGS_PER_RECORD * 4)
    return dst, tags


def merge_view(n_slots: int, world: int, rank: int, epoch: int, recv_base: int, tag_base: int):
    """(records, tags) addresses of `rank`'s half for the step's parity: records
    [world][n_home][2][PARTIAL_FLOATS], tags [world][n_home][2][8]."""
    nh = home_count(n_slots, world, rank)
    half = epoch & 1
    return (recv_base + half * world * nh * 2 * PARTIAL_FLOATS * 4,
            tag_base + half * world * nh * 2 * TAGS_PER_RECORD * 4)


def push_step(push_fn, merge_fn):
    """One fused split-KV step: push_fn() writes this rank's partials of every slot to the home
    ranks (and sets the tags); merge_fn() merges this rank's home slots once all tags arrive."""
    push_fn()
    return merge_fn()
