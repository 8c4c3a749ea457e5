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
"""
from __future__ import annotations

PARTIAL_FLOATS = 8 + 8 + 8 * 256


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
