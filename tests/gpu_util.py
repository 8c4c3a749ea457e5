"""Helpers for the GPU parity tests: numpy <-> device tensors."""
import numpy as np


def dev(x, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()
