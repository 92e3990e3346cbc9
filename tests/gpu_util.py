"""Helpers shared by the GPU tests."""
import numpy as np
import torch


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def misaligned(a):
    """A contiguous CUDA view of `a` starting one element into its storage
    (so 16-byte vector loads are not allowed)."""
    a = np.ascontiguousarray(a)
    flat = np.concatenate([np.zeros((1,) + a.shape[1:], a.dtype), a]) if a.ndim > 1 else \
        np.concatenate([np.zeros(1, a.dtype), a])
    t = cu(flat)
    return t[1:]
