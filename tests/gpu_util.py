"""Host<->device helpers for the GPU tests (torch supplies device memory only)."""
import numpy as np


def dev(a):
    """numpy array -> contiguous CUDA tensor with the same bytes."""
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a.copy()).cuda()


def host(t, dtype=None):
    """CUDA tensor -> numpy (optionally reinterpreted as dtype)."""
    a = t.detach().cpu().numpy()
    return a.view(dtype) if dtype is not None else a


def empty(nbytes_or_shape, dtype):
    import torch
    return torch.empty(nbytes_or_shape, dtype=dtype, device="cuda")
