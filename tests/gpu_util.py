"""Helpers for the GPU parity tests: torch for device memory, ctypes into
libxp_cuda.so for the kernels under test."""
import numpy as np
import torch

from xpose_b200._lib import check, lib


# Every tensor handed to the C ABI by pointer is kept alive here until the
# test ends: a temporary would return its block to torch's caching allocator
# before the asynchronous kernel reads it.
_ALIVE = []


def release():
    _ALIVE.clear()


def dev(a):
    """numpy -> CUDA tensor (same dtype, int types via view)."""
    t = _dev(a)
    _ALIVE.append(t)
    return t


def _dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).cuda()
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda()
    if a.dtype == np.uint64:
        return torch.from_numpy(a.view(np.int64)).cuda()
    return torch.from_numpy(a).cuda()


def host(t, dtype=None):
    a = t.detach().cpu().numpy()
    if dtype is not None:
        a = a.view(dtype)
    return a


def empty(n, dtype=torch.float32):
    t = torch.zeros(n, dtype=dtype, device="cuda")
    _ALIVE.append(t)
    return t


def ptr(t):
    return t.data_ptr()


def sync():
    torch.cuda.synchronize()


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
