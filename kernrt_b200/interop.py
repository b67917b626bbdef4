"""Zero-copy torch views of backend buffers (plumbing for tests and the bench).

PyTorch is used here only for device memory plumbing: filling backend buffers
with seeded synthetic data on the device and slicing rows out of them.  The
backend runs on its own non-blocking stream, so callers synchronise (the
backend's ``synchronize`` and ``torch.cuda.synchronize``) around mixed use.
"""
from __future__ import annotations

import numpy as np

_TYPESTR = {np.float32: "<f4", np.int32: "<i4", np.int8: "|i1", np.uint16: "<u2", np.int64: "<i8",
            np.uint8: "|u1"}


class _CudaArray:
    def __init__(self, ptr: int, shape, dtype):
        self.__cuda_array_interface__ = {
            "shape": tuple(int(s) for s in shape),
            "typestr": _TYPESTR[np.dtype(dtype).type],
            "data": (int(ptr), False),
            "version": 3,
            "strides": None,
        }


def as_torch(backend, buf: int, shape, dtype=np.float32, device: int = 0):
    """A torch tensor aliasing the first prod(shape) elements of `buf`."""
    import torch

    return torch.as_tensor(_CudaArray(backend.device_ptr(buf), shape, dtype), device=f"cuda:{device}")
