"""Helpers for the gpu tests: host <-> device copies and per-item slicing of
batched (ragged) tensors, following the layouts of include/pkcuda.h."""
from __future__ import annotations

import numpy as np

D, H, DH, FF = 1024, 8, 128, 4096


# Device tensors made by dev()/empty() stay referenced until the end of the
# test (conftest clears this list): an expression like dev(a).data_ptr()
# would otherwise free the block at once and torch's caching allocator would
# hand the same memory to the next operand.
ALIVE = []


def dev(a):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    ALIVE.append(t)
    return t


def empty(shape, dtype=None):
    import torch
    t = torch.empty(shape, dtype=dtype or torch.float32, device="cuda")
    ALIVE.append(t)
    return t


class _DeviceView:
    """A device address seen as a 1-D array (the CUDA array interface)."""

    def __init__(self, ptr, n, dtype):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": np.dtype(dtype).str,
                                         "data": (int(ptr), False), "version": 3}


def from_device(ptr, n, dtype):
    """Host copy of n elements of dtype at a device address owned elsewhere."""
    import torch
    t = torch.as_tensor(_DeviceView(ptr, n, dtype), device="cuda")
    torch.cuda.synchronize()
    return t.cpu().numpy().copy()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


class Layout:
    """Offsets of the per-item tensors of a batch with lengths T_b."""

    def __init__(self, lengths):
        self.T = list(lengths)
        self.frame = np.concatenate([[0], np.cumsum(self.T)]).astype(np.int64)
        self.score = np.concatenate([[0], np.cumsum([H * t * t for t in self.T])]).astype(np.int64)
        self.bd = np.concatenate([[0], np.cumsum([H * t * (2 * t - 1) for t in self.T])]).astype(np.int64)
        self.pos = np.concatenate([[0], np.cumsum([2 * t - 1 for t in self.T])]).astype(np.int64)

    @property
    def frames(self):
        return int(self.frame[-1])

    def frames_of(self, flat, b, width=D):
        """Rows of item b in a [frames, width] tensor."""
        return flat.reshape(-1, width)[self.frame[b]:self.frame[b + 1]]

    def chunk(self, flat, b, per_frame, shape):
        """Item b of a tensor whose items hold per_frame*T_b elements."""
        f = flat.reshape(-1)
        return f[self.frame[b] * per_frame:self.frame[b + 1] * per_frame].reshape(shape)

    def scores(self, flat, b):
        T = self.T[b]
        return flat.reshape(-1)[self.score[b]:self.score[b + 1]].reshape(H, T, T)

    def bds(self, flat, b):
        T = self.T[b]
        return flat.reshape(-1)[self.bd[b]:self.bd[b + 1]].reshape(H, T, 2 * T - 1)

    def posrows(self, flat, b):
        return flat.reshape(-1, D)[self.pos[b]:self.pos[b + 1]]
