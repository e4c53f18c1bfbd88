"""Device buffers shared by the ranks of a process group through CUDA IPC
(include/mbs_gemm_a4w4.h: mbs_ipc_*), for copy-engine exchanges over NVLink."""

from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib

__all__ = ["PeerBuffer"]

_HANDLE_BYTES = 64


class _CudaArray:
    """__cuda_array_interface__ view of a raw device allocation (no ownership)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerBuffer:
    """`nbytes` of device memory on every rank of `group`, each rank holding the
    device pointers of all ranks' buffers (its own and its peers', mapped
    through CUDA IPC).  Collective: every rank of the group constructs it with
    the same size.  Release with close() (also collective in practice: a peer
    must not write into a buffer that was freed)."""

    def __init__(self, nbytes: int, device: torch.device, group: Optional[dist.ProcessGroup] = None):
        self.nbytes, self.device, self.group = int(nbytes), device, group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * _HANDLE_BYTES)()
        with torch.cuda.device(device):
            _lib.call("mbs_ipc_alloc", self.nbytes, ctypes.byref(ptr), handle)
        self.ptr = int(ptr.value)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.ptrs = []
        self._opened = []
        with torch.cuda.device(device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.ptrs.append(self.ptr)
                    continue
                hb = (ctypes.c_ubyte * _HANDLE_BYTES).from_buffer_copy(h)
                pp = ctypes.c_void_p()
                _lib.call("mbs_ipc_open", hb, ctypes.byref(pp))
                self.ptrs.append(int(pp.value))
                self._opened.append(int(pp.value))

    def tensor(self, shape, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """This rank's buffer as a tensor of `shape` (no copy; lives as long as the buffer)."""
        itemsize = torch.empty((), dtype=dtype).element_size()
        n = 1
        for d in shape:
            n *= int(d)
        if n * itemsize > self.nbytes:
            raise ValueError("PeerBuffer.tensor: shape larger than the buffer")
        t = torch.as_tensor(_CudaArray(self.ptr, (n * itemsize,), "|u1"), device=self.device)
        return t.view(dtype).view(*shape)

    def close(self):
        with torch.cuda.device(self.device):
            for p in self._opened:
                _lib.call("mbs_ipc_close", p)
            self._opened = []
            if self.ptr:
                _lib.call("mbs_ipc_free", self.ptr)
                self.ptr = 0
