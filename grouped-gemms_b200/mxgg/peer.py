"""Device buffers shared by the ranks of one node through CUDA IPC.

``PeerBuffer(nbytes)`` is collective: every rank allocates ``nbytes`` with
``cudaMalloc`` (through ``mxgg_ipc_alloc``), the 64-byte IPC handles are
all-gathered over the process group, and every rank maps every peer's buffer
(``mxgg_ipc_open``).  ``ptrs[r]`` is then rank r's buffer as an address this
process can load from and store to over NVLink.  No NVLink multicast object
is involved: peers are reached with plain loads, stores and copies.
"""

import ctypes
from typing import List

import torch

from . import _lib


class _CudaArray:
    """Minimal ``__cuda_array_interface__`` holder so torch can view raw memory."""

    def __init__(self, ptr: int, nbytes: int, owner):
        self._owner = owner     # keeps the PeerBuffer alive while a view exists
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerBuffer:
    def __init__(self, nbytes: int, group=None):
        import torch.distributed as dist
        if nbytes <= 0:
            raise ValueError("PeerBuffer needs a positive size")
        self.nbytes = int(nbytes)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        lib = _lib.load()
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        _lib.check(lib.mxgg_ipc_alloc(self.nbytes, ctypes.byref(ptr), handle), "mxgg_ipc_alloc")
        self._own = ptr.value
        handles: List[bytes] = [b""] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self.ptrs: List[int] = []
        self._opened: List[int] = []
        for r in range(self.world):
            if r == self.rank:
                self.ptrs.append(self._own)
                continue
            p = ctypes.c_void_p()
            _lib.check(lib.mxgg_ipc_open(handles[r], ctypes.byref(p)), "mxgg_ipc_open")
            self.ptrs.append(p.value)
            self._opened.append(p.value)
        self._closed = False

    def view(self, shape, dtype: torch.dtype, offset: int = 0) -> torch.Tensor:
        """This rank's buffer as a tensor (no copy); valid while the buffer lives."""
        n = 1
        for d in shape:
            n *= int(d)
        nbytes = n * torch.empty((), dtype=dtype).element_size()
        if offset < 0 or offset + nbytes > self.nbytes:
            raise ValueError(f"view of {nbytes} bytes at {offset} exceeds the {self.nbytes}-byte buffer")
        if nbytes == 0:
            return torch.empty(shape, dtype=dtype, device=torch.device("cuda", torch.cuda.current_device()))
        raw = torch.as_tensor(_CudaArray(self._own + offset, nbytes, self), device="cuda")
        return raw.view(dtype).reshape(shape)

    def close(self) -> None:
        """Collective: unmap the peers' buffers, wait for every rank, free this one."""
        import torch.distributed as dist
        if self._closed:
            return
        torch.cuda.synchronize()
        lib = _lib.load()
        for p in self._opened:
            _lib.check(lib.mxgg_ipc_close(ctypes.c_void_p(p)), "mxgg_ipc_close")
        dist.barrier(group=self.group)
        _lib.check(lib.mxgg_ipc_free(ctypes.c_void_p(self._own)), "mxgg_ipc_free")
        self._closed = True
