"""Device buffers shared by the ranks of one node (one process per GPU) over CUDA IPC.

`PeerBuffer(nbytes, group)` allocates `nbytes` of zero-filled device memory on every rank of the
process group and maps every other rank's buffer into this process (peer access over NVLink), so
a kernel on this rank can store straight into any rank's buffer: `ptr(r)` is rank r's buffer as
seen from here.  Handles travel through `torch.distributed.all_gather_object`, which works with
the NCCL and gloo backends.  Plain IPC mappings only: no multicast objects are created.

The buffer lives until `close()` (or garbage collection); tensors from `view()` must not
outlive it, and no rank may still store into it: close after a barrier of the group.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import check, lib

HANDLE_BYTES = 64


class _CudaArray:
    """Zero-copy handle for torch.as_tensor through __cuda_array_interface__."""

    def __init__(self, ptr, shape, dtype):
        typestr = {torch.float16: "<f2", torch.float32: "<f4", torch.uint8: "|u1", torch.int32: "<i4"}[dtype]
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerBuffer:
    def __init__(self, nbytes, group=None, device=None):
        dist = torch.distributed
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.nbytes = int(nbytes)
        self._ptrs = [None] * self.world
        self._imported = []
        with torch.cuda.device(self.device):
            own = ctypes.c_void_p()
            check(lib.qlin_peer_alloc(self.nbytes, ctypes.byref(own)), "qlin_peer_alloc")
            self._ptrs[self.rank] = own.value
            handle = ctypes.create_string_buffer(HANDLE_BYTES)
            check(lib.qlin_peer_export(own, handle), "qlin_peer_export")
            handles = [None] * self.world
            if self.world > 1:
                dist.all_gather_object(handles, bytes(handle.raw), group=group)
            for r in range(self.world):
                if r == self.rank:
                    continue
                mapped = ctypes.c_void_p()
                check(lib.qlin_peer_import(ctypes.create_string_buffer(handles[r], HANDLE_BYTES),
                                           ctypes.byref(mapped)), "qlin_peer_import")
                self._ptrs[r] = mapped.value
                self._imported.append(mapped.value)

    def ptr(self, rank, offset=0):
        """Device address of byte `offset` of rank `rank`'s buffer, valid in this process."""
        return self._ptrs[rank] + offset

    def view(self, shape, dtype, offset=0):
        """This rank's buffer (from byte `offset`) as a tensor of `shape` / `dtype`, zero-copy."""
        n = 1
        for s in shape:
            n *= s
        if offset + n * torch.empty((), dtype=dtype).element_size() > self.nbytes:
            raise ValueError("view exceeds the buffer")
        base = torch.float16 if dtype == torch.bfloat16 else dtype
        t = torch.as_tensor(_CudaArray(self._ptrs[self.rank] + offset, shape, base), device=self.device)
        return t.view(dtype)

    def close(self):
        with torch.cuda.device(self.device):
            for p in self._imported:
                lib.qlin_peer_close(ctypes.c_void_p(p))
            self._imported = []
            if self._ptrs[self.rank] is not None:
                lib.qlin_peer_free(ctypes.c_void_p(self._ptrs[self.rank]))
            self._ptrs = [None] * self.world

    def __del__(self):
        try:
            if self._ptrs and self._ptrs[self.rank] is not None:
                self.close()
        except Exception:
            pass
