"""IPC-shared device buffers and their peer mappings (world size > 1 on one NVLink domain).

Each rank allocates its packed parameter buffer and its gradient receive buffer with the C
library's ``ha_malloc`` (plain cudaMalloc, so CUDA IPC can share them), exposes them to
torch as zero-copy tensors, hands the 64-byte IPC handles to every rank over the caller's
process group, and maps every peer's buffers with ``ha_ipc_open``.  The mapped peer
addresses go only to this library's own kernels (plain loads / stores) and to the copy
engines through ``cudaMemcpyAsync`` / ``cudaMemsetAsync`` in ``ha_copy_async`` (the gradient
push, the parameter all-gather and the early pushes of gradient landing); no other library's
kernel (torch, NCCL, cuBLAS) is ever given a peer address.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib

_TYPESTR = {torch.float32: "<f4", torch.bfloat16: "<i2", torch.float16: "<i2", torch.float64: "<f8",
            torch.int32: "<i4", torch.uint8: "|u1"}
_VIEW_AS = {torch.float32: None, torch.bfloat16: torch.int16, torch.float16: torch.int16, torch.float64: None,
            torch.int32: None, torch.uint8: None}


class DeviceBuffer:
    """``numel`` elements of ``dtype`` in IPC-shareable device memory, zero-filled, with a
    torch tensor view (``.tensor``) that keeps this object alive."""

    def __init__(self, numel: int, dtype: torch.dtype, device: torch.device):
        self.numel, self.dtype, self.device = int(numel), dtype, device
        self.nbytes = max(self.numel, 1) * torch.empty((), dtype=dtype).element_size()
        ptr = ctypes.c_void_p()
        with torch.cuda.device(device):
            _lib.call("ha_malloc", self.nbytes, ctypes.byref(ptr))
            self.ptr = int(ptr.value)
            _lib.call("ha_memset", self.ptr, 0, self.nbytes, torch.cuda.current_stream().cuda_stream)
            torch.cuda.current_stream().synchronize()
            self.__cuda_array_interface__ = {"shape": (max(self.numel, 1),), "typestr": _TYPESTR[dtype],
                                             "data": (self.ptr, False), "version": 3, "strides": None,
                                             "stream": None}
            t = torch.as_tensor(self, device=device)
        if _VIEW_AS[dtype] is not None:
            t = t.view(dtype)
        assert t.data_ptr() == self.ptr, "torch copied the IPC buffer instead of viewing it"
        self.tensor = t[:self.numel]

    def ipc_handle(self) -> bytes:
        buf = (ctypes.c_uint8 * 64)()
        _lib.call("ha_ipc_get_handle", self.ptr, ctypes.cast(buf, ctypes.c_void_p))
        return bytes(buf)

    def __del__(self):
        ptr = getattr(self, "ptr", None)
        if ptr:
            try:
                _lib.call("ha_free", ptr)
            except Exception:
                pass
            self.ptr = None


class PeerMap:
    """Every rank's address of a set of equally laid-out buffers.

    ``bases[name][r]`` is the address, valid on this rank, of rank r's buffer ``name``
    (this rank's own pointer for r == rank).  Opening fails cleanly (``ok`` False) when a
    peer's memory cannot be mapped; the caller decides collectively what to do."""

    def __init__(self, buffers: dict[str, DeviceBuffer], rank: int, world: int, group=None):
        self.rank, self.world = rank, world
        self.bases: dict[str, list[int]] = {}
        self._opened: list[int] = []
        names = sorted(buffers)
        mine = [buffers[n].ipc_handle() for n in names]
        everyone: list = [None] * world
        dist.all_gather_object(everyone, mine, group=group)
        self.ok = True
        self.error = ""
        for n in names:
            self.bases[n] = [0] * world
            self.bases[n][rank] = buffers[n].ptr
        for r in range(world):
            if r == rank:
                continue
            for k, n in enumerate(names):
                out = ctypes.c_void_p()
                h = (ctypes.c_uint8 * 64).from_buffer_copy(everyone[r][k])
                try:
                    _lib.call("ha_ipc_open", ctypes.cast(h, ctypes.c_void_p), ctypes.byref(out))
                except _lib.HAError as e:
                    self.ok = False
                    self.error = str(e)
                    return
                self.bases[n][r] = int(out.value)
                self._opened.append(int(out.value))

    def close(self) -> None:
        for p in self._opened:
            try:
                _lib.call("ha_ipc_close", p)
            except _lib.HAError:
                pass
        self._opened = []
