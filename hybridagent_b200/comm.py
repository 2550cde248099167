"""NCCL communicator of the ZeRO-1 step, owned by the C library (``ha_comm_*``).

The 128-byte NCCL unique id is created on rank 0 and handed to the other ranks over the
caller's existing ``torch.distributed`` process group (the group the reference's
``hybrid_rl/dist.py:init`` sets up), after which all optimizer traffic -- the used-mask MAX,
the gradient reduce-scatter, the norm SUM and the parameter all-gather -- goes through
this communicator on the caller's current CUDA stream.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib


class NcclComm:
    def __init__(self, rank: int, world: int, group=None):
        if not dist.is_initialized():
            raise RuntimeError("world_size > 1 needs an initialized torch.distributed process group "
                               "to exchange the NCCL id (hybrid_rl.dist.init does this)")
        self.rank, self.world = rank, world
        uid = (ctypes.c_uint8 * 128)()
        if rank == 0:
            _lib.call("ha_comm_unique_id", ctypes.cast(uid, ctypes.c_void_p))
        box = [bytes(uid)]
        dist.broadcast_object_list(box, src=0, group=group)
        uid = (ctypes.c_uint8 * 128).from_buffer_copy(box[0])
        handle = ctypes.c_void_p()
        _lib.call("ha_comm_init", ctypes.cast(uid, ctypes.c_void_p), world, rank, ctypes.byref(handle))
        self._handle = handle

    @property
    def handle(self) -> ctypes.c_void_p:
        if self._handle is None:
            raise RuntimeError("communicator already closed")
        return self._handle

    @staticmethod
    def _stream() -> int:
        return torch.cuda.current_stream().cuda_stream

    def reduce_scatter(self, send: int, recv: int, count: int, dtype: int) -> None:
        _lib.call("ha_reduce_scatter", self.handle, send, recv, count, dtype, self._stream())

    def all_gather(self, send: int, recv: int, count: int, dtype: int) -> None:
        _lib.call("ha_all_gather", self.handle, send, recv, count, dtype, self._stream())

    def all_reduce_sum(self, buf: torch.Tensor, dtype: int) -> None:
        _lib.call("ha_all_reduce_sum", self.handle, buf.data_ptr(), buf.numel(), dtype, self._stream())

    def all_reduce_max(self, buf: torch.Tensor, dtype: int) -> None:
        _lib.call("ha_all_reduce_max", self.handle, buf.data_ptr(), buf.numel(), dtype, self._stream())

    def close(self) -> None:
        if self._handle is not None:
            h, self._handle = self._handle, None
            _lib.call("ha_comm_destroy", h)
