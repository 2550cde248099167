"""NCCL communicator of the ZeRO-1 step, owned by the C library (``ha_comm_*``).

The 128-byte NCCL unique id is created on rank 0 and handed to the other ranks over the
caller's existing ``torch.distributed`` process group (the group the reference's
``hybrid_rl/dist.py:init`` sets up), after which all optimizer traffic -- the used-mask MAX,
the norm SUM, the barriers of the p2p path and, in nccl mode, the gradient reduce-scatter
and parameter all-gather -- goes through this communicator on the caller's current CUDA
stream.

Failure detection: every collective records a CUDA event after it is enqueued.  A
collective still pending ``timeout_s`` seconds after its enqueue means a rank stopped
participating; the communicator is then aborted (``ha_comm_abort``), which ends the blocked
collective, and the optimizer raises ``CommFailure`` instead of continuing (the reference
gets the same fail-closed behaviour from its process group's timeout, hybrid_rl/dist.py:29).
Two places enforce the deadline:

* ``read()`` -- every host read of a collective's result (the used mask, the norm): an
  asynchronous copy into pinned memory and an event the calling thread polls with the
  deadline.  No blocking CUDA call is made while a peer may be missing (a blocking copy
  to pageable memory can hold up other threads' CUDA calls until it returns);
* a watchdog thread that polls the outstanding events, for waits outside this library
  (the caller's next synchronisation after ``step``).

Enqueues and the abort take one lock, so the communicator is never used after it has been
aborted.
"""
from __future__ import annotations

import collections
import ctypes
import os
import threading
import time

import torch
import torch.distributed as dist

from . import _lib

DEFAULT_TIMEOUT_S = float(os.environ.get("HYBRIDAGENT_B200_COMM_TIMEOUT_S", "1800"))


class CommFailure(RuntimeError):
    """A collective of the optimizer's communicator did not complete in time (a rank
    stopped participating); the communicator has been aborted."""


def poll(done, deadline_s: float, on_timeout, spin_s: float = 0.005, nap_s: float = 0.00005) -> bool:
    """Waits until ``done()`` is true; returns False (after calling ``on_timeout()``) if it is
    still false after ``deadline_s`` seconds.  Spins for ``spin_s``, then naps ``nap_s``
    between checks (the GPU idles from the moment the awaited work ends until this returns and
    the caller launches the next, so the nap is short); never blocks inside a CUDA call."""
    t0 = time.monotonic()
    while not done():
        dt = time.monotonic() - t0
        if dt > deadline_s:
            on_timeout()
            return False
        if dt > spin_s:
            time.sleep(nap_s)
    return True


class NcclComm:
    def __init__(self, rank: int, world: int, group=None, timeout_s: float | None = None):
        if not dist.is_initialized():
            raise RuntimeError("world_size > 1 needs an initialized torch.distributed process group "
                               "to exchange the NCCL id (hybrid_rl.dist.init does this)")
        self.rank, self.world = rank, world
        self.timeout_s = DEFAULT_TIMEOUT_S if timeout_s is None else float(timeout_s)
        uid = (ctypes.c_uint8 * 128)()
        if rank == 0:
            _lib.call("ha_comm_unique_id", ctypes.cast(uid, ctypes.c_void_p))
        box = [bytes(uid)]
        dist.broadcast_object_list(box, src=0, group=group)
        uid = (ctypes.c_uint8 * 128).from_buffer_copy(box[0])
        handle = ctypes.c_void_p()
        _lib.call("ha_comm_init", ctypes.cast(uid, ctypes.c_void_p), world, rank, ctypes.byref(handle))
        self._handle = handle
        self._device = torch.cuda.current_device()
        self._lock = threading.Lock()
        self._pending: collections.deque = collections.deque()
        self.failure: str | None = None
        self._stop = threading.Event()
        self._watchdog = threading.Thread(target=self._watch, name="hybridagent_b200-comm-watchdog", daemon=True)
        self._watchdog.start()

    # ------------------------------------------------------------ failure handling
    def _abort_locked(self, what: str) -> None:
        """Aborts the communicator (caller holds the lock)."""
        if self.failure is not None:
            return
        self.failure = (f"{what} on rank {self.rank} did not complete within {self.timeout_s:g} s "
                        "(a rank stopped participating); the communicator was aborted")
        self._pending.clear()
        if self._handle is not None:
            try:
                _lib.call("ha_comm_abort", self._handle)
            except _lib.HAError:
                pass

    def _watch(self) -> None:
        torch.cuda.set_device(self._device)
        while not self._stop.wait(0.05):
            with self._lock:
                while self._pending and self._pending[0][0].query():
                    self._pending.popleft()
                if not self._pending or self.failure is not None:
                    continue
                what, t0 = self._pending[0][1], self._pending[0][2]
                if time.monotonic() - t0 > self.timeout_s:
                    self._abort_locked(what)

    def read(self, dev: torch.Tensor, host: torch.Tensor, what: str) -> torch.Tensor:
        """Copies ``dev`` (the result of an enqueued collective) into the pinned ``host``
        buffer and waits for it with the communicator's deadline; raises CommFailure after
        aborting the communicator if a rank never joins."""
        self.check()
        host.copy_(dev, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()

        def timeout():
            with self._lock:
                self._abort_locked(what)

        if not poll(ev.query, self.timeout_s, timeout):
            ev.synchronize()  # the aborted collective has ended: the copy behind it completes
        self.check()
        return host

    def check(self) -> None:
        """Raises CommFailure if the watchdog aborted the communicator."""
        if self.failure is not None:
            raise CommFailure(self.failure)

    def _enqueue(self, what: str, name: str, *args) -> None:
        with self._lock:
            self.check()
            if self._handle is None:
                raise RuntimeError("communicator already closed")
            _lib.call(name, self._handle, *args)
            ev = torch.cuda.Event()
            ev.record()
            self._pending.append((ev, what, time.monotonic()))

    # ------------------------------------------------------------ collectives
    @staticmethod
    def _stream() -> int:
        return torch.cuda.current_stream().cuda_stream

    def reduce_scatter(self, send: int, recv: int, count: int, dtype: int) -> None:
        self._enqueue("reduce-scatter", "ha_reduce_scatter", send, recv, count, dtype, self._stream())

    def all_gather(self, send: int, recv: int, count: int, dtype: int) -> None:
        self._enqueue("all-gather", "ha_all_gather", send, recv, count, dtype, self._stream())

    def all_reduce_sum(self, buf: torch.Tensor, dtype: int) -> None:
        self._enqueue("all-reduce(sum)", "ha_all_reduce_sum", buf.data_ptr(), buf.numel(), dtype, self._stream())

    def all_reduce_max(self, buf: torch.Tensor, dtype: int) -> None:
        self._enqueue("all-reduce(max)", "ha_all_reduce_max", buf.data_ptr(), buf.numel(), dtype, self._stream())

    def close(self) -> None:
        self._stop.set()
        self._watchdog.join(timeout=5)
        with self._lock:
            if self._handle is not None:
                h, self._handle = self._handle, None
                _lib.call("ha_comm_destroy", h)
