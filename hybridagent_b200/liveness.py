"""Host-side liveness of the peer ranks, for the pushes that run before any collective.

Gradient landing pushes gradients into the owners' receive windows while backward is still
running, before the step's first collective (whose deadline would notice a lost rank), so a
rank that died during that backward could otherwise receive stores into a window its process no
longer holds.  Every rank therefore runs a heartbeat: a daemon thread that bumps a counter
under ``<prefix>/<rank>`` in the caller's key-value store (the process group's store) every
``interval_s`` and, in the same beat, reads every peer's counter.  Before each early push a
rank asks which peers are stale (a peer whose counter has not moved for ``deadline_s`` of this
rank's own monotonic clock); with any stale peer the push is skipped, and the exchange in
``all_reduce_grads`` sends those gradients instead, after its deadline-bound collective has
confirmed (or reported as ``CommFailure``) that every rank is there.  Counters are compared only with their own earlier values, so clocks of different hosts
never meet.  Nothing here touches a GPU.
"""
from __future__ import annotations

import threading
import time


class Heartbeat:
    """This rank's heartbeat and its view of the peers' heartbeats."""

    def __init__(self, store, rank: int, world: int, *, interval_s: float = 0.25, deadline_s: float = 3.0,
                 prefix: str = "hybridagent_b200/heartbeat"):
        if deadline_s <= interval_s:
            raise ValueError("the staleness deadline must exceed the heartbeat interval")
        self.store, self.rank, self.world = store, int(rank), int(world)
        self.interval_s, self.deadline_s = float(interval_s), float(deadline_s)
        self.keys = [f"{prefix}/{r}" for r in range(self.world)]
        self.peers = [r for r in range(self.world) if r != self.rank]
        self._lock = threading.Lock()  # one store request at a time from this process's threads
        self._beats = 0
        self._stop = threading.Event()
        now = time.monotonic()
        self._seen = {r: (None, now) for r in self.peers}  # peer -> (last counter value, when it moved)
        self.failed: str | None = None  # the store itself stopped answering (its host is gone)
        self._beat()
        self._thread = threading.Thread(target=self._run, name=f"hybridagent_b200-heartbeat-{rank}", daemon=True)
        self._thread.start()

    def _beat(self) -> None:
        """Bumps this rank's counter and reads the peers' (the thread does both every
        interval, so a peer's counter is watched continuously, not only when asked)."""
        self._beats += 1
        try:
            with self._lock:
                self.store.set(self.keys[self.rank], str(self._beats))
                # check() each key first: a get would block on a key its peer has not written yet,
                # and one late peer must not hide the counters of the others
                present = [r for r in self.peers if self.store.check([self.keys[r]])]
                values = self.store.multi_get([self.keys[r] for r in present]) if present else []
        except Exception as e:  # noqa: BLE001 -- any store failure means the peers cannot be trusted
            self.failed = f"heartbeat store: {e}"
            return
        now = time.monotonic()
        with self._lock:
            for r, value in zip(present, values):
                value = bytes(value)
                if value != self._seen[r][0]:
                    self._seen[r] = (value, now)

    def _run(self) -> None:
        while not self._stop.wait(self.interval_s):
            self._beat()

    def stale_peers(self) -> list[int]:
        """Peers whose counter has not moved for ``deadline_s`` (every peer once the store
        stopped answering)."""
        if self.failed is not None:
            return list(self.peers)
        now = time.monotonic()
        with self._lock:
            return [r for r in self.peers if now - self._seen[r][1] > self.deadline_s]

    def all_fresh(self) -> bool:
        return not self.stale_peers()

    def stop(self) -> None:
        self._stop.set()
        self._thread.join(timeout=2 * self.interval_s + 1.0)
