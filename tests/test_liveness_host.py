"""Peer heartbeats that gate gradient landing's early pushes (host only, no GPU): a peer whose
heartbeat stops is reported stale after the deadline, a live one never is, and a stale peer
makes the early push drop its gradients back to the exchange."""
import os
import socket
import time
from types import SimpleNamespace

import torch.distributed as dist
import torch.multiprocessing as mp

from hybridagent_b200.liveness import Heartbeat


def test_stopped_heartbeat_goes_stale_in_one_store():
    store = dist.HashStore()
    a = Heartbeat(store, 0, 2, interval_s=0.05, deadline_s=1.0)
    b = Heartbeat(store, 1, 2, interval_s=0.05, deadline_s=1.0)
    try:
        time.sleep(0.2)
        assert a.stale_peers() == [] and b.stale_peers() == []
        for _ in range(6):  # stays fresh while it beats
            time.sleep(0.15)
            assert a.all_fresh()
        b.stop()  # rank 1 stalls: its counter stops moving
        time.sleep(1.6)
        assert a.stale_peers() == [1]
    finally:
        a.stop()
        b.stop()


def test_missing_peer_is_stale_after_the_deadline():
    store = dist.HashStore()
    a = Heartbeat(store, 0, 3, interval_s=0.05, deadline_s=1.0)
    c = Heartbeat(store, 2, 3, interval_s=0.05, deadline_s=1.0)  # rank 1 never starts
    try:
        assert a.stale_peers() == []  # within the deadline of construction
        time.sleep(1.6)
        assert a.stale_peers() == [1]  # the late peer hides nothing: rank 2 is seen beating
        assert c.stale_peers() == [1]
    finally:
        a.stop()
        c.stop()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, port: int, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, 2, interval_s=0.05, deadline_s=1.0)
    try:
        dist.barrier()
        time.sleep(0.3)
        fresh = hb.all_fresh()
        dist.barrier()
        if rank == 1:
            hb.stop()  # host-side stall: rank 1 stops beating (nothing of its in flight)
            time.sleep(2.5)
            stale = hb.stale_peers()
        else:
            time.sleep(2.0)
            stale = hb.stale_peers()
        q.put((rank, fresh, stale))
        dist.barrier()
    finally:
        hb.stop()
        dist.destroy_process_group()


def test_gloo_ranks_see_a_stalled_peer():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r: (fresh, stale) for r, fresh, stale in (q.get(timeout=60) for _ in procs)}
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    assert res[0][0] and res[1][0]  # both fresh while both beat
    assert res[0][1] == [1]  # rank 0 sees the stalled rank 1


def test_stale_peer_drops_the_early_push():
    from hybridagent_b200.optimizer import ZeroOneAdamW
    g = object()
    stub = SimpleNamespace(_land_pending=[(0, 1, g, None)], _land_pending_bytes=64, land_skipped=0,
                           _liveness=SimpleNamespace(all_fresh=lambda: False),
                           _classes=[SimpleNamespace(layout=SimpleNamespace(indices=[5, 7]))],
                           _landed={7: (g, 0), 5: (g, 0)})
    ZeroOneAdamW._land_flush(stub)
    assert stub._landed == {5: (g, 0)}  # tensor 7 goes back to the exchange
    assert stub.land_skipped == 1 and stub._land_pending == [] and stub._land_pending_bytes == 0
