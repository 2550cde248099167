"""Host-side deadline logic of the communicator (no GPU, no NCCL): the wait used for every
host read of a collective's result gives up after the deadline and runs the abort, and
never gives up early."""
import time

from hybridagent_b200.comm import poll


def test_poll_returns_when_done():
    calls = []
    t0 = time.monotonic()
    state = {"n": 0}

    def done():
        state["n"] += 1
        return state["n"] > 50

    assert poll(done, 5.0, lambda: calls.append("abort"))
    assert calls == [] and time.monotonic() - t0 < 1.0


def test_poll_times_out_and_aborts_once():
    calls = []
    t0 = time.monotonic()
    assert not poll(lambda: False, 0.3, lambda: calls.append("abort"))
    elapsed = time.monotonic() - t0
    assert calls == ["abort"]
    assert 0.3 <= elapsed < 1.5


def test_poll_does_not_busy_spin_after_the_spin_window():
    t0 = time.monotonic()
    late = {"q": 0}

    def done():
        if time.monotonic() - t0 > 0.01:  # well past the 1 ms spin window
            late["q"] += 1
        return False

    poll(done, 0.2, lambda: None, spin_s=0.001, nap_s=0.01)
    assert late["q"] < 40  # ~19 naps of 10 ms, not a busy loop
