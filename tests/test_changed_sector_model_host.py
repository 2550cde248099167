"""The changed-sector parameter writes as a model on the CPU (no GPU): W replicas of one packed
bf16 parameter buffer, an owner updating its masters, and the kernel's store rule (a 32-byte
sector -- 16 bf16 values, four 4-element groups -- is stored into every replica when any of its
values' rounding changed).  Starting from replicas that all hold RNE(master), every replica ends
bit-identical to a full write after every step; a replica written behind the optimizer's back
stays wrong under that rule alone, and one full write -- what the optimizer does for a step after
its version counters saw such a write on any rank -- repairs it everywhere."""
import numpy as np

from oracle import zero1 as Z

SECTOR = 16  # bf16 values per 32-byte sector


def _store_changed_sectors(old_master, new_master, replicas):
    old, new = Z.to_bf16(old_master), Z.to_bf16(new_master)
    n = len(new) // SECTOR * SECTOR
    changed = (old[:n] != new[:n]).reshape(-1, SECTOR).any(axis=1)
    mask = np.zeros(len(new), dtype=bool)
    mask[:n] = np.repeat(changed, SECTOR)
    mask[n:] = old[n:] != new[n:]  # the ragged tail goes element by element
    for r in replicas:
        r[mask] = new[mask]
    return int(mask.sum())


def _step(master, rng, lr):
    # an AdamW-sized move: about lr per element, a handful of bf16 roundings change per step
    return (master * np.float32(1 - lr * 0.01) - np.float32(lr) * rng.standard_normal(len(master)).astype(np.float32)
            ).astype(np.float32)


def test_replicas_stay_bit_identical_to_a_full_write():
    rng = np.random.default_rng(0)
    master = (rng.standard_normal(100_003) * 0.02).astype(np.float32)
    replicas = [Z.to_bf16(master) for _ in range(4)]
    stored = 0
    for _ in range(20):
        new = _step(master, rng, 1e-6)
        stored += _store_changed_sectors(master, new, replicas)
        master = new
        for r in replicas:
            assert np.array_equal(r, Z.to_bf16(master))
    assert 0 < stored < 20 * len(master)  # some sectors stored, never all of them


def test_a_replica_written_behind_the_optimizer_needs_a_full_write():
    rng = np.random.default_rng(1)
    master = (rng.standard_normal(4096) * 0.02).astype(np.float32)
    replicas = [Z.to_bf16(master) for _ in range(2)]
    replicas[1][:SECTOR] = 0  # rank 1 overwrites its copy of a few values (no version bump seen)
    new = master.copy()
    new[SECTOR:] = _step(master[SECTOR:], rng, 1e-3)  # the damaged sector's values do not move
    _store_changed_sectors(master, new, replicas)
    assert not np.array_equal(replicas[1], Z.to_bf16(new))  # the changed-sector rule leaves it wrong
    for r in replicas:  # the full write of a step marked dirty on any rank
        r[:] = Z.to_bf16(new)
    assert all(np.array_equal(r, Z.to_bf16(new)) for r in replicas)
