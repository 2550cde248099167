"""Owner-major shard layout: slots are aligned, disjoint, inside their owner's segment,
and cost little padding on the benchmark parameter sets."""
import pytest

from hybridagent_b200 import layout, workloads
from hybridagent_b200._lib import HA_BF16, HA_F32


@pytest.mark.parametrize("name", ["qwen3_8b", "gemma_12b", "qwen3_14b", "moe_26b_a4b"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_layout_properties(name, world):
    n = workloads.numels(workloads.WORKLOADS[name]())
    p = layout.plan(n, [HA_BF16] * len(n), world)
    (cls,) = p.classes
    assert cls.seg_len % layout.ALIGN == 0
    for r in range(world):
        slots = sorted((cls.offset[i], n[i]) for i in cls.indices if p.owner[i] == r)
        end = 0
        for off, size in slots:
            assert off % layout.ALIGN == 0 and off >= end
            end = off + size
        assert end <= cls.seg_len
    padding = (world * cls.seg_len - sum(n)) / sum(n)
    assert padding < 0.003, padding  # equal segments + 64-element slot alignment


def test_mixed_dtype_classes():
    n = [1000, 10, 5000, 64, 3]
    codes = [HA_BF16, HA_F32, HA_BF16, HA_F32, HA_BF16]
    p = layout.plan(n, codes, 2)
    assert [c.code for c in p.classes] == [HA_F32, HA_BF16]
    f32, bf16 = p.classes
    assert f32.indices == [1, 3] and bf16.indices == [0, 2, 4]
    assert p.owner == layout.greedy_owners(n, 2)
    for c in p.classes:
        for r in range(2):
            assert c.own_len[r] <= c.seg_len


@pytest.mark.parametrize("world", [2, 4, 8])
def test_push_chunk_order_covers_every_chunk_once_and_interleaves_owners(world):
    n = workloads.numels(workloads.qwen3_8b())
    p = layout.plan(n, [HA_BF16] * len(n), world)
    (cls,) = p.classes
    for rank in range(world):
        order = layout.push_chunk_order(cls, p.owner, rank, world, n, 16384)
        natural = layout.chunk_table([n[i] for i in cls.indices], 16384)
        assert sorted(map(tuple, order.tolist())) == sorted(map(tuple, natural.tolist()))
        owners = [p.owner[cls.indices[int(t)]] for t in order["tensor"][:4 * world]]
        # the first rounds visit every owner, starting after this rank and ending with it
        assert owners[:world] == [(rank + d) % world for d in range(1, world + 1)]
        assert len(set(owners)) == world


def test_push_destinations_land_in_the_senders_region():
    n = [1000, 64, 5000, 3, 70000]
    p = layout.plan(n, [HA_BF16] * len(n), 3)
    (cls,) = p.classes
    bases = [1 << 40, 2 << 40, 3 << 40]
    for rank in range(3):
        dst = layout.push_destinations(cls, p.owner, rank, 2, bases, 0)
        for k, i in enumerate(cls.indices):
            o = p.owner[i]
            elem = (dst[k] - bases[o]) // 2
            assert elem == rank * cls.seg_len + cls.offset[i]
            assert elem + n[i] <= (rank + 1) * cls.seg_len
    assert layout.peer_deltas([100, 300, 700], 1) == [-200, 400]


@pytest.mark.parametrize("world,S", [(2, 64 * 1000), (3, 64 * 7), (8, 64 * 50_000), (2, 64)])
def test_exchange_pieces_partition_every_slot_and_gap(world, S):
    import numpy as np
    n = [1000, 64, 5000, 3, 70000, 1, 12345, 640000]
    p = layout.plan(n, [HA_BF16] * len(n), world)
    (cls,) = p.classes
    pc = layout.exchange_pieces(cls, p.owner, n, S)
    assert pc.n_rounds == -(-cls.seg_len // S)
    covered = {i: np.zeros(n[i], np.int32) for i in cls.indices}
    # what each owner's region receives in each round, from every piece (tensors and gaps)
    written = {(o, r): np.zeros(S, np.int32) for o in range(world) for r in range(pc.n_rounds)}
    for t, so, o, do, c, r in zip(pc.tensor, pc.src_off, pc.owner, pc.dst_off, pc.count, pc.round):
        assert 0 < c and 0 <= do and do + c <= S
        written[(o, r)][do:do + c] += 1
        if t < 0:
            continue  # a zero-filled gap
        i = cls.indices[t]
        assert o == p.owner[i]
        assert cls.offset[i] + so == r * S + do  # same segment coordinate
        covered[i][so:so + c] += 1
    assert all((v == 1).all() for v in covered.values())
    for o in range(world):
        counts = pc.own_counts(cls, o)
        assert sum(counts) == cls.own_len[o] and all(0 <= x <= S for x in counts)
        for r in range(pc.n_rounds):
            w = written[(o, r)]
            assert (w[:counts[r]] == 1).all() and (w[counts[r]:] == 0).all()  # every summed element, once


def test_round_elems_for_budget():
    n = workloads.numels(workloads.qwen3_8b())
    p = layout.plan(n, [HA_BF16] * len(n), 8)
    (cls,) = p.classes
    S = layout.round_elems_for(cls, 8, 2, 2 << 30)
    assert S % layout.ALIGN == 0 and 2 * 8 * S * 2 <= 2 << 30
    assert layout.round_elems_for(cls, 8, 2, 1 << 60) == cls.seg_len
