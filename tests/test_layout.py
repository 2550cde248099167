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
