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
