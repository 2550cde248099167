"""Property tests (hypothesis) of the shard layout and the exchange plan over random tensor
lists, world sizes and round sizes: the host logic that decides every address the kernels
write.  CPU only."""
import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

from hybridagent_b200 import layout
from hybridagent_b200._lib import HA_BF16
from oracle import zero1 as Z

sizes_st = st.lists(st.integers(min_value=1, max_value=5000), min_size=1, max_size=40)
world_st = st.integers(min_value=1, max_value=9)
rounds_st = st.integers(min_value=1, max_value=80)  # round size in units of ALIGN elements


@settings(max_examples=150, deadline=None)
@given(sizes_st, world_st)
def test_plan_slots_are_aligned_disjoint_and_owned_by_the_greedy_rule(numels, world):
    p = layout.plan(numels, [HA_BF16] * len(numels), world)
    assert p.owner == Z.greedy_owners(numels, world)
    (cls,) = p.classes
    for r in range(world):
        mine = sorted((cls.offset[i], numels[i]) for i in cls.indices if p.owner[i] == r)
        end = 0
        for off, n in mine:
            assert off % layout.ALIGN == 0 and off >= end
            end = off + n
        assert cls.own_len[r] == layout.align_up(end) if mine else cls.own_len[r] == 0
        assert cls.own_len[r] <= cls.seg_len


@settings(max_examples=150, deadline=None)
@given(sizes_st, st.integers(min_value=2, max_value=9), rounds_st, st.integers(min_value=0, max_value=5))
def test_exchange_pieces_write_every_summed_element_once_per_round(numels, world, units, tail):
    p = layout.plan(numels, [HA_BF16] * len(numels), world)
    (cls,) = p.classes
    S = units * layout.ALIGN
    pc = layout.exchange_pieces(cls, p.owner, numels, S, tail)
    written = {}
    covered = {i: np.zeros(numels[i], np.int8) for i in cls.indices}
    for t, so, o, do, c, r in zip(pc.tensor, pc.src_off, pc.owner, pc.dst_off, pc.count, pc.round):
        assert c > 0 and 0 <= do and do + c <= S and 0 <= r < pc.n_rounds
        w = written.setdefault((int(o), int(r)), np.zeros(S, np.int8))
        w[do:do + c] += 1
        if t >= 0:
            i = cls.indices[t]
            assert p.owner[i] == o and cls.offset[i] + so == pc.bounds[r] + do
            covered[i][so:so + c] += 1
    assert all((v == 1).all() for v in covered.values())
    for o in range(world):
        counts = pc.own_counts(cls, o)
        assert sum(counts) == cls.own_len[o]
        for r in range(pc.n_rounds):
            w = written.get((o, r), np.zeros(S, np.int8))
            assert (w[:counts[r]] == 1).all() and (w[counts[r]:] == 0).all()


@settings(max_examples=100, deadline=None)
@given(sizes_st, st.integers(min_value=2, max_value=9), rounds_st, st.integers(min_value=-1, max_value=4),
       st.floats(min_value=0.0, max_value=1.0), st.integers(min_value=0, max_value=3))
def test_round_push_split_and_landing_pieces_partition(numels, world, units, streams, share, tail):
    p = layout.plan(numels, [HA_BF16] * len(numels), world)
    (cls,) = p.classes
    pc = layout.exchange_pieces(cls, p.owner, numels, units * layout.ALIGN, tail)
    for rank in range(world):
        for k in range(pc.n_rounds):
            kernel, groups = layout.round_push_split(pc, k, rank, streams, share, world)
            ce = np.concatenate(groups) if groups else np.zeros(0, np.int64)
            assert sorted(kernel.tolist() + ce.tolist()) == np.nonzero(pc.round == k)[0].tolist()
            assert (pc.owner[ce] != rank).all()
            if streams < 0:  # one group per destination, in rotation from rank + 1
                assert len(groups) == world - 1
                for j, g in enumerate(groups):
                    assert (pc.owner[g] == (rank + 1 + j) % world).all()
    lp = layout.landing_pieces(pc, len(cls.indices))
    flat = np.concatenate(lp) if lp else np.zeros(0, np.int64)
    assert sorted(flat.tolist()) == np.nonzero((pc.round < layout.LAND_ROUNDS) & (pc.tensor >= 0))[0].tolist()
    for k, idx in enumerate(lp):
        assert (pc.tensor[idx] == k).all()


@settings(max_examples=100, deadline=None)
@given(st.lists(st.integers(min_value=1, max_value=10**6), max_size=60), st.integers(min_value=1, max_value=8))
def test_balanced_groups_are_a_partition_within_one_item(sizes, n):
    entries = np.arange(100, 100 + len(sizes))
    groups = layout.balanced_groups(entries, np.asarray(sizes, np.int64), n)
    assert len(groups) == n
    assert sorted(np.concatenate(groups).tolist()) == entries.tolist()
    if sizes:
        loads = [sum(sizes[int(e) - 100] for e in g) for g in groups]
        assert max(loads) - min(loads) <= max(sizes)


@settings(max_examples=150, deadline=None)
@given(sizes_st, world_st, st.integers(min_value=1, max_value=200_000))
def test_gather_parts_cover_each_owned_segment(numels, world, part):
    """The copy-engine all-gather's parts: consecutive chunk ranges in segment order, each
    part's element range holding all of its chunks and the parts' ranges never overlapping."""
    p = layout.plan(numels, [HA_BF16] * len(numels), world)
    (cls,) = p.classes
    for r in range(world):
        owned = cls.owned(p.owner, r)
        if not owned:
            continue
        own_numels = [numels[i] for i in owned]
        chunks = layout.chunk_table(own_numels, 16384)
        parts = layout.gather_parts(chunks, [cls.offset[i] for i in owned], own_numels, 16384, part)
        assert parts[0][0] == 0 and sum(q[1] for q in parts) == len(chunks)
        for (c0, nc, e0, e1), nxt in zip(parts, parts[1:] + [None]):
            assert 0 < nc and e0 < e1 <= cls.own_len[r]
            if nxt is not None:
                assert nxt[0] == c0 + nc and nxt[2] >= e1
