"""Owner-major shard layout: slots are aligned, disjoint, inside their owner's segment,
and cost little padding on the benchmark parameter sets."""
import numpy as np
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
def test_interleaved_chunks_cover_every_chunk_once_and_interleave_owners(world):
    """Each exchange round's chunk list (the product's order) covers every chunk of every
    piece of the round once and visits the owners in turn, starting after this rank."""
    import numpy as np
    n = workloads.numels(workloads.qwen3_8b())
    p = layout.plan(n, [HA_BF16] * len(n), world)
    (cls,) = p.classes
    S = layout.round_elems_for(cls, world, 2, 4 << 30)
    pc = layout.exchange_pieces(cls, p.owner, n, S)
    for rank in range(world):
        for k in range(pc.n_rounds):
            entries = np.nonzero(pc.round == k)[0]
            order = layout.interleaved_chunks(entries, pc.owner, pc.count, rank, world, 16384)
            want = sorted((int(e), c) for e in entries for c in range(-(-int(pc.count[e]) // 16384)))
            assert sorted(map(tuple, order.tolist())) == want
            owners = [int(pc.owner[int(t)]) for t in order["tensor"][:world]]
            # the first pass visits every owner, starting after this rank and ending with it
            assert owners == [(rank + d) % world for d in range(1, world + 1)]


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


@pytest.mark.parametrize("world,S,tail", [(2, 64 * 1000, 0), (3, 64 * 7, 0), (8, 64 * 50_000, 0), (2, 64, 0),
                                          (2, 64 * 1000, 3), (3, 64 * 7, 2), (8, 64 * 50_000, 4), (2, 64, 3)])
def test_exchange_pieces_partition_every_slot_and_gap(world, S, tail):
    import numpy as np
    n = [1000, 64, 5000, 3, 70000, 1, 12345, 640000]
    p = layout.plan(n, [HA_BF16] * len(n), world)
    (cls,) = p.classes
    pc = layout.exchange_pieces(cls, p.owner, n, S, tail)
    if tail == 0:
        assert pc.n_rounds == -(-cls.seg_len // S)
    else:
        assert -(-cls.seg_len // S) <= pc.n_rounds <= -(-cls.seg_len // S) + tail
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
        assert cls.offset[i] + so == pc.bounds[r] + do  # same segment coordinate
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


def _emulate_gather(memory, copies, chunks, chunk_elems, esz):
    """ha_gather on simulated memory (``memory``: base >> 40 -> numpy array; addresses are
    base << 40 plus a byte offset): per chunk, src == dst skips, src == 0 zero-fills."""
    import numpy as np
    for t, j in zip(chunks["tensor"], chunks["index"]):
        c = copies[int(t)]
        src, dst, n = int(c["src"]), int(c["dst"]), int(c["numel"])
        lo, hi = int(j) * chunk_elems, min(n, (int(j) + 1) * chunk_elems)
        assert 0 <= lo < hi
        if src == dst:
            continue
        d = memory[dst >> 40]
        do = (dst & ((1 << 40) - 1)) // esz
        if src == 0:
            d[do + lo:do + hi] = 0
        else:
            s = memory[src >> 40]
            so = (src & ((1 << 40) - 1)) // esz
            d[do + lo:do + hi] = s[so + lo:so + hi]
    return np


@pytest.mark.parametrize("world,S,tail", [(2, 64 * 20, 0), (3, 64 * 7, 0), (2, 64 * 100_000, 0), (2, 64 * 20, 3),
                                          (2, 64 * 100_000, 3)])
def test_landing_then_residual_equals_plain_exchange(world, S, tail):
    """Early pushes of landed gradients (rounds 0 and 1, in two buckets, then one tensor
    landing again with new values, as a later backward of the same step would) followed by
    the exchange's own pushes with the landed pieces skipped leave every round's window
    half exactly as a plain exchange of the final gradients does."""
    import numpy as np
    from hybridagent_b200._lib import CHUNK_DTYPE, COPY_DTYPE
    n = [1000, 64, 5000, 3, 7000, 1, 1234, 6400, 640]
    p = layout.plan(n, [HA_BF16] * len(n), world)
    (cls,) = p.classes
    pc = layout.exchange_pieces(cls, p.owner, n, S, tail)
    rank, esz, CH = world - 1, 2, 256
    rng = np.random.default_rng(world * S)
    present = [k != 2 for k in range(len(cls.indices))]  # entry 2 has no gradient here: zero-filled
    entry_ptrs = np.array([(10 + k) << 40 if present[k] else 0 for k in range(len(cls.indices))], np.uint64)
    recv = [(100 + o) << 40 for o in range(world)]
    dst = layout.piece_destinations(pc, recv, rank, world, esz)

    def memory(grads):
        mem = {100 + o: np.full(2 * world * S, 0xDEAD, np.uint16) for o in range(world)}
        mem.update({10 + k: g.copy() for k, g in grads.items()})
        return mem

    def push_round(mem, k, src):
        entries = np.nonzero(pc.round == k)[0]
        copies = np.zeros(len(dst), COPY_DTYPE)
        copies["src"], copies["dst"], copies["numel"] = src, dst, pc.count
        per = (pc.count[entries] + CH - 1) // CH
        chunks = np.zeros(int(per.sum()), CHUNK_DTYPE)
        chunks["tensor"] = np.repeat(entries, per)
        chunks["index"] = np.concatenate([np.arange(x) for x in per]) if len(per) else []
        _emulate_gather(mem, copies, chunks, CH, esz)

    grads = {k: rng.integers(1, 1 << 15, n[i]).astype(np.uint16)
             for k, i in enumerate(cls.indices) if present[k]}
    mem = memory(grads)
    lp = layout.landing_pieces(pc, len(cls.indices))
    assert sorted(np.concatenate(lp).tolist()) == np.nonzero((pc.round < 2) & (pc.tensor >= 0))[0].tolist()
    landed_entries = [k for k in grads if len(lp[k])]
    buckets = [landed_entries[::2], landed_entries[1::2], landed_entries[:1]]
    for b, bucket in enumerate(buckets):
        if b == 2:  # a later backward changes the first gradient in place: the second push must win
            mem[10 + bucket[0]] ^= np.uint16(0x5555)
        idx = np.concatenate([lp[k] for k in bucket])
        base = np.concatenate([np.full(len(lp[k]), entry_ptrs[k], np.uint64) for k in bucket])
        copies, chunks = layout.landing_batch(base + (pc.src_off[idx] * esz).astype(np.uint64), dst[idx],
                                              pc.count[idx], CH)
        _emulate_gather(mem, copies, chunks, CH, esz)
    landed = np.zeros(len(cls.indices), bool)
    landed[landed_entries] = True
    src = layout.piece_sources(pc, entry_ptrs, esz, dst, landed)
    early = (pc.round < 2) & (pc.tensor >= 0) & landed[np.maximum(pc.tensor, 0)]
    assert early.any() and (src[early] == dst[early]).all() and (src[~early] != dst[~early]).all()
    # the reference: a plain exchange of the gradients as they are now
    ref = memory({k: mem[10 + k] for k in grads})
    src_plain = layout.piece_sources(pc, entry_ptrs, esz)
    for k in range(pc.n_rounds):
        push_round(mem, k, src)
        push_round(ref, k, src_plain)
        h = (k % 2) * world * S + rank * S
        for o in range(world):
            cnt = pc.own_counts(cls, o)[k]
            assert np.array_equal(mem[100 + o][h:h + cnt], ref[100 + o][h:h + cnt]), (k, o)


def test_balanced_groups():
    import numpy as np
    entries = np.array([10, 11, 12, 13, 14, 15])
    sizes = np.array([5, 100, 7, 60, 40, 1])
    groups = layout.balanced_groups(entries, sizes, 2)
    assert sorted(np.concatenate(groups).tolist()) == entries.tolist()
    loads = [int(sizes[np.searchsorted(entries, g)].sum()) for g in groups]
    assert max(loads) - min(loads) <= max(sizes)
    assert all((np.diff(g) > 0).all() for g in groups)  # original order kept
    assert [len(g) for g in layout.balanced_groups(entries[:0], sizes[:0], 3)] == [0, 0, 0]


@pytest.mark.parametrize("S", [64, 64 * 4, 64 * 1000])
def test_empty_owner_segments(S):
    """More ranks than tensors: the ranks that own nothing have an empty padded load, receive
    no pieces, reduce nothing in any round and land nothing early."""
    import numpy as np
    n = [1000, 64, 5]
    p = layout.plan(n, [HA_BF16] * len(n), 5)
    (cls,) = p.classes
    assert sorted(p.owner) == [0, 1, 2]
    assert [cls.own_len[r] for r in (3, 4)] == [0, 0]
    pc = layout.exchange_pieces(cls, p.owner, n, S)
    assert not np.isin(pc.owner, [3, 4]).any()
    for r in (3, 4):
        assert pc.own_counts(cls, r) == [0] * pc.n_rounds
        assert cls.owned(p.owner, r) == []
    lp = layout.landing_pieces(pc, len(cls.indices))
    assert sum(len(x) for x in lp) == int(((pc.round < 2) & (pc.tensor >= 0)).sum())
    dst = layout.piece_destinations(pc, [(10 + r) << 40 for r in range(5)], 4, 5, 2)
    assert ((dst >> np.uint64(40)) - np.uint64(10) < np.uint64(3)).all()  # only owners 0-2 receive


def test_split_smallest():
    import numpy as np
    e = np.array([5, 6, 7, 8, 9])
    sz = np.array([50, 10, 30, 5, 100])
    rest, small = layout.split_smallest(e, sz, 0.2)  # 20% of 195 = 39: sizes 5, 10 (15), +30 > 39
    assert small.tolist() == [6, 8] and rest.tolist() == [5, 7, 9]
    rest, small = layout.split_smallest(e, sz, 0.0)
    assert small.tolist() == [] and rest.tolist() == e.tolist()
    rest, small = layout.split_smallest(e, sz, 1.0)
    assert small.tolist() == e.tolist() and rest.tolist() == []


@pytest.mark.parametrize("world,streams,share", [(2, 0, 0.1), (2, 2, 0.0), (2, 2, 0.1), (3, 4, 0.3), (8, 2, 0.1)])
def test_round_push_split_partitions_every_round(world, streams, share):
    """Kernel list and copy-engine groups partition each round's pieces; the copy engines get
    only peer-bound pieces, the kernel every piece of this rank's own and at most the share of
    the peer-bound bytes (smallest first)."""
    import numpy as np
    n = workloads.numels(workloads.qwen3_8b())[:60]
    p = layout.plan(n, [HA_BF16] * len(n), world)
    (cls,) = p.classes
    pc = layout.exchange_pieces(cls, p.owner, n, 64 * 100_000)
    for rank in range(world):
        for k in range(pc.n_rounds):
            kernel, groups = layout.round_push_split(pc, k, rank, streams, share)
            ce = np.concatenate(groups) if groups else np.zeros(0, np.int64)
            everything = np.nonzero(pc.round == k)[0]
            assert sorted(kernel.tolist() + ce.tolist()) == everything.tolist()
            assert (np.diff(kernel) > 0).all()
            if streams == 0:
                assert groups == [] and kernel.tolist() == everything.tolist()
                continue
            assert len(groups) == streams and (pc.owner[ce] != rank).all()
            own = everything[pc.owner[everything] == rank]
            assert np.isin(own, kernel).all()
            by_kernel = kernel[pc.owner[kernel] != rank]
            remote_bytes = int(pc.count[everything[pc.owner[everything] != rank]].sum())
            assert int(pc.count[by_kernel].sum()) <= share * remote_bytes
            if len(by_kernel) and len(ce):
                assert pc.count[by_kernel].max() <= pc.count[ce].min()  # the smallest ones



@pytest.mark.parametrize("part", [1, 16384, 50000, 10 ** 9])
def test_gather_parts_cover_the_owned_segment_in_order(part):
    """Copy-engine all-gather parts: consecutive chunk ranges, element ranges that start where
    the previous part ended (or at a later slot) and contain every element of their chunks."""
    numels = [100000, 7, 40000, 16384, 1, 65536 * 3 + 5]
    offsets = []
    o = 0
    for n in numels:
        offsets.append(o)
        o += layout.align_up(n)
    ch = layout.chunk_table(numels, 16384)
    parts = layout.gather_parts(ch, offsets, numels, 16384, part)
    assert parts[0][0] == 0 and sum(p[1] for p in parts) == len(ch)
    covered = np.zeros(o, dtype=bool)
    for (c0, nc, e0, e1), nxt in zip(parts, parts[1:] + [None]):
        assert e0 < e1
        if nxt is not None:
            assert nxt[0] == c0 + nc and nxt[2] >= e1
        assert nc == 1 or e1 - e0 <= max(part, 1)
        for q in range(c0, c0 + nc):
            k, j = int(ch[q]["tensor"]), int(ch[q]["index"])
            a = offsets[k] + j * 16384
            b = offsets[k] + min((j + 1) * 16384, numels[k])
            assert e0 <= a and b <= e1
            covered[a:b] = True
    for k, n in enumerate(numels):
        assert covered[offsets[k]:offsets[k] + n].all()


def test_peer_groups_one_destination_per_stream():
    owners = np.array([0, 1, 2, 3, 1, 2, 0, 3])
    groups = layout.peer_groups(np.array([1, 2, 3, 4, 5, 7]), owners, rank=0, world=4)
    assert [g.tolist() for g in groups] == [[1, 4], [2, 5], [3, 7]]
    groups = layout.peer_groups(np.array([0, 2, 6]), owners, rank=2, world=4)
    assert [g.tolist() for g in groups] == [[], [0, 6], []]


@pytest.mark.parametrize("seg_len,S,tail", [(0, 64, 3), (64, 64, 3), (6400, 640, 0), (6400, 640, 3), (6401, 640, 3),
                                            (640 * 7 + 64, 640, 5), (1 << 30, 64 << 20, 3), (100_000, 1 << 20, 4)])
def test_round_bounds(seg_len, S, tail):
    b = layout.round_bounds(seg_len, S, tail)
    n = max(1, -(-seg_len // S))
    lens = np.diff(b)
    assert b[0] == 0 and b[-1] >= seg_len and (lens > 0).all() and (lens <= S).all()
    assert (b % layout.ALIGN == 0).all()
    assert list(b[:n]) == [k * S for k in range(n)]  # full rounds unchanged
    assert len(b) - 1 <= n + tail
    if tail == 0:
        assert list(b) == [k * S for k in range(n + 1)]
    tail_lens = [min(int(hi), seg_len) - int(lo) for lo, hi in zip(b[n - 1:-1], b[n:]) if lo < seg_len]
    if len(tail_lens) > 1:  # each split part at most half of what was left before it
        assert all(a >= c for a, c in zip(tail_lens, tail_lens[1:-1]))
        assert tail_lens[-1] <= -(-(seg_len - (n - 1) * S) // 2)
