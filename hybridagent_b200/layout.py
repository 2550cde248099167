"""Shard layout of the ZeRO-1 step: who owns which tensor, and where it lives in HBM.

Ownership is the reference's greedy rule (hybrid_rl/optimizer.py:46-53, via the C ABI's
``ha_greedy_owners``): largest tensor first, each to the currently least-loaded rank, ties
to the lowest rank.  Every rank computes it from the tensor sizes alone, so all ranks
agree without communicating.

The reference keeps each parameter where the model allocated it and moves gradients and
parameters with one collective per bucket or tensor.  Here the tensors of each dtype
class are materialised **owner-major**: rank r's tensors sit contiguously in segment r of
one packed buffer, each starting on an ``ALIGN``-element boundary, and every segment has
the same length ``seg_len`` (the largest rank's padded load).  That turns the reference's
per-owner reduces into one equal-count reduce-scatter and its per-tensor broadcasts into
one all-gather, while each tensor's owner stays exactly the reference's.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from . import _lib

ALIGN = 64  # elements: 128-byte (bf16) / 256-byte (fp32) aligned slots


def align_up(n: int, a: int = ALIGN) -> int:
    return (n + a - 1) // a * a


def greedy_owners(numels: list[int], world: int) -> list[int]:
    """Owner rank of every tensor (optimizer.py:46-53)."""
    n = len(numels)
    sizes = np.ascontiguousarray(numels, dtype=np.int64)
    out = np.zeros(n, dtype=np.int32)
    _lib.call("ha_greedy_owners", n, _lib.np_ptr(sizes), world, _lib.np_ptr(out))
    return out.tolist()


@dataclass
class DtypeClass:
    """All tensors of one parameter dtype and their owner-major slots."""
    code: int                                   # HA_F32 / HA_BF16 / HA_F16
    indices: list[int]                          # global tensor indices, in list order
    offset: dict[int, int] = field(default_factory=dict)   # index -> element offset in its owner's segment
    seg_len: int = 0                            # elements per rank segment
    own_len: list[int] = field(default_factory=list)       # padded elements used in each rank's segment

    def owned(self, owner: list[int], rank: int) -> list[int]:
        return [i for i in self.indices if owner[i] == rank]


@dataclass
class Plan:
    world: int
    numels: list[int]
    owner: list[int]
    classes: list[DtypeClass]

    def loads(self) -> list[int]:
        out = [0] * self.world
        for i, n in enumerate(self.numels):
            out[self.owner[i]] += n
        return out


def plan(numels: list[int], dtype_codes: list[int], world: int) -> Plan:
    owner = greedy_owners(numels, world)
    classes: list[DtypeClass] = []
    for code in sorted(set(dtype_codes)):
        cls = DtypeClass(code, [i for i, c in enumerate(dtype_codes) if c == code])
        fill = [0] * world
        for i in cls.indices:
            r = owner[i]
            cls.offset[i] = fill[r]
            fill[r] += align_up(numels[i])
        cls.own_len = fill
        cls.seg_len = align_up(max(fill))
        classes.append(cls)
    return Plan(world, list(numels), owner, classes)


def chunk_table(numels: list[int], chunk_elems: int, include: list[bool] | None = None) -> np.ndarray:
    """ha_chunk list covering the given table entries (ha_plan_chunks)."""
    n = len(numels)
    sizes = np.ascontiguousarray(numels, dtype=np.int64)
    inc = None if include is None else np.ascontiguousarray(include, dtype=np.uint8)
    count = ctypes.c_int64(0)
    _lib.call("ha_plan_chunks", n, _lib.np_ptr(sizes), _lib.np_ptr(inc), chunk_elems, None, 0, ctypes.byref(count))
    out = np.zeros(count.value, dtype=_lib.CHUNK_DTYPE)
    if count.value:
        _lib.call("ha_plan_chunks", n, _lib.np_ptr(sizes), _lib.np_ptr(inc), chunk_elems, _lib.np_ptr(out),
                  count.value, ctypes.byref(count))
        _lib.call("ha_check_chunks", n, _lib.np_ptr(sizes), _lib.np_ptr(out), count.value, chunk_elems)
    return out


def push_destinations(cls: DtypeClass, owner: list[int], rank: int, elem_bytes: int,
                      grad_bases: list[int] | None, local_grad_base: int) -> list[int]:
    """Where this rank's gradient of every tensor of ``cls`` goes (bytes addresses).

    p2p (``grad_bases`` = every rank's address of its receive buffer, as mapped here): into
    the owner's buffer, region ``rank`` (rank r's contributions occupy elements
    [r*seg_len, (r+1)*seg_len)), at the tensor's offset in the owner's segment -- so the
    owner finds all ranks' copies of a tensor at the same offset of consecutive regions.
    nccl (``grad_bases`` None): into the local owner-major pack, segment ``owner``, the
    layout an equal-count reduce-scatter expects."""
    out = []
    for i in cls.indices:
        if grad_bases is None:
            out.append(local_grad_base + (owner[i] * cls.seg_len + cls.offset[i]) * elem_bytes)
        else:
            out.append(grad_bases[owner[i]] + (rank * cls.seg_len + cls.offset[i]) * elem_bytes)
    return out


def peer_deltas(param_bases: list[int], rank: int) -> list[int]:
    """Byte offsets from this rank's packed parameter buffer to each peer's (rank order,
    skipping this rank): the same element lives at the same offset on every rank."""
    return [b - param_bases[rank] for r, b in enumerate(param_bases) if r != rank]


@dataclass
class Pieces:
    """The parts of a dtype class's gradients that one exchange round moves.

    Round k covers elements [bounds[k], bounds[k+1]) of every owner's segment, at most
    S = round_elems of them (round_bounds: k*S, unless the last round is split), so a tensor
    whose slot crosses a bound is split.  Entry j: element ``src_off[j]`` of table entry
    ``tensor[j]`` (an index into ``cls.indices``), ``count[j]`` elements, owned by
    ``owner[j]``, landing at element ``dst_off[j]`` of the sender's region (S elements) of
    that round's receive window; ``round[j]`` is its round."""
    tensor: np.ndarray
    src_off: np.ndarray
    owner: np.ndarray
    dst_off: np.ndarray
    count: np.ndarray
    round: np.ndarray
    n_rounds: int
    round_elems: int
    bounds: np.ndarray

    def own_counts(self, cls: DtypeClass, rank: int) -> list[int]:
        """Elements of ``rank``'s segment each round reduces (its padded load, split)."""
        b, n = self.bounds, cls.own_len[rank]
        return [max(0, min(int(b[k + 1]), n) - int(b[k])) for k in range(self.n_rounds)]


def round_bounds(seg_len: int, S: int, tail_split: int = 0) -> np.ndarray:
    """Start of every exchange round in each owner's segment, then the end of the last one.

    Rounds of S elements; with ``tail_split`` = t > 0 the last round's part of the segment is
    cut into up to t + 1 rounds of halving length (1/2, 1/4, ... of it, multiples of ALIGN, the
    last taking the rest).  The owner's sum of the last round runs after every push, with
    nothing left to overlap it, so a short last round shortens the step by most of that sum,
    at the cost of t more rounds (a barrier and a sum launch each)."""
    assert S % ALIGN == 0 and S > 0
    n = max(1, -(-seg_len // S))
    bounds = [k * S for k in range(n)]
    last = bounds[-1]
    rest = max(seg_len - last, 0)
    for _ in range(max(tail_split, 0)):
        part = align_up(-(-rest // 2))
        if rest <= ALIGN or part >= rest:
            break
        last += part
        rest -= part
        bounds.append(last)
    bounds.append(max(n * S, last + ALIGN))
    return np.asarray(bounds, dtype=np.int64)


def round_elems_for(cls: DtypeClass, world: int, elem_bytes: int, budget_bytes: int) -> int:
    """Largest round (multiple of ALIGN elements) whose double-buffered receive window of
    ``world`` regions fits ``budget_bytes``, and no larger than one segment."""
    s = budget_bytes // (2 * world * elem_bytes)
    s = max(ALIGN, s // ALIGN * ALIGN)
    return min(s, max(cls.seg_len, ALIGN))


def exchange_pieces(cls: DtypeClass, owner: list[int], numels: list[int], round_elems: int,
                    tail_split: int = 0) -> Pieces:
    """Pieces of every tensor's slot, plus zero-fill pieces (``tensor`` -1) over the gaps
    between slots up to each owner's padded load: the two halves of the receive window are
    reused by rounds with different layouts, so every element an owner adds must be
    rewritten by every round (a gap left untouched would still hold an older round's
    values).  Rounds as ``round_bounds(cls.seg_len, round_elems, tail_split)``."""
    S = round_elems
    bounds = round_bounds(cls.seg_len, S, tail_split)
    cols = [[] for _ in range(6)]

    def emit(k, start, n, o, src0):
        r = int(np.searchsorted(bounds, start, side="right")) - 1
        lo = start
        while lo < start + n:
            hi = min(start + n, int(bounds[r + 1]))
            for col, val in zip(cols, (k, src0 + lo - start, o, lo - int(bounds[r]), hi - lo, r)):
                col.append(val)
            lo, r = hi, r + 1

    ends = {}
    for k, i in enumerate(cls.indices):
        off, n, o = cls.offset[i], numels[i], owner[i]
        if n:
            emit(k, off, n, o, 0)
        ends.setdefault(o, []).append((off, off + n))
    for o, slots in ends.items():  # the gaps of owner o's segment, up to its padded load
        pos = 0
        for lo, hi in sorted(slots) + [(cls.own_len[o], cls.own_len[o])]:
            if lo > pos:
                emit(-1, pos, lo - pos, o, 0)
            pos = max(pos, hi)
    arr = [np.asarray(c, dtype=np.int64) for c in cols]
    return Pieces(*arr, n_rounds=len(bounds) - 1, round_elems=S, bounds=bounds)


LAND_ROUNDS = 2  # exchange rounds whose window halves are free between one update and the next exchange


def landing_pieces(pc: Pieces, n_entries: int) -> list[np.ndarray]:
    """Per table entry, the indices of its pieces that may be pushed while the gradient is
    still landing during backward: the pieces of rounds 0 and 1.  Between the barrier that
    ends an update (after every owner's sums of the previous exchange) and the first barrier
    of the next exchange nobody reads either half of any receive window, so those pieces can
    be stored early; later rounds reuse a half and must wait for the exchange's barriers."""
    sel = np.nonzero((pc.round < LAND_ROUNDS) & (pc.tensor >= 0))[0]
    order = sel[np.argsort(pc.tensor[sel], kind="stable")]
    bounds = np.searchsorted(pc.tensor[order], np.arange(n_entries + 1))
    return [order[bounds[k]:bounds[k + 1]] for k in range(n_entries)]


def piece_destinations(pc: Pieces, recv_bases: list[int], rank: int, world: int, elem_bytes: int) -> np.ndarray:
    """Address of every piece in its owner's receive window: half ``round % 2``, region
    ``rank`` (windows of 2 x world regions of ``round_elems`` elements)."""
    bases = np.asarray(recv_bases, dtype=np.uint64)
    S = pc.round_elems
    return bases[pc.owner] + (((pc.round % 2) * world * S + rank * S + pc.dst_off) * elem_bytes).astype(np.uint64)


def piece_sources(pc: Pieces, entry_ptrs: np.ndarray, elem_bytes: int, dst: np.ndarray | None = None,
                  landed: np.ndarray | None = None) -> np.ndarray:
    """Source address of every piece: its gradient's address (``entry_ptrs`` per table
    entry, 0 for a tensor without one: zero-fill) plus the piece's offset; gaps zero-fill.
    The early pieces (rounds < LAND_ROUNDS) of entries marked in ``landed`` were pushed
    during backward and get src == dst, which the gather kernel skips."""
    pt = np.where(pc.tensor >= 0, np.asarray(entry_ptrs, dtype=np.uint64)[np.maximum(pc.tensor, 0)], 0)
    pt = pt.astype(np.uint64)
    src = np.where(pt != 0, pt + (pc.src_off * elem_bytes).astype(np.uint64), 0).astype(np.uint64)
    if landed is not None:
        skip = (pc.round < LAND_ROUNDS) & (pc.tensor >= 0) & np.asarray(landed, dtype=bool)[np.maximum(pc.tensor, 0)]
        src[skip] = dst[skip]
    return src


def split_smallest(entries: np.ndarray, sizes: np.ndarray, share: float) -> tuple[np.ndarray, np.ndarray]:
    """(rest, smallest): the smallest entries whose sizes add up to at most ``share`` of the
    total go to the second array; both keep the original order."""
    entries = np.asarray(entries, dtype=np.int64)
    if share <= 0 or len(entries) == 0:
        return entries, entries[:0]
    sizes = np.asarray(sizes, dtype=np.int64)
    order = np.argsort(sizes, kind="stable")
    take = order[np.cumsum(sizes[order]) <= share * int(sizes.sum())]
    mask = np.zeros(len(entries), dtype=bool)
    mask[take] = True
    return entries[~mask], entries[mask]


def balanced_groups(entries: np.ndarray, sizes: np.ndarray, n: int) -> list[np.ndarray]:
    """Splits ``entries`` into ``n`` groups of about equal total size (largest first, each to
    the currently smallest group); each group keeps its entries in their original order."""
    groups: list[list[int]] = [[] for _ in range(n)]
    load = [0] * n
    for j in np.argsort(-np.asarray(sizes, dtype=np.int64), kind="stable").tolist():
        g = load.index(min(load))
        groups[g].append(j)
        load[g] += int(sizes[j])
    return [np.asarray(entries, dtype=np.int64)[sorted(g)] for g in groups]


def peer_groups(entries: np.ndarray, entry_owner: np.ndarray, rank: int, world: int) -> list[np.ndarray]:
    """``entries`` bound for peers grouped by destination: group j holds those owned by rank
    (rank + 1 + j) % world, in their original order (world - 1 groups).  One copy-engine
    stream per group keeps every peer's ingress fed from every rank at once."""
    owners = np.asarray(entry_owner)[entries] if len(entries) else np.zeros(0, dtype=np.int64)
    return [np.asarray(entries, dtype=np.int64)[owners == (rank + 1 + j) % world] for j in range(world - 1)]


def round_push_split(pc: Pieces, k: int, rank: int, push_streams: int,
                     kernel_share: float, world: int = 0) -> tuple[np.ndarray, list[np.ndarray]]:
    """Round k's pieces split between the push kernel and the copy engines.  With
    ``push_streams`` 0 the kernel pushes every piece; otherwise it takes this rank's own
    pieces and the smallest peer-bound ones (``kernel_share`` of their bytes), and the rest
    go to the copy engines: ``push_streams`` > 0 groups of about equal bytes, or (-1) one
    group per destination peer (``peer_groups``, needs ``world``)."""
    entries = np.nonzero(pc.round == k)[0]
    if push_streams == 0:
        return entries, []
    remote = entries[pc.owner[entries] != rank]
    remote, by_kernel = split_smallest(remote, pc.count[remote], kernel_share)
    kernel = np.sort(np.concatenate([entries[pc.owner[entries] == rank], by_kernel]))
    if push_streams < 0:
        return kernel, peer_groups(np.sort(remote), pc.owner, rank, world)
    return kernel, balanced_groups(remote, pc.count[remote], push_streams)


def gather_parts(chunks: np.ndarray, offsets: list[int], numels: list[int], chunk_elems: int,
                 part_elems: int) -> list[tuple[int, int, int, int]]:
    """The owned segment's update cut into parts for the copy-engine parameter all-gather.

    ``chunks`` is the update's ha_chunk list over the owned tensors (entry k: slot offset
    ``offsets[k]`` in the owner's segment, ``numels[k]`` elements).  Returns (first chunk,
    chunk count, first element, end element) per part, each part about ``part_elems``
    elements of the segment: updating part j and copying its elements [first, end) to the
    peers can start as soon as part j's chunks are done, while part j + 1 updates.  Parts
    cover the segment from its first slot to the end of its last, gaps included (the gaps
    hold nothing anyone reads), and never split a chunk."""
    n = len(chunks)
    if n == 0:
        return []
    t = chunks["tensor"].astype(np.int64)
    j = chunks["index"].astype(np.int64)
    off = np.asarray(offsets, dtype=np.int64)[t]
    num = np.asarray(numels, dtype=np.int64)[t]
    start = off + j * chunk_elems
    end = off + np.minimum((j + 1) * chunk_elems, num)
    if np.any(start[1:] < end[:-1]):
        raise ValueError("gather_parts: chunks are not in segment order")
    parts, c0 = [], 0
    while c0 < n:
        # the last chunk whose end stays within part_elems of this part's start (at least one)
        c1 = int(np.searchsorted(end, start[c0] + max(part_elems, 1), side="right"))
        c1 = max(c1, c0 + 1)
        parts.append((c0, c1 - c0, int(start[c0]), int(end[c1 - 1])))
        c0 = c1
    return parts


def landing_batch(src: np.ndarray, dst: np.ndarray, count: np.ndarray, chunk_elems: int) -> tuple[np.ndarray, np.ndarray]:
    """ha_copy entries (piece j: ``count[j]`` elements from address ``src[j]`` to ``dst[j]``)
    and the ha_chunk list that covers them, for one early push of landed gradients."""
    n = len(src)
    copies = np.zeros(n, dtype=_lib.COPY_DTYPE)
    copies["src"] = src
    copies["dst"] = dst
    copies["numel"] = count
    per = (np.asarray(count, dtype=np.int64) + chunk_elems - 1) // chunk_elems
    total = int(per.sum())
    chunks = np.zeros(total, dtype=_lib.CHUNK_DTYPE)
    if total:
        chunks["tensor"] = np.repeat(np.arange(n, dtype=np.uint32), per)
        chunks["index"] = np.arange(total, dtype=np.int64) - np.repeat(np.cumsum(per) - per, per)
        _lib.call("ha_check_chunks", n, _lib.np_ptr(np.ascontiguousarray(count, dtype=np.int64)), _lib.np_ptr(chunks),
                  total, chunk_elems)
    return copies, chunks


def interleaved_chunks(entries: np.ndarray, entry_owner: np.ndarray, entry_numel: np.ndarray, rank: int, world: int,
                       chunk_elems: int) -> np.ndarray:
    """ha_chunk list over the given table entries (one exchange round's pieces), one chunk
    per owner in turn, starting at owner rank+1 and ending with this rank's own.

    Chunks run roughly in list order, so a piece-ordered list would keep every in-flight CTA
    on one destination at a time: local copies and NVLink stores would not overlap, and since
    every rank walks the pieces in the same order, all ranks would store into the same owner
    at once and share its ingress.  Taking one chunk per owner in turn, rotated by rank, makes
    every owner receive from every peer at any moment, with the local copies alongside."""
    per_owner: list[list[tuple[int, int]]] = [[] for _ in range(world)]
    for e in entries.tolist():
        n_chunks = (int(entry_numel[e]) + chunk_elems - 1) // chunk_elems
        per_owner[int(entry_owner[e])].extend((e, c) for c in range(n_chunks))
    order = [(rank + d) % world for d in range(1, world + 1)]
    out = []
    pos = [0] * world
    remaining = sum(len(x) for x in per_owner)
    while remaining:
        for o in order:
            if pos[o] < len(per_owner[o]):
                out.append(per_owner[o][pos[o]])
                pos[o] += 1
                remaining -= 1
    tab = np.zeros(len(out), dtype=_lib.CHUNK_DTYPE)
    if out:
        tab["tensor"] = [k for k, _ in out]
        tab["index"] = [c for _, c in out]
    return tab
