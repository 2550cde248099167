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
