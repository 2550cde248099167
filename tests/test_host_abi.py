"""CPU checks of the C ABI: the library loads without a GPU, exports every symbol the
header declares, and its host helpers compute exactly what the reference computes."""
import ctypes
import os
import re

import numpy as np
import pytest

from hybridagent_b200 import _lib, layout, workloads
from oracle import zero1 as Z

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "hybridagent_b200.h")


def declared_symbols() -> set[str]:
    text = open(HEADER).read()
    return set(re.findall(r"^\s*(?:int|const char\*)\s+(ha_\w+)\s*\(", text, flags=re.M))


def test_header_declares_the_bound_symbols():
    assert declared_symbols() == set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name
    assert L.ha_abi_version() == 1


@pytest.mark.parametrize("name", ["qwen3_8b", "gemma_12b", "qwen3_14b", "moe_26b_a4b", "config1_cpu"])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_greedy_owners_match_reference_rule(name, world):
    n = workloads.numels(workloads.WORKLOADS[name]())
    assert layout.greedy_owners(n, world) == Z.greedy_owners(n, world)


def test_greedy_owner_ties_and_order():
    assert layout.greedy_owners([5, 5, 5, 5], 2) == [0, 1, 0, 1]
    assert layout.greedy_owners([1, 9, 9, 3], 3) == [2, 0, 1, 2] == Z.greedy_owners([1, 9, 9, 3], 3)
    assert layout.greedy_owners([7], 4) == [0]


def test_fill_step_scalars_bitwise_like_python():
    lrs = np.array([1e-6, 3e-4, 0.1, 1e-6], np.float64)
    steps = np.array([1, 7, 101, 100000], np.int64)
    tab = np.zeros(4, dtype=_lib.TENSOR_DTYPE)
    b1, b2, wd = 0.9, 0.999, 0.01
    _lib.call("ha_fill_step_scalars", 4, _lib.np_ptr(lrs), _lib.np_ptr(steps), b1, b2, wd, _lib.np_ptr(tab))
    for k in range(4):
        lr, t = float(lrs[k]), int(steps[k])
        c1 = 1.0 - b1 ** t  # optimizer.py:182-183, Python floats
        c2 = 1.0 - b2 ** t
        assert tab[k]["decay"] == np.float32(1.0 - lr * wd)
        assert tab[k]["neg_lr"] == np.float32(-lr)
        assert tab[k]["rc1"] == np.float32(1.0 / c1)  # torch CUDA: x / c == x * float(1.0 / c)
        assert tab[k]["rc2"] == np.float32(1.0 / c2)


def test_make_scalars():
    sc = _lib.AdamwScalars()
    _lib.call("ha_make_scalars", 0.9, 0.999, 1e-8, 0.01, _lib.HA_BF16, 1, 1.0 / (3.7 + 1e-6), ctypes.byref(sc))
    assert (sc.b1, sc.a1, sc.b2, sc.a2, sc.eps) == tuple(float(np.float32(x)) for x in
                                                         (0.9, 1.0 - 0.9, 0.999, 1.0 - 0.999, 1e-8))
    assert sc.use_decay == 1 and sc.clip == 1 and sc.clip_mult == float(np.float32(1.0 / (3.7 + 1e-6)))
    _lib.call("ha_make_scalars", 0.9, 0.999, 1e-8, 0.0, _lib.HA_F32, 0, 0.0, ctypes.byref(sc))
    assert sc.use_decay == 0 and sc.clip == 0
    with pytest.raises(_lib.HAError):
        _lib.call("ha_make_scalars", 0.9, 0.999, 1e-8, 0.0, 7, 0, 0.0, ctypes.byref(sc))


def test_chunk_tables():
    numels = [0, 1, 16384, 16385, 40000]
    tab = layout.chunk_table(numels, 16384)
    assert [(int(c["tensor"]), int(c["index"])) for c in tab] == [
        (1, 0), (2, 0), (3, 0), (3, 1), (4, 0), (4, 1), (4, 2)]
    only = layout.chunk_table(numels, 16384, include=[False, False, True, False, True])
    assert [int(c["tensor"]) for c in only] == [2, 4, 4, 4]
    sizes = np.array(numels, np.int64)
    bad = tab.copy()
    bad[3]["index"] = 2  # 2*16384 >= 16385
    with pytest.raises(_lib.HAError, match="beyond numel"):
        _lib.call("ha_check_chunks", len(numels), _lib.np_ptr(sizes), _lib.np_ptr(bad), len(bad), 16384)
    bad = tab.copy()
    bad[0]["tensor"] = 9
    with pytest.raises(_lib.HAError, match="out of range"):
        _lib.call("ha_check_chunks", len(numels), _lib.np_ptr(sizes), _lib.np_ptr(bad), len(bad), 16384)


def test_kernel_entry_points_validate_arguments_without_a_gpu():
    sc = _lib.AdamwScalars()
    with pytest.raises(_lib.HAError, match="chunk_elems"):
        _lib.call("ha_adamw_step", None, None, 1, 123, _lib.HA_BF16, _lib.HA_BF16, ctypes.byref(sc), None)
    with pytest.raises(_lib.HAError, match="param dtype"):
        _lib.call("ha_adamw_step", None, None, 1, _lib.HA_ADAMW_CHUNK, _lib.HA_BF16, _lib.HA_F16, ctypes.byref(sc),
                  None)
    _lib.call("ha_adamw_step", None, None, 0, _lib.HA_ADAMW_CHUNK, _lib.HA_BF16, _lib.HA_BF16, ctypes.byref(sc), None)
    with pytest.raises(_lib.HAError, match="elem_bytes"):
        _lib.call("ha_gather", None, None, 1, 16384, 3, None)
    with pytest.raises(_lib.HAError, match="max_ctas"):
        _lib.call("ha_gather_capped", None, None, 1, 16384, 2, 0, None)
    _lib.call("ha_gather_capped", None, None, 0, 16384, 2, 8, None)  # nothing to copy: no launch
    with pytest.raises(_lib.HAError, match="elem_bytes"):
        _lib.call("ha_copy_async", None, 0, 8, None)
    bad = np.zeros(1, dtype=_lib.COPY_DTYPE)  # dst 0
    with pytest.raises(_lib.HAError, match="entry 0"):
        _lib.call("ha_copy_async", _lib.np_ptr(bad), 1, 2, None)
    same = np.zeros(1, dtype=_lib.COPY_DTYPE)
    same["src"] = same["dst"] = 4096
    same["numel"] = 10
    _lib.call("ha_copy_async", _lib.np_ptr(same), 1, 2, None)  # src == dst: skipped, no CUDA call
    with pytest.raises(_lib.HAError):
        _lib.call("ha_grad_sumsq", None, None, 5, _lib.HA_SUMSQ_CHUNK, _lib.HA_BF16, None, None, None)
    with pytest.raises(_lib.HAError, match="max_ctas"):
        _lib.call("ha_grad_sumsq_ctas", None, None, 5, _lib.HA_SUMSQ_CHUNK, _lib.HA_BF16, None, None, -1, None)
    with pytest.raises(_lib.HAError):
        _lib.call("ha_reduce_scatter", None, None, None, 1, _lib.HA_BF16, None)
