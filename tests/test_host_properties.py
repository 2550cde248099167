"""Property tests (hypothesis) of the C host helpers against the reference's own Python
arithmetic: the per-tensor step scalars (hybrid_rl/optimizer.py:180-185, Python floats, then
fp32 as torch receives them), the clip multiplier and the chunk planner.  CPU only."""
import ctypes
import math

import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

from hybridagent_b200 import _lib, layout

lr_st = st.floats(min_value=1e-9, max_value=1.0)
step_st = st.integers(min_value=1, max_value=10**7)


@settings(max_examples=300, deadline=None)
@given(st.lists(st.tuples(lr_st, step_st), min_size=1, max_size=20), st.floats(min_value=0.0, max_value=0.99),
       st.floats(min_value=0.5, max_value=0.99999), st.floats(min_value=0.0, max_value=0.5))
def test_step_scalars_equal_pythons(entries, beta1, beta2, wd):
    lrs = np.array([e[0] for e in entries], np.float64)
    steps = np.array([e[1] for e in entries], np.int64)
    tab = np.zeros(len(entries), dtype=_lib.TENSOR_DTYPE)
    _lib.call("ha_fill_step_scalars", len(entries), _lib.np_ptr(lrs), _lib.np_ptr(steps), beta1, beta2, wd,
              _lib.np_ptr(tab))
    for k, (lr, t) in enumerate(entries):
        c1 = 1.0 - beta1 ** t
        c2 = 1.0 - beta2 ** t
        assert tab[k]["decay"] == np.float32(1.0 - lr * wd)
        assert tab[k]["neg_lr"] == np.float32(-lr)
        assert tab[k]["rc1"] == np.float32(1.0 / c1)
        assert tab[k]["rc2"] == np.float32(1.0 / c2)


@settings(max_examples=300, deadline=None)
@given(st.floats(min_value=0.0, max_value=1e6, allow_nan=False), st.floats(min_value=1e-3, max_value=100.0))
def test_clip_multiplier_is_the_python_scale_as_fp32(norm, max_norm):
    if not norm > max_norm:
        return
    scale = float(max_norm) / (norm + 1e-6)  # optimizer.py:156
    sc = _lib.AdamwScalars()
    _lib.call("ha_make_scalars", 0.9, 0.999, 1e-8, 0.0, _lib.HA_BF16, 1, scale, ctypes.byref(sc))
    assert sc.clip == 1 and sc.clip_mult == float(np.float32(scale))


@settings(max_examples=200, deadline=None)
@given(st.lists(st.integers(min_value=0, max_value=200_000), max_size=30),
       st.sampled_from([8, 64, 16384, 32768]))
def test_chunk_table_lists_every_chunk_once_in_order(numels, chunk):
    tab = layout.chunk_table(numels, chunk)
    want = [(k, j) for k, n in enumerate(numels) for j in range(math.ceil(n / chunk))]
    assert list(zip(tab["tensor"].tolist(), tab["index"].tolist())) == want
