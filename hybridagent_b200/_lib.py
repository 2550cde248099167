"""ctypes binding of ``libhybridagent_b200.so`` (declared in ``include/hybridagent_b200.h``).

The library is the product: nothing here falls back to another implementation.  If the
shared object is missing or fails to load, :func:`lib` raises with the reason.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libhybridagent_b200.so")

HA_OK, HA_ERR_INVALID, HA_ERR_CUDA, HA_ERR_NCCL, HA_ERR_UNSUPPORTED = 0, 1, 2, 3, 4
HA_F32, HA_BF16, HA_F16, HA_F64, HA_I32, HA_U8 = 0, 1, 2, 3, 4, 5
HA_ADAMW_CHUNK = 16384
HA_SUMSQ_CHUNK = 32768
HA_NOALLOC_SUMSQ_MAX_CHUNKS = 262144
HA_SUM_REGIONS_CHUNK = 16384
HA_MAX_PEERS = 15

# numpy mirrors of the C structs (layouts asserted against the header's sizes)
TENSOR_DTYPE = np.dtype([("grad", "<u8"), ("master", "<u8"), ("exp_avg", "<u8"), ("exp_avg_sq", "<u8"),
                         ("param", "<u8"), ("numel", "<i8"), ("decay", "<f4"), ("neg_lr", "<f4"),
                         ("rc1", "<f4"), ("rc2", "<f4")])
CHUNK_DTYPE = np.dtype([("tensor", "<u4"), ("index", "<u4")])
COPY_DTYPE = np.dtype([("src", "<u8"), ("dst", "<u8"), ("numel", "<i8"), ("reserved", "<i8")])
assert TENSOR_DTYPE.itemsize == 64 and CHUNK_DTYPE.itemsize == 8 and COPY_DTYPE.itemsize == 32


class AdamwScalars(ctypes.Structure):
    _fields_ = [("b1", ctypes.c_float), ("a1", ctypes.c_float), ("b2", ctypes.c_float), ("a2", ctypes.c_float),
                ("eps", ctypes.c_float), ("use_decay", ctypes.c_int32), ("clip", ctypes.c_int32),
                ("clip_mult", ctypes.c_float)]


class Peers(ctypes.Structure):
    _fields_ = [("n", ctypes.c_int32), ("reserved", ctypes.c_int32), ("delta", ctypes.c_int64 * 15)]


class HAError(RuntimeError):
    """A non-zero status from the C ABI, with the library's message."""

    def __init__(self, code: int, where: str, message: str):
        super().__init__(f"{where} failed ({code}): {message}")
        self.code = code


# every exported symbol of include/hybridagent_b200.h with its ctypes signature
_vp, _i64, _i32, _dbl, _f32, _sz = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_double,
                                    ctypes.c_float, ctypes.c_size_t)
SIGNATURES: dict[str, tuple[list, object]] = {
    "ha_last_error": ([], ctypes.c_char_p),
    "ha_abi_version": ([], ctypes.c_int),
    "ha_greedy_owners": ([_i64, _vp, _i32, _vp], ctypes.c_int),
    "ha_plan_chunks": ([_i64, _vp, _vp, _i64, _vp, _i64, ctypes.POINTER(ctypes.c_int64)], ctypes.c_int),
    "ha_check_chunks": ([_i64, _vp, _vp, _i64, _i64], ctypes.c_int),
    "ha_fill_step_scalars": ([_i64, _vp, _vp, _dbl, _dbl, _dbl, _vp], ctypes.c_int),
    "ha_make_scalars": ([_dbl, _dbl, _dbl, _dbl, ctypes.c_int, ctypes.c_int, _dbl, ctypes.POINTER(AdamwScalars)],
                        ctypes.c_int),
    "ha_adamw_step": ([_vp, _vp, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.POINTER(AdamwScalars), _vp],
                      ctypes.c_int),
    "ha_grad_sumsq": ([_vp, _vp, _i64, _i64, ctypes.c_int, _vp, _vp, _vp], ctypes.c_int),
    "ha_grad_sumsq_ctas": ([_vp, _vp, _i64, _i64, ctypes.c_int, _vp, _vp, ctypes.c_int, _vp], ctypes.c_int),
    "ha_grad_sumsq_noalloc": ([_vp, _vp, _i64, _i64, ctypes.c_int, _vp, _vp], ctypes.c_int),
    "ha_scale_grads": ([_vp, _vp, _i64, _i64, ctypes.c_int, _f32, _vp], ctypes.c_int),
    "ha_gather": ([_vp, _vp, _i64, _i64, ctypes.c_int, _vp], ctypes.c_int),
    "ha_gather_capped": ([_vp, _vp, _i64, _i64, ctypes.c_int, ctypes.c_int32, _vp], ctypes.c_int),
    "ha_copy_async": ([_vp, _i64, ctypes.c_int, _vp], ctypes.c_int),
    "ha_malloc": ([_sz, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "ha_free": ([_vp], ctypes.c_int),
    "ha_memset": ([_vp, ctypes.c_int, _sz, _vp], ctypes.c_int),
    "ha_ipc_get_handle": ([_vp, _vp], ctypes.c_int),
    "ha_ipc_open": ([_vp, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "ha_ipc_close": ([_vp], ctypes.c_int),
    "ha_sum_regions": ([_vp, _i32, _i64, _i64, _vp, ctypes.c_int, _vp, _vp, _vp], ctypes.c_int),
    "ha_adamw_step_peers": ([_vp, _vp, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.POINTER(AdamwScalars),
                             ctypes.POINTER(Peers), _vp], ctypes.c_int),
    "ha_adamw_step_delta": ([_vp, _vp, _i64, _i64, ctypes.c_int, ctypes.POINTER(AdamwScalars), _vp, _vp, _vp],
                            ctypes.c_int),
    "ha_comm_unique_id": ([_vp], ctypes.c_int),
    "ha_comm_init": ([_vp, _i32, _i32, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "ha_comm_destroy": ([_vp], ctypes.c_int),
    "ha_comm_abort": ([_vp], ctypes.c_int),
    "ha_reduce_scatter": ([_vp, _vp, _vp, _sz, ctypes.c_int, _vp], ctypes.c_int),
    "ha_all_gather": ([_vp, _vp, _vp, _sz, ctypes.c_int, _vp], ctypes.c_int),
    "ha_all_reduce_sum": ([_vp, _vp, _sz, ctypes.c_int, _vp], ctypes.c_int),
    "ha_all_reduce_max": ([_vp, _vp, _sz, ctypes.c_int, _vp], ctypes.c_int),
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it was not built (``python -m hybridagent_b200.build``)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m hybridagent_b200.build` "
                               "(hybridagent_b200 has no CPU or eager fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(code: int, where: str) -> None:
    if code != HA_OK:
        raise HAError(code, where, lib().ha_last_error().decode(errors="replace"))


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def np_ptr(a: np.ndarray | None) -> int | None:
    if a is None:
        return None
    assert a.flags.c_contiguous
    return a.ctypes.data
