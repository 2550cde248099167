"""TEST INFRASTRUCTURE ONLY -- the checker for the CUDA product, never the product.

CPU restatement of HybridAgent's ZeRO-1 AdamW step (``hybrid_rl/optimizer.py``) over
numpy host arrays.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg
of ``bench.py`` import this module.

Per-element arithmetic lives in ``zero1_oracle.c`` (built by ``oracle/Makefile`` into
``oracle/_build``); this file restates the per-tensor and per-rank logic around it:

* greedy largest-first ownership, ties to the lowest rank (optimizer.py:46-53);
* the used mask and the SUM of every rank's gradient onto its owner (optimizer.py:101-142);
* the global gradient norm over owned gradients and the in-place clip (optimizer.py:146-160);
* per-tensor bias-corrected AdamW with decoupled weight decay and the low-precision
  parameter copy (optimizer.py:163-191).

Gradients and parameters are numpy arrays: float32 for fp32, uint16 bit patterns for
bf16 / fp16 (the dtype travels beside the array as ``F32`` / ``BF16`` / ``F16``).

Parity pins: ``tests/golden/*.npz`` were written by the unmodified reference optimizer
(``tests/golden/make_golden.py``); ``tests/test_oracle_golden.py`` checks this oracle in its
torch-CPU rounding form against them.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

F32, BF16, F16 = 0, 1, 2

# rounding-form bits, mirrored from zero1_oracle.c
ADD_FMA, ADDCMUL_INNER, ADDCMUL_LEFT, DIV_RECIP, ADDCDIV_FMA, SCALAR_IN_DTYPE, NAN_CUDA = 1, 2, 4, 8, 16, 32, 64
FORM_TORCH_CPU = ADD_FMA | ADDCMUL_LEFT
FORM_TORCH_CUDA = ADD_FMA | ADDCMUL_INNER | DIV_RECIP | ADDCDIV_FMA | NAN_CUDA

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libzero1_oracle.so")
_lib = None


def build() -> str:
    """Compile zero1_oracle.c with the committed Makefile; returns the library path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
                os.path.join(_HERE, "zero1_oracle.c")):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        vp, i64, dbl, u32, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_double, ctypes.c_uint, ctypes.c_int
        L.ora_adamw_tensor_clipped.argtypes = [u32, i32, i32, i64, vp, vp, vp, vp, vp, dbl, dbl, dbl, dbl, dbl,
                                               i64, i32, dbl]
        L.ora_adamw_tensor_clipped.restype = None
        L.ora_clip_inplace.argtypes = [i32, u32, i64, vp, dbl]
        L.ora_clip_multiplier.argtypes = [i32, u32, dbl]
        L.ora_clip_multiplier.restype = ctypes.c_float
        L.ora_sumsq.argtypes = [i32, i64, vp]
        L.ora_sumsq.restype = dbl
        L.ora_f32_to_bf16.argtypes = [u32, i64, vp, vp]
        L.ora_f32_to_f16.argtypes = [u32, i64, vp, vp]
        L.ora_bf16_rank_sum.argtypes = [i64, i32, vp, vp]
        L.ora_form_torch_cpu.restype = i32
        L.ora_form_torch_cuda.restype = i32
        assert L.ora_form_torch_cpu() == FORM_TORCH_CPU and L.ora_form_torch_cuda() == FORM_TORCH_CUDA
        _lib = L
    return _lib


def _ptr(a: np.ndarray | None) -> int | None:
    if a is None:
        return None
    assert a.flags.c_contiguous
    return a.ctypes.data


def _check(a: np.ndarray, dtype: int) -> None:
    want = np.float32 if dtype == F32 else np.uint16
    if a.dtype != want or not a.flags.c_contiguous:
        raise TypeError(f"expected contiguous {want} array, got {a.dtype}")


# ---------------------------------------------------------------- elementwise pieces

def to_bf16(x: np.ndarray, form: int = FORM_TORCH_CUDA) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().ora_f32_to_bf16(form, x.size, _ptr(x), _ptr(out))
    return out


def to_f16(x: np.ndarray, form: int = FORM_TORCH_CUDA) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().ora_f32_to_f16(form, x.size, _ptr(x), _ptr(out))
    return out


def widen(a: np.ndarray, dtype: int) -> np.ndarray:
    """Low-precision bit patterns (or fp32) -> fp32 values."""
    if dtype == F32:
        return a.astype(np.float32, copy=False)
    if dtype == BF16:
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.view(np.float16).astype(np.float32)


def narrow(x: np.ndarray, dtype: int, form: int = FORM_TORCH_CUDA) -> np.ndarray:
    if dtype == F32:
        return np.ascontiguousarray(x, dtype=np.float32)
    return to_bf16(x, form) if dtype == BF16 else to_f16(x, form)


def sumsq(grad: np.ndarray, dtype: int) -> float:
    """Sum of float(g)**2 over one tensor, accumulated in double (optimizer.py:151)."""
    _check(grad, dtype)
    return float(lib().ora_sumsq(dtype, grad.size, _ptr(grad)))


def clip_multiplier(dtype: int, form: int, scale: float) -> float:
    return float(lib().ora_clip_multiplier(dtype, form, scale))


def clip_inplace(grad: np.ndarray, dtype: int, form: int, scale: float) -> None:
    """grad.mul_(scale) in the gradient's dtype (optimizer.py:159)."""
    _check(grad, dtype)
    lib().ora_clip_inplace(dtype, form, grad.size, _ptr(grad), scale)


def adamw_tensor(form: int, grad: np.ndarray, grad_dtype: int, master: np.ndarray, exp_avg: np.ndarray,
                 exp_avg_sq: np.ndarray, param: np.ndarray | None, param_dtype: int, *, lr: float, beta1: float,
                 beta2: float, eps: float, weight_decay: float, step: int, clip_scale: float | None = None) -> None:
    """One owned tensor's update in place (optimizer.py:176-191).  ``param`` None means the
    fp32 master is the parameter (optimizer.py:71-73).  ``clip_scale`` folds the in-place
    clip of optimizer.py:159 into the gradient read."""
    _check(grad, grad_dtype)
    for a in (master, exp_avg, exp_avg_sq):
        _check(a, F32)
        assert a.size == grad.size
    if param is not None:
        _check(param, param_dtype)
    lib().ora_adamw_tensor_clipped(
        form, grad_dtype, -1 if param is None else param_dtype, grad.size, _ptr(grad), _ptr(master),
        _ptr(exp_avg), _ptr(exp_avg_sq), _ptr(param), lr, beta1, beta2, eps, weight_decay, int(step),
        0 if clip_scale is None else 1, 0.0 if clip_scale is None else float(clip_scale))


def bf16_rank_sum(per_rank: list[np.ndarray]) -> np.ndarray:
    """Sum of W bf16 gradients, rounding to bf16 after each addition in rank order."""
    n = per_rank[0].size
    arrs = [np.ascontiguousarray(a, dtype=np.uint16) for a in per_rank]
    ptrs = (ctypes.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
    out = np.empty(n, np.uint16)
    lib().ora_bf16_rank_sum(n, len(arrs), ptrs, _ptr(out))
    return out


# ---------------------------------------------------------------- per-tensor / per-rank logic

def greedy_owners(numels: list[int], world: int) -> list[int]:
    """Largest tensors first, each to the currently least-loaded rank, ties to the lowest
    rank; equal sizes keep list order (stable sort) -- optimizer.py:46-53."""
    order = sorted(range(len(numels)), key=lambda i: -numels[i])
    loads = [0] * world
    owner = [0] * len(numels)
    for i in order:
        r = min(range(world), key=lambda k: loads[k])
        owner[i] = r
        loads[r] += numels[i]
    return owner


def norm_from_sumsq(total: float) -> float:
    """float(total.sqrt()) of an fp32 total (optimizer.py:154)."""
    return float(np.sqrt(np.float32(total)))


def clip_scale_for(norm: float, max_norm: float) -> float | None:
    """The multiplier optimizer.py:155-156 applies, or None when it does not clip."""
    if max_norm > 0 and norm > max_norm:
        return float(max_norm) / (norm + 1e-6)
    return None


@dataclass
class OracleState:
    """Everything one rank of the reference holds for its owned tensors."""
    master: dict[int, np.ndarray] = field(default_factory=dict)
    exp_avg: dict[int, np.ndarray] = field(default_factory=dict)
    exp_avg_sq: dict[int, np.ndarray] = field(default_factory=dict)
    param_steps: dict[int, int] = field(default_factory=dict)


class OracleZeroOne:
    """All W ranks of the reference optimizer simulated in one process on numpy arrays.

    ``params[i]`` is the (shared) parameter array of tensor i, ``dtypes[i]`` its dtype; the
    parameter copy is identical on every rank after each step (the broadcast of
    optimizer.py:192-194), so one array per tensor represents all ranks.
    """

    def __init__(self, params: list[np.ndarray], dtypes: list[int], lrs: list[float], *, world: int,
                 betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, form: int = FORM_TORCH_CUDA):
        self.world = world
        self.betas = (float(betas[0]), float(betas[1]))
        self.eps = float(eps)
        self.weight_decay = float(weight_decay)
        self.form = form
        self.params = [np.ascontiguousarray(p).reshape(-1).copy() for p in params]
        self.dtypes = list(dtypes)
        self.lrs = [float(x) for x in lrs]
        self.owner = greedy_owners([p.size for p in self.params], world)
        self.state = [OracleState() for _ in range(world)]
        for i, p in enumerate(self.params):
            st = self.state[self.owner[i]]
            st.master[i] = widen(p, self.dtypes[i]).copy()
            st.exp_avg[i] = np.zeros(p.size, np.float32)
            st.exp_avg_sq[i] = np.zeros(p.size, np.float32)
            st.param_steps[i] = 0
        self.step_count = 0
        self.grads: list[np.ndarray | None] = [None] * len(self.params)  # owner-side reduced grads

    def reduce_grads(self, per_rank: list[list[np.ndarray | None]], round_once: bool = False) -> None:
        """all_reduce_grads (optimizer.py:95-143): used = any rank has a grad; the owner
        receives the sum, missing grads counting as zeros.  W == 1 keeps the grads.

        16-bit sums round after every addition in rank order (a chain of reductions in the
        gradient dtype, as a per-hop reduce does); ``round_once`` instead adds in fp32 in rank
        order and rounds once (the peer-to-peer owner sum of the B200 build).  The two agree at
        W = 2, where either rounds the one fp32 sum once."""
        if self.world == 1:
            self.grads = [None if g is None else g.reshape(-1).copy() for g in per_rank[0]]
            return
        out: list[np.ndarray | None] = []
        for i in range(len(self.params)):
            present = [per_rank[r][i] for r in range(self.world)]
            if all(g is None for g in present):
                out.append(None)
                continue
            dt = self.dtypes[i]
            filled = [np.zeros(self.params[i].size, np.float32 if dt == F32 else np.uint16) if g is None
                      else g.reshape(-1) for g in present]
            if round_once and dt != F32:
                acc = widen(filled[0], dt).astype(np.float32).copy()
                for g in filled[1:]:
                    acc = acc + widen(g, dt).astype(np.float32)
                out.append(narrow(acc, dt))
            elif dt == BF16:
                out.append(bf16_rank_sum(filled))
            elif dt == F32:
                acc = filled[0].astype(np.float32).copy()
                for g in filled[1:]:
                    acc = acc + g
                out.append(acc)
            else:
                acc = widen(filled[0], F16)
                for g in filled[1:]:
                    acc = widen(to_f16(acc + widen(g, F16)), F16)
                out.append(to_f16(acc))
        self.grads = out

    def sumsq(self) -> float:
        return sum(sumsq(g, self.dtypes[i]) for i, g in enumerate(self.grads) if g is not None)

    def clip_grad_norm(self, max_norm: float, norm: float | None = None) -> float:
        """Returns the pre-clip global norm; clips the owned grads in place
        (optimizer.py:145-160).  ``norm`` overrides the computed norm (used to replay a
        norm that another implementation summed in a different order)."""
        if norm is None:
            norm = norm_from_sumsq(self.sumsq())
        scale = clip_scale_for(norm, max_norm)
        if scale is not None:
            for i, g in enumerate(self.grads):
                if g is not None:
                    clip_inplace(g, self.dtypes[i], self.form, scale)
        return norm

    def step(self) -> None:
        """optimizer.py:162-194 over every rank's owned tensors."""
        self.step_count += 1
        b1, b2 = self.betas
        for i, g in enumerate(self.grads):
            if g is None:
                continue
            st = self.state[self.owner[i]]
            st.param_steps[i] += 1
            dt = self.dtypes[i]
            adamw_tensor(self.form, g, dt, st.master[i], st.exp_avg[i], st.exp_avg_sq[i],
                         None if dt == F32 else self.params[i], dt, lr=self.lrs[i], beta1=b1, beta2=b2,
                         eps=self.eps, weight_decay=self.weight_decay, step=st.param_steps[i])
            if dt == F32:
                self.params[i] = st.master[i]

    def tensor_state(self, i: int) -> tuple[np.ndarray, np.ndarray, np.ndarray, int]:
        st = self.state[self.owner[i]]
        return st.master[i], st.exp_avg[i], st.exp_avg_sq[i], st.param_steps[i]


def ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """|a - b| in units in the last place of fp32, via the ordered integer mapping; NaNs
    compare equal to NaNs and infinitely far from numbers."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)

    def key(x):
        i = x.view(np.int32).astype(np.int64)
        return np.where(i < 0, -(i & 0x7FFFFFFF), i)

    d = np.abs(key(a) - key(b))
    na, nb = np.isnan(a), np.isnan(b)
    d = np.where(na & nb, 0, d)
    d = np.where(na ^ nb, np.iinfo(np.int64).max, d)
    return d


def max_rel_err(a: np.ndarray, b: np.ndarray) -> float:
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    denom = np.maximum(np.abs(b), np.finfo(np.float32).tiny)
    fin = np.isfinite(a) & np.isfinite(b)
    if not fin.any():
        return 0.0
    return float(np.max(np.abs(a[fin] - b[fin]) / denom[fin]))


def isclose_norm(a: float, b: float, rel: float) -> bool:
    if math.isnan(a) or math.isnan(b):
        return math.isnan(a) and math.isnan(b)
    if math.isinf(a) or math.isinf(b):
        return a == b
    return abs(a - b) <= rel * max(abs(b), 1e-30)
