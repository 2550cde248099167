"""Shared test helpers: golden fixtures, oracle replays and the parity criteria."""
from __future__ import annotations

import os

import numpy as np

from cases import BF16, CASES_BY_NAME, F16, F32, Case
from oracle import zero1 as Z

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as f:
        return {k: f[k] for k in f.files}


def oracle_for(case: Case, form: int) -> Z.OracleZeroOne:
    """The oracle set up exactly as make_golden.py sets up the reference."""
    ora = Z.OracleZeroOne(case.initial_params(), [case.dtype] * len(case.shapes), [case.lr] * len(case.shapes),
                          world=case.world, betas=case.betas, eps=case.eps, weight_decay=case.weight_decay,
                          form=form)
    if case.preload_state:
        for i in range(len(case.shapes)):
            master, m, v, step = case.preload(i)
            M, EA, EAS, _ = ora.tensor_state(i)
            M[:] = master
            EA[:] = m
            EAS[:] = v
            ora.state[ora.owner[i]].param_steps[i] = step
            ora.params[i] = M if case.dtype == F32 else Z.narrow(master, case.dtype, form)
    return ora


def oracle_replay(case: Case, form: int, norms: list[float] | None = None) -> tuple[Z.OracleZeroOne, list[float]]:
    """Runs every step of a case; ``norms`` replays externally computed norms (so the clip
    factor matches the run being compared against)."""
    ora = oracle_for(case, form)
    out = []
    for s in range(case.steps):
        ora.reduce_grads([case.grads(s, r) for r in range(case.world)])
        n = ora.clip_grad_norm(case.max_norm, norm=None if norms is None else norms[s])
        out.append(n)
        if np.isfinite(n) or case.call_step_after_nonfinite:
            ora.step()
    return ora, out


def assert_bits_equal(a: np.ndarray, b: np.ndarray, what: str) -> None:
    a = np.ascontiguousarray(a).reshape(-1)
    b = np.ascontiguousarray(b).reshape(-1)
    if a.dtype == np.float32:
        nan = np.isnan(a) & np.isnan(b)
        diff = (a.view(np.uint32) != b.view(np.uint32)) & ~nan
    else:
        diff = a != b
        if a.dtype == np.uint16:  # bf16 / fp16 NaN encodings may differ between devices
            nan = ((a & 0x7FFF) > 0x7F80) & ((b & 0x7FFF) > 0x7F80)
            diff &= ~nan
    n = int(diff.sum())
    assert n == 0, f"{what}: {n} of {a.size} elements differ (first at {int(np.argmax(diff))})"


def assert_state_close(a: np.ndarray, b: np.ndarray, what: str, *, max_ulp: int = 2, rel: float = 1e-6,
                       lr_ulps: tuple[float, int] | None = None) -> None:
    """The north star's fp32 parity criterion, per element: within ``max_ulp`` units in the
    last place, or a relative error of at most ``rel``; NaN matches NaN.

    ``lr_ulps=(lr, k)`` adds the one documented exception, for masters compared across devices
    (this build / torch's CUDA kernels against the reference's CPU run): torch's CPU and CUDA
    kernels round the update term ``lr * m_hat / (sqrt(v_hat) + eps)`` differently
    (optimizer.py:188-189: ``x / c`` vs ``x * (1 / c)``, MKL's sqrt, ``addcdiv_``'s two forms), by
    up to an ulp of ``lr`` per step; a master within a few updates of zero then differs by more
    than 2 of its own ulps.  Such elements pass if ``|a - b| <= k`` ulps of ``lr``.  ``lr`` may be
    an array, per element the magnitude of that element's update term, where it exceeds ``lr``
    (``m_hat / sqrt(v_hat)`` above 1): a rounding of the term then moves the master by an ulp of
    the term."""
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    b = np.ascontiguousarray(b, dtype=np.float32).reshape(-1)
    ulp = Z.ulp_distance(a, b)
    fin = np.isfinite(a) & np.isfinite(b)
    diff = np.abs(a.astype(np.float64) - b.astype(np.float64))
    rel_err = np.where(fin, diff / np.maximum(np.abs(b.astype(np.float64)), np.finfo(np.float64).tiny), 0.0)
    ok = (ulp <= max_ulp) | (fin & (rel_err <= rel))
    if lr_ulps is not None:
        lr, k = lr_ulps
        ok |= fin & (diff <= k * np.spacing(np.abs(np.asarray(lr, dtype=np.float32))).astype(np.float64))
    bad = ~ok
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {a.size} elements outside {max_ulp} ulp / rel {rel}"
                           f"{'' if lr_ulps is None else f' / {lr_ulps[1]} ulp(lr)'} "
                           f"(worst ulp {int(ulp[bad].max())} at {int(np.argmax(bad))})")


def lr_exception(case: Case) -> tuple[float, int]:
    """``lr_ulps`` for a case: two ulps of its learning rate per step it ran."""
    return case.lr, 2 * case.steps


# ---------------------------------------------------------------- torch conversions
def torch_dtype(code: int):
    import torch
    return {F32: torch.float32, BF16: torch.bfloat16, F16: torch.float16}[code]


def to_torch(a: np.ndarray, code: int, shape=None, device="cpu"):
    """numpy fp32 values / 16-bit patterns -> torch tensor of dtype ``code``."""
    import torch
    a = np.ascontiguousarray(a)
    t = torch.from_numpy(a.copy()) if code == F32 else torch.from_numpy(a.view(np.int16).copy()).view(torch_dtype(code))
    if shape is not None:
        t = t.reshape(shape)
    return t.to(device)


def to_numpy(t, code: int) -> np.ndarray:
    """torch tensor -> numpy fp32 values / 16-bit patterns (flat)."""
    import torch
    t = t.detach().to("cpu").contiguous().reshape(-1)
    if code == F32:
        return t.numpy().copy()
    return t.view(torch.int16).numpy().view(np.uint16).copy()
