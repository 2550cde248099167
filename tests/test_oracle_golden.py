"""Pins the CPU oracle against golden vectors written by the unmodified reference
optimizer (tests/golden/make_golden.py, torch 2.11 CPU).

The oracle's torch-CPU rounding form must reproduce the reference's exp_avg and
exp_avg_sq bit for bit and its master weights to the parity criterion (torch's CPU sqrt
goes through MKL and can differ from the correctly rounded sqrt by 1 ulp, which shows in
the master only with large learning rates).  The oracle's norm (exact fp64 sum of the
squares, then fp32 as the reference) must agree with the reference's fp32 sum to 1e-6.
The torch-CUDA rounding form -- the one the GPU kernels follow -- differs from torch's CPU
kernels only in rounding, so it is held to the same criterion on the state.
"""
import numpy as np
import pytest

from cases import CASES
from helpers import Z, assert_bits_equal, assert_state_close, golden, lr_exception, oracle_replay

NORM_REL = 1e-6


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_owner_map(case):
    g = golden(case.name)
    assert Z.greedy_owners(case.numels, case.world) == g["owner"].tolist()


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_norms(case):
    g = golden(case.name)
    ora, norms = oracle_replay(case, Z.FORM_TORCH_CPU)
    for s, (mine, ref) in enumerate(zip(norms, g["norms"].tolist())):
        assert Z.isclose_norm(mine, ref, NORM_REL), f"step {s}: oracle norm {mine} vs reference {ref}"


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_state_cpu_form(case):
    g = golden(case.name)
    ora, _ = oracle_replay(case, Z.FORM_TORCH_CPU, norms=g["norms"].tolist())
    for i in range(len(case.shapes)):
        master, m, v, steps = ora.tensor_state(i)
        assert steps == int(g[f"param_steps_{i}"])
        assert_bits_equal(m, g[f"exp_avg_{i}"], f"exp_avg[{i}]")
        assert_bits_equal(v, g[f"exp_avg_sq_{i}"], f"exp_avg_sq[{i}]")
        # MKL's sqrt on the reference's host vs the C library's here: the master within the criterion
        assert_state_close(master, g[f"master_{i}"], f"master[{i}]", lr_ulps=lr_exception(case))
        if case.dtype == Z.F32:
            assert_state_close(ora.params[i], g[f"param_{i}"], f"param[{i}]", lr_ulps=lr_exception(case))
        else:
            # the low-precision copy is round-to-nearest-even of the master, bit for bit
            assert_bits_equal(Z.narrow(g[f"master_{i}"], case.dtype, Z.FORM_TORCH_CPU), g[f"param_{i}"],
                              f"param[{i}] from golden master")
            assert_bits_equal(Z.narrow(master, case.dtype, Z.FORM_TORCH_CPU), ora.params[i], f"oracle param[{i}]")


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_state_cuda_form_within_tolerance(case):
    g = golden(case.name)
    ora, _ = oracle_replay(case, Z.FORM_TORCH_CUDA, norms=g["norms"].tolist())
    for i in range(len(case.shapes)):
        master, m, v, _ = ora.tensor_state(i)
        assert_bits_equal(m, g[f"exp_avg_{i}"], f"exp_avg[{i}]")  # same fma form on both devices
        assert_state_close(v, g[f"exp_avg_sq_{i}"], f"exp_avg_sq[{i}]")
        assert_state_close(master, g[f"master_{i}"], f"master[{i}]", lr_ulps=lr_exception(case))


def test_skip_decisions():
    """inf -> +inf norm, nan -> nan norm: the caller's fail-closed check fires on the same step."""
    for name, want in (("bf16_inf", np.isposinf), ("bf16_nan", np.isnan)):
        g = golden(name)
        ora, norms = oracle_replay(next(c for c in CASES if c.name == name), Z.FORM_TORCH_CPU)
        assert np.isfinite(g["norms"][0]) and want(g["norms"][1])
        assert np.isfinite(norms[0]) and want(norms[1])


def test_sumsq_exactness():
    """bf16 squares are exact in fp32; the fp64 accumulation is exact for small sums."""
    x = np.array([1.5, -2.0, 0.25, 3.0], np.float32)
    assert Z.sumsq(Z.to_bf16(x), Z.BF16) == float(np.sum(x.astype(np.float64) ** 2))


def test_clip_multiplier_forms():
    scale = 1.0 / (3.7 + 1e-6)
    assert Z.clip_multiplier(Z.BF16, Z.FORM_TORCH_CUDA, scale) == float(np.float32(scale))
    assert Z.clip_multiplier(Z.BF16, Z.FORM_TORCH_CPU, scale) == float(np.float32(scale))
    rounded = Z.clip_multiplier(Z.BF16, Z.SCALAR_IN_DTYPE, scale)
    assert rounded != float(np.float32(scale)) and abs(rounded - scale) / scale < 2 ** -8


def test_ulp_distance():
    a = np.array([1.0, -0.0, np.nan, 1.0], np.float32)
    b = np.array([np.nextafter(np.float32(1.0), np.float32(2.0)), 0.0, np.nan, np.nan], np.float32)
    d = Z.ulp_distance(a, b)
    assert d[0] == 1 and d[1] == 0 and d[2] == 0 and d[3] > 2 ** 40
