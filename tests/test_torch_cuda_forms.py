"""Pins the oracle's torch-CUDA rounding form against torch's own CUDA kernels: the
reference's op sequence (oracle/torch_ops.py) run on the GPU must equal the oracle
replayed with the same norms, bit for bit, on every single-rank golden case."""
import numpy as np
import pytest

from cases import CASES
from helpers import Z, assert_bits_equal, oracle_replay, to_numpy, to_torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", [c for c in CASES if c.world == 1], ids=lambda c: c.name)
def test_torch_cuda_equals_oracle_cuda_form(case):
    import torch
    from oracle.torch_ops import TorchZeroOneW1
    dev = "cuda"
    params = [to_torch(p, case.dtype, s, dev) for p, s in zip(case.initial_params(), case.shapes)]
    opt = TorchZeroOneW1(params, case.lr, betas=case.betas, eps=case.eps, weight_decay=case.weight_decay)
    if case.preload_state:
        for i, s in enumerate(case.shapes):
            master, m, v, step = case.preload(i)
            opt.master[i].copy_(torch.from_numpy(master).reshape(s))
            opt.exp_avg[i].copy_(torch.from_numpy(m).reshape(s))
            opt.exp_avg_sq[i].copy_(torch.from_numpy(v).reshape(s))
            opt.steps[i] = step
            if case.dtype != Z.F32:
                params[i].copy_(opt.master[i].to(params[i].dtype))
    norms = []
    for s in range(case.steps):
        grads = [None if x is None else to_torch(x, case.dtype, sh, dev) for x, sh in zip(case.grads(s, 0), case.shapes)]
        norms.append(opt.step(grads, case.max_norm))
    ora, _ = oracle_replay(case, Z.FORM_TORCH_CUDA, norms=norms)
    for i in range(len(case.shapes)):
        master, m, v, steps = ora.tensor_state(i)
        assert steps == opt.steps[i]
        assert_bits_equal(to_numpy(opt.master[i], 0), master, f"master[{i}]")
        assert_bits_equal(to_numpy(opt.exp_avg[i], 0), m, f"exp_avg[{i}]")
        assert_bits_equal(to_numpy(opt.exp_avg_sq[i], 0), v, f"exp_avg_sq[{i}]")
        assert_bits_equal(to_numpy(params[i], case.dtype), ora.params[i], f"param[{i}]")
    # the oracle's exact norm agrees with torch's fp32 CUDA sum
    _, own = oracle_replay(case, Z.FORM_TORCH_CUDA, norms=None)
    for a, b in zip(own, norms):
        assert Z.isclose_norm(a, b, 1e-6), (a, b)


def _fma(a, b, c):
    """fp32 fused multiply-add through double (exact product; one double rounding then
    one fp32 rounding -- equal to a true fma except in double-rounding ties, which random
    inputs of this size do not hit)."""
    return (np.asarray(a, np.float64) * np.asarray(b, np.float64) + np.asarray(c, np.float64)).astype(np.float32)


def test_scalar_division_form():
    """torch CUDA computes ``tensor / python_float`` as tensor * float32(1.0 / c): the
    reciprocal in double, rounded once (optimizer.py:188-189 divide by the corrections)."""
    import torch
    g = torch.Generator().manual_seed(2)
    x = torch.randn(1 << 16, generator=g) * 1e-3
    X = x.numpy()
    xd = x.cuda()
    other_form_differs = False
    for beta in (0.9, 0.999):
        for t in list(range(1, 40)) + [99, 100, 101, 1000, 10000]:
            c = 1.0 - beta ** t
            got = (xd / c).cpu().numpy()
            assert np.array_equal(got.view(np.uint32), (X * np.float32(1.0 / c)).view(np.uint32)), (beta, t)
            other_form_differs |= not np.array_equal(got, X * (np.float32(1) / np.float32(c)))
    assert other_form_differs  # the fp32-reciprocal form is distinguishable and wrong


@pytest.mark.parametrize("lr,wd", [(1e-3, 0.1), (1e-6, 0.01)])
def test_elementwise_op_forms(lr, wd):
    """Each op of optimizer.py:184-189 on torch CUDA against its oracle form, fed torch's
    own intermediates."""
    import torch
    f32 = np.float32
    g = torch.Generator().manual_seed(3)
    n = 1 << 18
    grad, m, v, ms = (torch.randn(n, generator=g) * s for s in (1e-3, 1e-3, 1e-6, 0.02))
    v = v.abs()
    b1, b2, eps, t = 0.9, 0.999, 1e-8, 3
    c1, c2 = 1 - b1 ** t, 1 - b2 ** t
    G, MS = grad.numpy(), ms.numpy()
    gd, md, vd, msd = (x.cuda() for x in (grad, m, v, ms))
    msd.mul_(1.0 - lr * wd)
    A = msd.cpu().numpy()
    assert np.array_equal(A, MS * f32(1.0 - lr * wd))
    md.mul_(b1)
    MB = md.cpu().numpy()
    md.add_(gd, alpha=1.0 - b1)
    assert np.array_equal(md.cpu().numpy(), _fma(f32(1 - b1), G, MB))
    vd.mul_(b2)
    VB = vd.cpu().numpy()
    vd.addcmul_(gd, gd, value=1.0 - b2)
    V = vd.cpu().numpy()
    assert np.array_equal(V, _fma(f32(1 - b2), G * G, VB))
    den = (vd / c2).sqrt().add_(eps)
    D = den.cpu().numpy()
    assert np.array_equal(D, np.sqrt((V * f32(1.0 / c2)).astype(np.float64)).astype(f32) + f32(eps))
    mh = md / c1
    MH = mh.cpu().numpy()
    msd.addcdiv_(mh, den, value=-lr)
    assert np.array_equal(msd.cpu().numpy(), _fma(f32(-lr), MH / D, A))
