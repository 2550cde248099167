"""The torch-op restatement (oracle/torch_ops.py) reproduces the reference's golden
vectors bit for bit on CPU -- so the same code run on a CUDA device stands for the
reference there (tests/test_torch_cuda_forms.py)."""
import numpy as np
import pytest

from cases import CASES
from helpers import assert_bits_equal, golden, to_numpy, to_torch
from oracle.torch_ops import TorchZeroOneW1


@pytest.mark.parametrize("case", [c for c in CASES if c.world == 1], ids=lambda c: c.name)
def test_torch_restatement_matches_reference_on_cpu(case):
    import torch
    g = golden(case.name)
    params = [to_torch(p, case.dtype, s) for p, s in zip(case.initial_params(), case.shapes)]
    opt = TorchZeroOneW1(params, case.lr, betas=case.betas, eps=case.eps, weight_decay=case.weight_decay)
    if case.preload_state:
        for i, s in enumerate(case.shapes):
            master, m, v, step = case.preload(i)
            opt.master[i].copy_(torch.from_numpy(master).reshape(s))
            opt.exp_avg[i].copy_(torch.from_numpy(m).reshape(s))
            opt.exp_avg_sq[i].copy_(torch.from_numpy(v).reshape(s))
            opt.steps[i] = step
            if case.dtype != 0:
                params[i].copy_(opt.master[i].to(params[i].dtype))
    for s in range(case.steps):
        grads = [None if x is None else to_torch(x, case.dtype, sh) for x, sh in zip(case.grads(s, 0), case.shapes)]
        norm = opt.step(grads, case.max_norm)
        ref = float(g["norms"][s])
        assert norm == ref or (np.isnan(norm) and np.isnan(ref))
    for i in range(len(case.shapes)):
        assert opt.steps[i] == int(g[f"param_steps_{i}"])
        assert_bits_equal(to_numpy(opt.master[i], 0), g[f"master_{i}"], f"master[{i}]")
        assert_bits_equal(to_numpy(opt.exp_avg[i], 0), g[f"exp_avg_{i}"], f"exp_avg[{i}]")
        assert_bits_equal(to_numpy(opt.exp_avg_sq[i], 0), g[f"exp_avg_sq_{i}"], f"exp_avg_sq[{i}]")
        assert_bits_equal(to_numpy(params[i], case.dtype), g[f"param_{i}"], f"param[{i}]")
