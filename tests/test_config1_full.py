"""BASELINE configuration 1 at its real shapes (64 fp32 tensors, 8,912,896 parameters, fresh
gradients ~N(0, 1e-3) for 10 steps, lr 1e-6, wd 0.01, clip 1.0 -- every step clips), pinned to
the unmodified reference (tests/golden/cfg1_full.npz: its norms, the SHA-256 of every final
array, and 50,000 seeded sample positions; written by tests/golden/make_golden.py).

CPU: the torch restatement reproduces every digest and norm; the oracle's torch-CPU form,
given the reference's norms, reproduces every exp_avg / exp_avg_sq digest.
GPU: the product's norms agree with the reference's to 2 fp32 ulp; its state and parameters
equal the oracle's torch-CUDA form replaying those norms, bit for bit, on every element; and
given the reference's own norms its state matches the reference at every sample position:
exp_avg exactly, master within 2 ulp, exp_avg_sq within 3 ulp (torch's CPU and CUDA kernels
round ``addcmul_`` differently, optimizer.py:187, and ten steps accumulate it)."""
import numpy as np
import pytest

from cases import CASES_BY_NAME, digest, sample_positions
from helpers import Z, assert_bits_equal, golden, oracle_for, to_numpy, to_torch

CASE = CASES_BY_NAME["cfg1_full"]


def _samples(arrays, tensor, offset):
    return np.array([arrays[t].reshape(-1)[o] for t, o in zip(tensor, offset)], dtype=np.float32)


def test_config1_shapes_are_baseline_config1():
    from hybridagent_b200 import workloads
    assert CASE.shapes == workloads.config1_cpu()
    assert sum(CASE.numels) == 8_912_896


def test_torch_restatement_reproduces_reference_digests():
    import torch

    from oracle.torch_ops import TorchZeroOneW1
    g = golden(CASE.name)
    threads = torch.get_num_threads()
    torch.set_num_threads(1)  # as the golden run (make_golden.py): one summation order
    try:
        params = [to_torch(p, CASE.dtype, s) for p, s in zip(CASE.initial_params(), CASE.shapes)]
        opt = TorchZeroOneW1(params, CASE.lr, betas=CASE.betas, eps=CASE.eps, weight_decay=CASE.weight_decay)
        for s in range(CASE.steps):
            norm = opt.step([to_torch(x, CASE.dtype, sh) for x, sh in zip(CASE.grads(s, 0), CASE.shapes)],
                            CASE.max_norm)
            assert norm == float(g["norms"][s]), s
    finally:
        torch.set_num_threads(threads)
    for i in range(len(CASE.shapes)):
        for key, t in (("master", opt.master[i]), ("exp_avg", opt.exp_avg[i]), ("exp_avg_sq", opt.exp_avg_sq[i]),
                       ("param", params[i])):
            assert digest(to_numpy(t, 0)) == g[f"sha256_{key}"][i], (key, i)


def test_oracle_cpu_form_with_reference_norms():
    g = golden(CASE.name)
    ora = oracle_for(CASE, Z.FORM_TORCH_CPU)
    for s in range(CASE.steps):
        ora.reduce_grads([CASE.grads(s, 0)])
        ora.clip_grad_norm(CASE.max_norm, norm=float(g["norms"][s]))
        ora.step()
    tensor, offset = sample_positions(CASE)
    for i in range(len(CASE.shapes)):
        _, m, v, steps = ora.tensor_state(i)
        assert steps == int(g["param_steps"][i])
        assert digest(m) == g["sha256_exp_avg"][i], i
        assert digest(v) == g["sha256_exp_avg_sq"][i], i
    master = _samples([ora.tensor_state(i)[0] for i in range(len(CASE.shapes))], tensor, offset)
    assert int(Z.ulp_distance(master, g["sample_master"]).max()) <= 2


@pytest.mark.gpu
def test_config1_on_gpu_against_reference():
    import torch

    from hybridagent_b200 import ZeroOneAdamW
    g = golden(CASE.name)
    dev = torch.device("cuda", 0)
    tensor, offset = sample_positions(CASE)

    def run(replay_reference_norms: bool):
        params = [torch.nn.Parameter(to_torch(p, CASE.dtype, s, dev))
                  for p, s in zip(CASE.initial_params(), CASE.shapes)]
        opt = ZeroOneAdamW([{"params": params, "lr": CASE.lr}], rank=0, world_size=1, betas=CASE.betas,
                           eps=CASE.eps, weight_decay=CASE.weight_decay)
        norms = []
        for s in range(CASE.steps):
            opt.zero_grad(set_to_none=True)
            for p, x, sh in zip(params, CASE.grads(s, 0), CASE.shapes):
                p.grad = to_torch(x, CASE.dtype, sh, dev)
            opt.all_reduce_grads()
            norms.append(opt.clip_grad_norm(CASE.max_norm))
            if replay_reference_norms:  # the clip factor of the reference's norm (optimizer.py:156)
                opt._pending_clip = CASE.max_norm / (float(g["norms"][s]) + 1e-6)
            opt.step()
        torch.cuda.synchronize()
        state = [[to_numpy(d[i], 0) for i in range(len(CASE.shapes))] for d in (opt.master, opt.exp_avg, opt.exp_avg_sq)]
        return norms, state, [to_numpy(p.data, 0) for p in params]

    # own norms: within 2 fp32 ulp of the reference's; every element equal to the oracle's CUDA form
    norms, state, params = run(False)
    ulps = Z.ulp_distance(np.float32(norms), np.float32(g["norms"]))
    assert int(ulps.max()) <= 2, (norms, g["norms"].tolist())
    ora = oracle_for(CASE, Z.FORM_TORCH_CUDA)
    for s in range(CASE.steps):
        ora.reduce_grads([CASE.grads(s, 0)])
        ora.clip_grad_norm(CASE.max_norm, norm=norms[s])
        ora.step()
    for i in range(len(CASE.shapes)):
        m_o, ea_o, eas_o, _ = ora.tensor_state(i)
        assert_bits_equal(state[0][i], m_o, f"master[{i}]")
        assert_bits_equal(state[1][i], ea_o, f"exp_avg[{i}]")
        assert_bits_equal(state[2][i], eas_o, f"exp_avg_sq[{i}]")
        assert_bits_equal(params[i], ora.params[i], f"param[{i}]")

    # the reference's norms: the reference's values at every sample position
    _, state, params = run(True)
    got = [_samples(a, tensor, offset) for a in state]
    assert np.array_equal(got[1].view(np.uint32), g["sample_exp_avg"].view(np.uint32))
    assert int(Z.ulp_distance(got[0], g["sample_master"]).max()) <= 2
    assert int(Z.ulp_distance(got[2], g["sample_exp_avg_sq"]).max()) <= 3
    assert np.array_equal(_samples(params, tensor, offset).view(np.uint32), got[0].view(np.uint32))
