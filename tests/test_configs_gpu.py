"""Parity on the benchmark configurations' parameter sets and value distributions, at a
size the CPU oracle replays in seconds: the leading and trailing tensors of each set
(~40 M parameters: attention / MLP or expert matrices, norm vectors, embeddings cut off),
three optimizer steps through the public API, every element compared with the oracle
(torch-CUDA form, replaying this run's norms):

* qwen3_8b / gemma_12b: grads ~N(0, 1e-4), master ~N(0, 0.02), m ~N(0, 1e-5),
  v ~|N(0, 1e-8)|, step 100;
* qwen3_14b: grads scaled to a global norm of 4 (clip always active), and one step with a
  seeded +inf or NaN in one tensor -- the norm is non-finite and the caller skips the
  step (hybrid_rl/train.py:292-294), leaving every state bit unchanged;
* moe_26b_a4b: per-expert tensors, a seeded 40 % of each layer's experts get all-zero
  (not absent) gradients: they still decay and advance their step.
"""
import math
import zlib

import numpy as np
import pytest

from helpers import Z, assert_bits_equal, to_numpy, to_torch

pytestmark = pytest.mark.gpu

MAX_PARAMS = 40_000_000


def _subset(name):
    from hybridagent_b200 import workloads
    shapes = workloads.WORKLOADS[name]()
    head = workloads.truncated(shapes, MAX_PARAMS // 2)
    tail = []
    total = 0
    for s in reversed(shapes[len(head):]):
        n = math.prod(s)
        if n > MAX_PARAMS // 8:
            continue  # skip embeddings / lm_head
        if total + n > MAX_PARAMS // 2:
            break
        tail.append(s)
        total += n
    return head + tail[::-1]


def _moe_zero_experts(shapes, step, rng_seed):
    """Indices of expert matrices that get all-zero gradients this step (40 % of experts)."""
    rng = np.random.default_rng([rng_seed, step])
    zero = set()
    expert_mats = [i for i, s in enumerate(shapes) if s in ((704, 2816), (2816, 704))]
    # experts are consecutive triples (gate, up, down)
    triples = [expert_mats[k:k + 3] for k in range(0, len(expert_mats) - 2, 3)]
    for t in triples:
        if rng.random() < 0.4:
            zero.update(t)
    return zero


@pytest.mark.parametrize("name", ["qwen3_8b", "gemma_12b", "qwen3_14b", "moe_26b_a4b"])
def test_config_parity(name):
    import torch

    from hybridagent_b200 import ZeroOneAdamW

    shapes = _subset(name)
    numels = [math.prod(s) for s in shapes]
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    init32 = [(rng.standard_normal(n) * 0.02).astype(np.float32) for n in numels]
    init = [Z.to_bf16(x) for x in init32]
    params = [torch.nn.Parameter(to_torch(b, Z.BF16, s, "cuda")) for b, s in zip(init, shapes)]
    opt = ZeroOneAdamW([{"params": params, "lr": 1e-6}], rank=0, world_size=1, weight_decay=0.01)
    ora = Z.OracleZeroOne(init, [Z.BF16] * len(shapes), [1e-6] * len(shapes), world=1, weight_decay=0.01)
    for i, s in enumerate(shapes):
        m = (rng.standard_normal(numels[i]) * 1e-5).astype(np.float32)
        v = np.abs(rng.standard_normal(numels[i]) * 1e-8).astype(np.float32)
        opt.master[i].copy_(torch.from_numpy(init32[i]).reshape(s))
        opt.exp_avg[i].copy_(torch.from_numpy(m).reshape(s))
        opt.exp_avg_sq[i].copy_(torch.from_numpy(v).reshape(s))
        opt.param_steps[i] = 100
        M, EA, EAS, _ = ora.tensor_state(i)
        M[:] = init32[i]
        EA[:] = m
        EAS[:] = v
        ora.state[0].param_steps[i] = 100
    skipped = 0
    for step in range(3):
        grads = [Z.to_bf16((rng.standard_normal(n) * 1e-4).astype(np.float32)) for n in numels]
        if name == "qwen3_14b":
            total = math.sqrt(sum(Z.sumsq(g, Z.BF16) for g in grads))
            grads = [Z.to_bf16(Z.widen(g, Z.BF16) * np.float32(4.0 / total)) for g in grads]
            if step == 1:  # the seeded non-finite step
                bad = int(rng.integers(len(grads)))
                grads[bad][int(rng.integers(numels[bad]))] = Z.to_bf16(np.array([np.inf], np.float32))[0]
        if name == "moe_26b_a4b":
            for i in _moe_zero_experts(shapes, step, 5):
                grads[i] = np.zeros(numels[i], np.uint16)
        opt.zero_grad(set_to_none=True)
        for p, g, s in zip(params, grads, shapes):
            p.grad = to_torch(g, Z.BF16, s, "cuda")
        opt.all_reduce_grads()
        norm = opt.clip_grad_norm(1.0)
        ora.reduce_grads([grads])
        exact = Z.norm_from_sumsq(ora.sumsq())
        assert Z.isclose_norm(norm, exact, 1e-6), (step, norm, exact)
        if not math.isfinite(norm):  # the caller's fail-closed skip
            assert name == "qwen3_14b" and step == 1
            skipped += 1
            continue
        if name == "qwen3_14b":
            assert norm > 3.9  # clipping active
        ora.clip_grad_norm(1.0, norm=norm)
        opt.step()
        ora.step()
    assert skipped == (1 if name == "qwen3_14b" else 0)
    for i in range(len(shapes)):
        master, m, v, steps = ora.tensor_state(i)
        assert opt.param_steps[i] == steps == 100 + 3 - skipped
        assert_bits_equal(to_numpy(opt.master[i], 0), master, f"{name} master[{i}]")
        assert_bits_equal(to_numpy(opt.exp_avg[i], 0), m, f"{name} exp_avg[{i}]")
        assert_bits_equal(to_numpy(opt.exp_avg_sq[i], 0), v, f"{name} exp_avg_sq[{i}]")
        assert_bits_equal(to_numpy(params[i].data, Z.BF16), ora.params[i], f"{name} param[{i}]")
