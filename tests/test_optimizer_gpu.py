"""The drop-in ZeroOneAdamW at world size 1 on a B200, driven exactly like the
reference's trainer (zero_grad -> grads -> all_reduce_grads -> clip_grad_norm -> step,
hybrid_rl/train.py:248-295) over every single-rank golden case.

* state and parameters: bit for bit equal to the oracle's torch-CUDA form replayed with
  this optimizer's norms; and, run again with the reference's norms (the clip factor its
  fp32 norm gives), within the parity criterion of the reference's own CPU results (the
  golden vectors: exp_avg bit for bit; exp_avg_sq within 2 ulp or 1e-6 relative; the master
  too, or within two ulps of lr per step where torch's CPU and CUDA kernels round the update
  term differently);
* norms: within 1e-6 relative of the reference's;
* skip decisions: the same steps return non-finite norms.
"""
import math

import numpy as np
import pytest

from cases import CASES
from helpers import (Z, assert_bits_equal, assert_state_close, golden, lr_exception, oracle_replay, to_numpy,
                     to_torch)

pytestmark = pytest.mark.gpu

NORM_REL = 1e-6


def build(case, **kw):
    import torch
    from hybridagent_b200 import ZeroOneAdamW
    params = [torch.nn.Parameter(to_torch(p, case.dtype, s, "cuda")) for p, s in zip(case.initial_params(), case.shapes)]
    opt = ZeroOneAdamW([{"params": params, "lr": case.lr}], rank=0, world_size=1, betas=case.betas, eps=case.eps,
                       weight_decay=case.weight_decay, **kw)
    if case.preload_state:
        for i, s in enumerate(case.shapes):
            master, m, v, step = case.preload(i)
            opt.master[i].copy_(torch.from_numpy(master).reshape(s))
            opt.exp_avg[i].copy_(torch.from_numpy(m).reshape(s))
            opt.exp_avg_sq[i].copy_(torch.from_numpy(v).reshape(s))
            opt.param_steps[i] = step
            if not opt.master_is_parameter[i]:
                params[i].data.copy_(opt.master[i].to(params[i].dtype))
    return params, opt


def run_steps(case, params, opt, steps, ref_norms=None):
    """``ref_norms``: after each clip_grad_norm, the clip factor the reference's own norm gives
    (optimizer.py:155-156) replaces this build's, isolating the per-element arithmetic."""
    norms = []
    for s in steps:
        opt.zero_grad(set_to_none=True)
        for p, g, shape in zip(params, case.grads(s, 0), case.shapes):
            p.grad = None if g is None else to_torch(g, case.dtype, shape, "cuda")
        opt.all_reduce_grads()
        n = opt.clip_grad_norm(case.max_norm)
        norms.append(n)
        if ref_norms is not None:
            ref = float(ref_norms[s])
            opt._pending_clip = case.max_norm / (ref + 1e-6) if case.max_norm > 0 and ref > case.max_norm else None
        if math.isfinite(n) or case.call_step_after_nonfinite:
            opt.step()
    return norms


@pytest.mark.parametrize("case", [c for c in CASES if c.world == 1], ids=lambda c: c.name)
def test_matches_oracle_and_reference(case):
    g = golden(case.name)
    params, opt = build(case)
    assert opt.owner == g["owner"].tolist()
    norms = run_steps(case, params, opt, range(case.steps))
    for s, (mine, ref) in enumerate(zip(norms, g["norms"].tolist())):
        assert Z.isclose_norm(mine, ref, NORM_REL), f"step {s}: {mine} vs reference {ref}"
    ora, _ = oracle_replay(case, Z.FORM_TORCH_CUDA, norms=norms)
    for i in range(len(case.shapes)):
        master, m, v, steps = ora.tensor_state(i)
        assert opt.param_steps[i] == steps == int(g[f"param_steps_{i}"])
        assert_bits_equal(to_numpy(opt.master[i], 0), master, f"master[{i}]")
        assert_bits_equal(to_numpy(opt.exp_avg[i], 0), m, f"exp_avg[{i}]")
        assert_bits_equal(to_numpy(opt.exp_avg_sq[i], 0), v, f"exp_avg_sq[{i}]")
        assert_bits_equal(to_numpy(params[i].data, case.dtype), ora.params[i], f"param[{i}]")
    assert opt.step_count == case.steps
    # against the reference's own (CPU) results, given the reference's norms: exp_avg bit for bit,
    # exp_avg_sq within the criterion, the master within it or the documented lr exception (torch's
    # CPU and CUDA kernels round the update term differently); the norm itself is held above
    params, opt = build(case)
    run_steps(case, params, opt, range(case.steps), ref_norms=g["norms"])
    for i in range(len(case.shapes)):
        assert_bits_equal(to_numpy(opt.exp_avg[i], 0), g[f"exp_avg_{i}"], f"ref exp_avg[{i}]")
        assert_state_close(to_numpy(opt.exp_avg_sq[i], 0), g[f"exp_avg_sq_{i}"], f"ref exp_avg_sq[{i}]")
        assert_state_close(to_numpy(opt.master[i], 0), g[f"master_{i}"], f"ref master[{i}]", lr_ulps=lr_exception(case))


def test_skip_decisions_match_reference():
    for name, want in (("bf16_inf", math.isinf), ("bf16_nan", math.isnan)):
        case = next(c for c in CASES if c.name == name)
        params, opt = build(case)
        norms = run_steps(case, params, opt, range(case.steps))
        g = golden(name)["norms"]
        assert [math.isfinite(x) for x in norms] == [bool(np.isfinite(x)) for x in g]
        assert want(norms[1])


def test_state_dict_round_trip_is_bit_identical():
    import torch
    from hybridagent_b200 import ZeroOneAdamW
    case = next(c for c in CASES if c.name == "bf16_clip")
    params, opt = build(case)
    run_steps(case, params, opt, range(2))
    sd = opt.state_dict()
    fresh = [torch.nn.Parameter(p.detach().clone()) for p in params]
    opt2 = ZeroOneAdamW([{"params": fresh, "lr": case.lr}], rank=0, world_size=1, betas=case.betas, eps=case.eps,
                        weight_decay=case.weight_decay)
    opt2.load_state_dict(sd)
    assert opt2.step_count == 2 and dict(opt2.param_steps) == dict(opt.param_steps)
    run_steps(case, params, opt, [2])
    run_steps(case, fresh, opt2, [2])
    for i in range(len(params)):
        assert torch.equal(params[i].data, fresh[i].data)
        for a, b in ((opt.master, opt2.master), (opt.exp_avg, opt2.exp_avg), (opt.exp_avg_sq, opt2.exp_avg_sq)):
            assert torch.equal(a[i], b[i])
    bad = dict(sd, world=2)
    with pytest.raises(ValueError):
        opt2.load_state_dict(bad)


def test_pending_clip_semantics():
    """apply_pending_clip scales the gradients exactly like the reference's in-place
    mul_; a second clip_grad_norm sees the clipped gradients."""
    import torch
    case = next(c for c in CASES if c.name == "bf16_big_lr_clip")
    params, opt = build(case)
    grads = case.grads(0, 0)
    for p, g, s in zip(params, grads, case.shapes):
        p.grad = to_torch(g, case.dtype, s, "cuda")
    n1 = opt.clip_grad_norm(1.0)
    assert n1 > 1.0
    opt.apply_pending_clip()
    scale = 1.0 / (n1 + 1e-6)
    for p, g in zip(params, grads):
        want = g.copy()
        Z.clip_inplace(want, case.dtype, Z.FORM_TORCH_CUDA, scale)
        assert_bits_equal(to_numpy(p.grad, case.dtype), want, "clipped grad")
    n2 = opt.clip_grad_norm(1.0)
    assert abs(n2 - 1.0) < 1e-2
    opt.zero_grad(set_to_none=False)
    assert all(torch.count_nonzero(p.grad) == 0 for p in params)


def test_constructor_contract():
    import torch
    from hybridagent_b200 import ZeroOneAdamW
    p = torch.nn.Parameter(torch.zeros(8, device="cuda"))
    with pytest.raises(ValueError, match="betas"):
        ZeroOneAdamW([{"params": [p], "lr": 1e-3}], rank=0, world_size=1, betas=(0.9, 1.0))
    with pytest.raises(ValueError, match="rank/world"):
        ZeroOneAdamW([{"params": [p], "lr": 1e-3}], rank=1, world_size=1)
    with pytest.raises(ValueError, match="no trainable"):
        ZeroOneAdamW([{"params": [torch.zeros(3, device="cuda")], "lr": 1e-3}], rank=0, world_size=1)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        ZeroOneAdamW([{"params": [torch.nn.Parameter(torch.zeros(3))], "lr": 1e-3}], rank=0, world_size=1)
    with pytest.raises(NotImplementedError):
        ZeroOneAdamW([{"params": [p], "lr": 1e-3}], rank=0, world_size=1, use_8bit=True)
    # duplicates and frozen parameters are dropped like optimizer.py:36-44
    q = torch.nn.Parameter(torch.zeros(4, device="cuda"), requires_grad=False)
    opt = ZeroOneAdamW([{"params": [p, p, q], "lr": 1e-3}, {"params": [p], "lr": 1.0}], rank=0, world_size=1)
    assert len(opt.params) == 1 and opt.lrs == [1e-3]
    assert opt.state_summary() == "ZeRO-1 FP32 AdamW: 1 tensors; rank 0 owns 0.0M parameters"


def test_mixed_dtypes_and_strided_grads():
    """bf16, fp16 and fp32 parameters in one optimizer (one launch per dtype class) with
    non-contiguous gradients; every tensor bit for bit equal to the oracle."""
    import torch
    from hybridagent_b200 import ZeroOneAdamW
    rng = np.random.default_rng(4)
    spec = [((64, 96), Z.BF16), ((32,), Z.F32), ((100,), Z.BF16), ((48, 16), Z.F32), ((40, 24), Z.F16)]
    init = [Z.narrow((rng.standard_normal(int(np.prod(s))) * 0.02).astype(np.float32), d) for s, d in spec]
    params = [torch.nn.Parameter(to_torch(b, d, s, "cuda")) for b, (s, d) in zip(init, spec)]
    opt = ZeroOneAdamW([{"params": params[:3], "lr": 1e-3}, {"params": params[3:], "lr": 3e-4}], rank=0,
                       world_size=1, weight_decay=0.05)
    ora = Z.OracleZeroOne(init, [d for _, d in spec], [1e-3, 1e-3, 1e-3, 3e-4, 3e-4], world=1, weight_decay=0.05)
    for step in range(3):
        grads = [Z.narrow((rng.standard_normal(int(np.prod(s))) * 0.3).astype(np.float32), d) for s, d in spec]
        for p, g, (s, d) in zip(params, grads, spec):
            t = to_torch(g, d, s, "cuda")
            p.grad = t.t().contiguous().t() if len(s) == 2 else t  # column-major storage, same values
            assert len(s) == 1 or not p.grad.is_contiguous()
        norm = opt.clip_grad_norm(1.0)
        opt.step()
        ora.reduce_grads([grads])
        ora.clip_grad_norm(1.0, norm=norm)
        ora.step()
    for i, (s, d) in enumerate(spec):
        master, m, v, _ = ora.tensor_state(i)
        assert_bits_equal(to_numpy(opt.master[i], 0), master, f"master[{i}]")
        assert_bits_equal(to_numpy(opt.exp_avg[i], 0), m, f"exp_avg[{i}]")
        assert_bits_equal(to_numpy(opt.exp_avg_sq[i], 0), v, f"exp_avg_sq[{i}]")
        assert_bits_equal(to_numpy(params[i].data, d), ora.params[i], f"param[{i}]")


def test_apply_pending_clip_scales_strided_gradients_in_place():
    import torch
    from hybridagent_b200 import ZeroOneAdamW
    rng = np.random.default_rng(8)
    shape = (48, 80)
    g = Z.to_bf16((rng.standard_normal(48 * 80) * 0.5).astype(np.float32))
    p = torch.nn.Parameter(torch.zeros(shape, dtype=torch.bfloat16, device="cuda"))
    opt = ZeroOneAdamW([{"params": [p], "lr": 1e-3}], rank=0, world_size=1)
    p.grad = to_torch(g, Z.BF16, shape, "cuda").t().contiguous().t()
    assert not p.grad.is_contiguous()
    n = opt.clip_grad_norm(1.0)
    assert n > 1.0
    opt.apply_pending_clip()
    want = g.copy()
    Z.clip_inplace(want, Z.BF16, Z.FORM_TORCH_CUDA, 1.0 / (n + 1e-6))
    assert_bits_equal(to_numpy(p.grad, Z.BF16), want, "strided clipped grad")


def test_checkpoint_files_resume_bit_identically(tmp_path):
    import torch
    from hybridagent_b200 import ZeroOneAdamW
    from hybridagent_b200.checkpoint import load_optimizer_state, save_optimizer_state
    case = next(c for c in CASES if c.name == "bf16_sparse")
    params, opt = build(case)
    run_steps(case, params, opt, range(2))
    save_optimizer_state(opt, tmp_path / "checkpoint-2")
    fresh = [torch.nn.Parameter(p.detach().clone()) for p in params]
    opt2 = ZeroOneAdamW([{"params": fresh, "lr": case.lr}], rank=0, world_size=1, betas=case.betas, eps=case.eps,
                        weight_decay=case.weight_decay)
    load_optimizer_state(opt2, tmp_path / "checkpoint-2")
    run_steps(case, params, opt, [2])
    run_steps(case, fresh, opt2, [2])
    for i in range(len(params)):
        assert torch.equal(params[i].data, fresh[i].data)
        assert torch.equal(opt.exp_avg_sq[i], opt2.exp_avg_sq[i]) and torch.equal(opt.master[i], opt2.master[i])
        assert opt.param_steps[i] == opt2.param_steps[i]


def test_ten_thousand_ragged_tensors():
    """10,000 tensors of every small length (every numel mod 8, 1-element tensors, a few
    multi-chunk ones) through the public API, two clipped steps with some gradients absent:
    every element bit for bit equal to the oracle (the MoE set's 11,852-tensor scale)."""
    from cases import BF16, Case
    rng = np.random.default_rng(10_000)
    sizes = [int(n) for n in rng.integers(1, 300, 10_000)]
    sizes[:8] = [1, 2, 3, 4, 5, 6, 7, 8]
    sizes[100:103] = [16383, 16385, 70001]
    overrides = {(s, -1, int(i)): "none" for s in range(2) for i in rng.integers(0, len(sizes), 50)}
    case = Case("many_tensors", 99, [(n,) for n in sizes], BF16, steps=2, grad_sigma=3e-2, lr=1e-3,
                overrides=overrides)
    params, opt = build(case)
    norms = run_steps(case, params, opt, range(case.steps))
    assert all(math.isfinite(n) and n > case.max_norm for n in norms)  # clip active
    ora, _ = oracle_replay(case, Z.FORM_TORCH_CUDA, norms=norms)
    got_master = to_numpy(torch_cat([opt.master[i].reshape(-1) for i in range(len(sizes))]), 0)
    got_m = to_numpy(torch_cat([opt.exp_avg[i].reshape(-1) for i in range(len(sizes))]), 0)
    got_v = to_numpy(torch_cat([opt.exp_avg_sq[i].reshape(-1) for i in range(len(sizes))]), 0)
    got_p = to_numpy(torch_cat([p.data.reshape(-1) for p in params]), case.dtype)
    want = [ora.tensor_state(i) for i in range(len(sizes))]
    assert_bits_equal(got_master, np.concatenate([w[0] for w in want]), "master")
    assert_bits_equal(got_m, np.concatenate([w[1] for w in want]), "exp_avg")
    assert_bits_equal(got_v, np.concatenate([w[2] for w in want]), "exp_avg_sq")
    assert_bits_equal(got_p, np.concatenate(ora.params), "param")
    assert [opt.param_steps[i] for i in range(len(sizes))] == [w[3] for w in want]


def torch_cat(ts):
    import torch
    return torch.cat(ts)


def test_parameters_written_behind_the_optimizer_are_rewritten():
    """Steps write only the changed groups of the bf16 copies unless a parameter or master was
    written by anything else since: torch's version counters catch in-place writes (here a
    parameter zeroed with copy_), mark_parameters_dirty() the writes through .data; the next
    step then writes every parameter in full, and every parameter ends equal to the oracle."""
    import torch
    case = next(c for c in CASES if c.name == "bf16_preloaded")
    params, opt = build(case)  # build() writes the masters: the first step is a full write
    norms = run_steps(case, params, opt, [0])
    assert opt.dense_steps == 1
    norms += run_steps(case, params, opt, [1])
    assert opt.dense_steps == 1  # clean: changed groups only
    with torch.no_grad():
        params[0].copy_(torch.zeros_like(params[0]))
    params[5].data.fill_(3.0)
    opt.mark_parameters_dirty([5])
    norms += run_steps(case, params, opt, [2])
    assert opt.dense_steps == 2
    ora, _ = oracle_replay(case, Z.FORM_TORCH_CUDA, norms=norms)
    for i in range(len(case.shapes)):
        assert_bits_equal(to_numpy(params[i].data, case.dtype), ora.params[i], f"param[{i}]")
        assert_bits_equal(to_numpy(opt.master[i], 0), ora.tensor_state(i)[0], f"master[{i}]")


def test_staged_tables_follow_changes_and_skips():
    """clip_grad_norm uploads the next update's tables before its host read; step() uses them
    only if nothing changed: a step count edited between the two calls is honoured, and a step
    the caller skips after clip_grad_norm advances no count."""
    import torch
    from helpers import oracle_for
    case = next(c for c in CASES if c.name == "bf16_clip")
    params, opt = build(case)
    ora = oracle_for(case, Z.FORM_TORCH_CUDA)

    def grads_in(s):
        opt.zero_grad(set_to_none=True)
        for p, g, shape in zip(params, case.grads(s, 0), case.shapes):
            p.grad = to_torch(g, case.dtype, shape, "cuda")
        ora.reduce_grads([case.grads(s, 0)])

    grads_in(0)
    opt.all_reduce_grads()
    ora.clip_grad_norm(case.max_norm, norm=opt.clip_grad_norm(case.max_norm))
    opt.step()
    ora.step()
    grads_in(1)  # a count edited between clip_grad_norm and step
    opt.all_reduce_grads()
    n = opt.clip_grad_norm(case.max_norm)
    opt.param_steps[3] = opt.param_steps[3] + 5
    ora.state[0].param_steps[3] += 5
    ora.clip_grad_norm(case.max_norm, norm=n)
    opt.step()
    ora.step()
    grads_in(2)  # clip_grad_norm, then the caller skips the step
    opt.all_reduce_grads()
    opt.clip_grad_norm(case.max_norm)
    grads_in(1)
    opt.all_reduce_grads()
    ora.clip_grad_norm(case.max_norm, norm=opt.clip_grad_norm(case.max_norm))
    opt.step()
    ora.step()
    torch.cuda.synchronize()
    for i in range(len(case.shapes)):
        master, m, v, steps = ora.tensor_state(i)
        assert opt.param_steps[i] == steps
        assert_bits_equal(to_numpy(opt.master[i], 0), master, f"master[{i}]")
        assert_bits_equal(to_numpy(opt.exp_avg[i], 0), m, f"exp_avg[{i}]")
        assert_bits_equal(to_numpy(opt.exp_avg_sq[i], 0), v, f"exp_avg_sq[{i}]")
        assert_bits_equal(to_numpy(params[i].data, case.dtype), ora.params[i], f"param[{i}]")


def _backward_into(params, grads, case, parts=1):
    """Gradients produced by autograd: ``parts`` backward passes of sum(p * g / parts) (exact in
    binary floating point), so each parameter's gradient equals g."""
    import torch
    half = [None if g is None else to_torch(g, case.dtype, p.shape, "cuda") * (1.0 / parts)
            for p, g in zip(params, grads)]
    for _ in range(parts):
        terms = [(p * h).sum() for p, h in zip(params, half) if h is not None]
        if terms:
            torch.autograd.backward(terms)


def test_landing_at_world_one_takes_the_norm_as_gradients_land():
    """land_grads=True at world size 1: the square sums are taken while backward runs and
    clip_grad_norm only adds them; norms and every state bit equal the oracle replaying them, and
    a gradient landed twice (two backward passes) or changed in place after landing falls back to
    the full pass with the same results."""
    import torch
    case = next(c for c in CASES if c.name == "bf16_clip")
    params, opt = build(case, land_grads=True)
    ref_params, ref = build(case)
    norms = []
    for s in range(case.steps):
        grads = case.grads(s, 0)
        for ps, o in ((params, opt), (ref_params, ref)):
            o.zero_grad(set_to_none=True)
            _backward_into(ps, grads, case, parts=2 if (s == 1 and o is opt) else 1)
            if s == 2 and o is opt:
                params[0].grad.mul_(1.0)  # in place after landing: its version moves
            o.all_reduce_grads()
            n = o.clip_grad_norm(case.max_norm)
            if o is opt:
                norms.append(n)
            else:
                assert abs(n - norms[-1]) <= 1e-6 * n, (s, n, norms[-1])
            o.step()
    torch.cuda.synchronize()
    assert opt.land_norm_steps == 1  # step 0 landed; step 1 landed twice, step 2 changed: full passes
    ora, _ = oracle_replay(case, Z.FORM_TORCH_CUDA, norms=norms)
    for i in range(len(case.shapes)):
        master, m, v, _ = ora.tensor_state(i)
        assert_bits_equal(to_numpy(opt.master[i], 0), master, f"master[{i}]")
        assert_bits_equal(to_numpy(opt.exp_avg[i], 0), m, f"exp_avg[{i}]")
        assert_bits_equal(to_numpy(opt.exp_avg_sq[i], 0), v, f"exp_avg_sq[{i}]")
        assert_bits_equal(to_numpy(params[i].data, case.dtype), ora.params[i], f"param[{i}]")
    opt.close()
