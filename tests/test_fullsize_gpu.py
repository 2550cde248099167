"""Full-size parity on the Qwen3-8B-shaped parameter set (8.19 G bf16 parameters, 399
tensors, fp32 state pre-loaded at step 100; 131 GB on one B200), one clipped step through
the public API.  The oracle cannot replay 8 G elements in seconds, so the check uses
properties that do not depend on size:

* the norm equals sqrt(float32(sum of float64(g)**2)) taken independently on the GPU in
  fp64, to 1e-6;
* 100,000 elements drawn at random across all tensors, with their pre-step gradient /
  master / m / v copied to the host, updated by the oracle (torch-CUDA form, same clip
  factor, same step count) equal the GPU results bit for bit;
* every parameter equals round-to-nearest-even of its new master, on every element.
"""
import math

import numpy as np
import pytest

from helpers import Z

pytestmark = pytest.mark.gpu

SAMPLES = 100_000


def test_qwen3_8b_one_clipped_step():
    import torch

    from hybridagent_b200 import ZeroOneAdamW, workloads

    torch.cuda.empty_cache()
    free, _ = torch.cuda.mem_get_info()
    shapes = workloads.qwen3_8b()
    numels = [math.prod(s) for s in shapes]
    n_total = sum(numels)
    if free < n_total * 16.5:
        pytest.skip(f"needs {n_total * 16.5 / 1e9:.0f} GB free on the device, {free / 1e9:.0f} GB free")
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11)
    params = [torch.nn.Parameter((torch.randn(s, device=dev, generator=g) * 0.02).to(torch.bfloat16)) for s in shapes]
    opt = ZeroOneAdamW([{"params": params, "lr": 1e-6}], rank=0, world_size=1, weight_decay=0.01)
    for i in range(len(params)):
        opt.exp_avg[i].normal_(0, 1e-5, generator=g)
        opt.exp_avg_sq[i].normal_(0, 1e-8, generator=g).abs_()
        opt.param_steps[i] = 100
    for p in params:
        p.grad = (torch.randn(p.shape, device=dev, generator=g) * 1e-4).to(torch.bfloat16)

    # host copies of the sampled elements' inputs
    rng = np.random.default_rng(5)
    cum = np.cumsum([0] + numels)
    flat = np.sort(rng.choice(n_total, size=SAMPLES, replace=False))
    tid = np.searchsorted(cum, flat, side="right") - 1
    pre = []
    for i in np.unique(tid):
        idx = torch.from_numpy(flat[tid == i] - cum[i]).to(dev)
        pre.append((int(i), idx,
                    params[i].grad.reshape(-1)[idx].view(torch.int16).cpu().numpy().view(np.uint16),
                    opt.master[i].reshape(-1)[idx].cpu().numpy(), opt.exp_avg[i].reshape(-1)[idx].cpu().numpy(),
                    opt.exp_avg_sq[i].reshape(-1)[idx].cpu().numpy()))
    exact = sum(float(p.grad.double().square().sum()) for p in params)

    opt.all_reduce_grads()
    norm = opt.clip_grad_norm(1.0)
    opt.step()
    torch.cuda.synchronize()

    want = float(np.sqrt(np.float32(exact)))
    assert abs(norm - want) <= 1e-6 * want, (norm, want)
    scale = Z.clip_scale_for(norm, 1.0)
    assert scale is not None  # ~N(0, 1e-4) over 8.19 G elements: norm ~ 9
    for i, idx, grad, master, m, v in pre:
        param = np.zeros(len(grad), np.uint16)
        Z.adamw_tensor(Z.FORM_TORCH_CUDA, grad, Z.BF16, master, m, v, param, Z.BF16, lr=1e-6, beta1=0.9,
                       beta2=0.999, eps=1e-8, weight_decay=0.01, step=101, clip_scale=scale)
        got_master = opt.master[i].reshape(-1)[idx].cpu().numpy()
        assert np.array_equal(got_master.view(np.uint32), master.view(np.uint32)), f"master of tensor {i}"
        assert np.array_equal(opt.exp_avg[i].reshape(-1)[idx].cpu().numpy().view(np.uint32), m.view(np.uint32))
        assert np.array_equal(opt.exp_avg_sq[i].reshape(-1)[idx].cpu().numpy().view(np.uint32), v.view(np.uint32))
        got_param = params[i].data.reshape(-1)[idx].view(torch.int16).cpu().numpy().view(np.uint16)
        assert np.array_equal(got_param, param), f"param of tensor {i}"
    for i, p in enumerate(params):
        assert torch.equal(p.data, opt.master[i].to(torch.bfloat16)), f"param {i} is not RNE(master)"
        assert opt.param_steps[i] == 101
    del opt, params, pre
    torch.cuda.empty_cache()
