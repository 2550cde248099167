"""TEST INFRASTRUCTURE ONLY -- a checker, never the product.

The reference's per-tensor update and clip written as the same torch eager op sequence
(hybrid_rl/optimizer.py:151, 159, 176-191), runnable on any torch device.  On CPU it
reproduces the golden vectors of the reference bit for bit (tests/test_torch_ops_cpu.py);
on a CUDA device it yields what the reference computes there, which pins the oracle's
torch-CUDA rounding form (tests/test_torch_cuda_forms.py).  bench.py's reference arm
times this sequence on the host's CPU cores as the reference CPU baseline.
"""
from __future__ import annotations

import torch


@torch.no_grad()
def clip_(grads: list[torch.Tensor | None], max_norm: float, total: torch.Tensor | None = None) -> float:
    """optimizer.py:148-160 for one process: fp32 sum of squares, sqrt, in-place clip."""
    if total is None:
        total = torch.zeros((), device=next(g for g in grads if g is not None).device, dtype=torch.float32)
        for g in grads:
            if g is not None:
                total.add_(g.detach().float().square().sum())
    norm = float(total.sqrt())
    if max_norm > 0 and norm > max_norm:
        scale = float(max_norm) / (norm + 1e-6)
        for g in grads:
            if g is not None:
                g.mul_(scale)
    return norm


@torch.no_grad()
def adamw_tensor_(param: torch.Tensor, grad: torch.Tensor, master: torch.Tensor, exp_avg: torch.Tensor,
                  exp_avg_sq: torch.Tensor, *, lr: float, betas: tuple[float, float], eps: float,
                  weight_decay: float, step: int, master_is_parameter: bool) -> None:
    """optimizer.py:176-191 for one owned tensor whose step counter is already ``step``."""
    beta1, beta2 = betas
    gradient = grad.detach().float()
    correction1 = 1.0 - beta1 ** step
    correction2 = 1.0 - beta2 ** step
    if weight_decay:
        master.mul_(1.0 - lr * weight_decay)
    exp_avg.mul_(beta1).add_(gradient, alpha=1.0 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(gradient, gradient, value=1.0 - beta2)
    denominator = (exp_avg_sq / correction2).sqrt().add_(eps)
    master.addcdiv_(exp_avg / correction1, denominator, value=-lr)
    if not master_is_parameter:
        param.copy_(master.to(param.dtype))


class TorchZeroOneW1:
    """The reference optimizer's world-size-1 path (no collectives) over torch tensors on
    any device, used as the timed CPU baseline and as a CUDA-side checker."""

    def __init__(self, params: list[torch.Tensor], lr: float, *, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0):
        self.params = params
        self.lr, self.betas, self.eps, self.weight_decay = float(lr), tuple(betas), float(eps), float(weight_decay)
        self.master = [p if p.dtype == torch.float32 else p.detach().float().clone() for p in params]
        self.exp_avg = [torch.zeros_like(m) for m in self.master]
        self.exp_avg_sq = [torch.zeros_like(m) for m in self.master]
        self.steps = [0] * len(params)

    def step(self, grads: list[torch.Tensor | None], max_norm: float) -> float:
        norm = clip_(grads, max_norm)
        for i, g in enumerate(grads):
            if g is None:
                continue
            self.steps[i] += 1
            adamw_tensor_(self.params[i], g, self.master[i], self.exp_avg[i], self.exp_avg_sq[i], lr=self.lr,
                          betas=self.betas, eps=self.eps, weight_decay=self.weight_decay, step=self.steps[i],
                          master_is_parameter=self.params[i].dtype == torch.float32)
        return norm
