"""AdamW with gradient clipping over a stage's flat buffers, and the StepLR schedule.

Matches torch.optim.AdamW(lr, betas=(0.9, 0.999), eps=1e-6, weight_decay=0.01) preceded by
clip_grad_norm_(max_norm=1.0) (BERT/experiment/base.py:303-304, BERT/src/engine.py:56-67).
By default the norm is the stage's own (the reference clips each pipeline stage locally);
``global_clip`` all-reduces the squared norm over the pipeline first.

On CUDA the update is two kernels: a squared-norm reduction and one fused pass that
applies the clip coefficient (read on the device), the AdamW update, refreshes the bf16
shadow weights and zeroes the gradients.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist

from revpp.models.params import FlatParams


class FlatAdamW:
    def __init__(self, flat: FlatParams, lr: float, betas=(0.9, 0.999), eps: float = 1e-6,
                 weight_decay: float = 0.01, max_grad_norm: float = 1.0):
        self.flat = flat
        self.lr = lr
        self.beta1, self.beta2 = betas
        self.eps = eps
        self.weight_decay = weight_decay
        self.max_grad_norm = max_grad_norm
        self.kernels = flat.device.type == "cuda"
        if self.kernels:
            from revpp.ops import ext

            self._C = ext()
        self._sumsq = torch.zeros(1, dtype=torch.float32, device=flat.device)

    def grad_sumsq(self) -> torch.Tensor:
        """Squared L2 norm of the stage gradient, as a 1-element device tensor."""
        self._sumsq.zero_()
        if self.kernels:
            self._C.grad_sumsq(self.flat.grad, self._sumsq)
        else:
            self._sumsq.add_(self.flat.grad.double().pow(2).sum().float())
        return self._sumsq

    def step(self, sumsq: Optional[torch.Tensor] = None, zero_grad: bool = True) -> None:
        f = self.flat
        f.step += 1
        if self.max_grad_norm > 0 and sumsq is None:
            sumsq = self.grad_sumsq()
        if self.kernels:
            self._C.adamw_step(f.data, f.grad, f.exp_avg, f.exp_avg_sq, shadow=f.shadow, lr=self.lr,
                               beta1=self.beta1, beta2=self.beta2, eps=self.eps, wd=self.weight_decay, step=f.step,
                               max_norm=self.max_grad_norm, sumsq=sumsq if self.max_grad_norm > 0 else None,
                               zero_grad=zero_grad)
            return
        with torch.no_grad():
            g = f.grad
            if self.max_grad_norm > 0:
                norm = float(sumsq.sqrt())
                coef = min(1.0, self.max_grad_norm / (norm + 1e-6))
                g = g * coef
            f.data.mul_(1.0 - self.lr * self.weight_decay)
            f.exp_avg.lerp_(g, 1.0 - self.beta1)
            f.exp_avg_sq.mul_(self.beta2).addcmul_(g, g, value=1.0 - self.beta2)
            bc1 = 1.0 - self.beta1 ** f.step
            bc2 = 1.0 - self.beta2 ** f.step
            denom = (f.exp_avg_sq.sqrt() / math.sqrt(bc2)).add_(self.eps)
            f.data.addcdiv_(f.exp_avg, denom, value=-self.lr / bc1)
            f.refresh_shadow()
            if zero_grad:
                f.grad.zero_()

    def state_dict(self) -> dict:
        return {"lr": self.lr, **self.flat.state_dict()}

    def load_state_dict(self, sd: dict) -> None:
        self.lr = float(sd.get("lr", self.lr))
        self.flat.load_state_dict(sd)


class StepLR:
    """lr <- lr * gamma every ``step_size`` epochs (torch.optim.lr_scheduler.StepLR, step_size=1)."""

    def __init__(self, opt: FlatAdamW, step_size: int = 1, gamma: float = 1.0):
        self.opt = opt
        self.step_size = step_size
        self.gamma = gamma
        self.epoch = 0

    def step(self) -> None:
        self.epoch += 1
        if self.epoch % self.step_size == 0:
            self.opt.lr *= self.gamma


def allreduce_sumsq(sumsq: torch.Tensor, group=None) -> torch.Tensor:
    """Global gradient norm across pipeline stages (``--global-clip``)."""
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(sumsq, op=dist.ReduceOp.SUM, group=group)
    return sumsq
