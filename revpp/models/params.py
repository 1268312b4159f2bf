"""Flat parameter storage for one pipeline stage.

All parameters of a stage live in one fp32 buffer (master weights), with one fp32
gradient buffer, one bf16 shadow copy (the GEMM operands, refreshed by the fused
AdamW kernel) and the two Adam moment buffers.  Each parameter becomes a view into
these buffers, so

  * the optimizer, the gradient norm and the replica all-reduce are one pass over a
    contiguous buffer (no multi-tensor launch lists);
  * kernels accumulate weight gradients straight into ``grad_of(p)`` (fp32), including
    across micro-batches;
  * ``state_dict()`` / ``load_state_dict()`` of the module keep working (they copy
    through the views).

Each parameter starts on a 64-element boundary so every view is 256-byte aligned
(TMA and vector loads need 16 bytes).
"""
from __future__ import annotations

from typing import Dict, List

import torch
import torch.nn as nn

ALIGN = 64


class FlatParams:
    def __init__(self, module: nn.Module, device: torch.device | str, want_shadow: bool = True):
        device = torch.device(device)
        self.module = module
        self.params: List[nn.Parameter] = []
        self.names: List[str] = []
        seen = set()
        for name, p in module.named_parameters():
            if id(p) in seen:
                continue
            seen.add(id(p))
            self.params.append(p)
            self.names.append(name)
        self.offsets: List[int] = []
        off = 0
        for p in self.params:
            self.offsets.append(off)
            off += (p.numel() + ALIGN - 1) // ALIGN * ALIGN
        self.numel = max(off, ALIGN)
        self.device = device
        self.data = torch.zeros(self.numel, dtype=torch.float32, device=device)
        self.grad = torch.zeros(self.numel, dtype=torch.float32, device=device)
        self._index: Dict[int, int] = {}
        for i, (p, o) in enumerate(zip(self.params, self.offsets)):
            n = p.numel()
            self.data[o:o + n].copy_(p.detach().reshape(-1).to(device=device, dtype=torch.float32))
            p.data = self.data[o:o + n].view(p.shape)
            self._index[id(p)] = i
        self.shadow = torch.zeros(self.numel, dtype=torch.bfloat16, device=device) if want_shadow else None
        self.exp_avg = torch.zeros(self.numel, dtype=torch.float32, device=device)
        self.exp_avg_sq = torch.zeros(self.numel, dtype=torch.float32, device=device)
        self.step = 0
        self.refresh_shadow()

    # ------------------------------------------------------------------ views
    def _span(self, p: torch.Tensor):
        i = self._index[id(p)]
        o = self.offsets[i]
        return o, self.params[i].numel(), self.params[i].shape

    def grad_of(self, p: torch.Tensor) -> torch.Tensor:
        o, n, shape = self._span(p)
        return self.grad[o:o + n].view(shape)

    def shadow_of(self, p: torch.Tensor) -> torch.Tensor:
        assert self.shadow is not None
        o, n, shape = self._span(p)
        return self.shadow[o:o + n].view(shape)

    def refresh_shadow(self) -> None:
        if self.shadow is not None:
            self.shadow.copy_(self.data)

    def zero_grad(self) -> None:
        self.grad.zero_()

    def named_grads(self):
        for name, p in zip(self.names, self.params):
            yield name, self.grad_of(p)

    def state_dict(self) -> dict:
        return {"exp_avg": self.exp_avg.cpu(), "exp_avg_sq": self.exp_avg_sq.cpu(), "step": self.step,
                "names": list(self.names)}

    def load_state_dict(self, sd: dict) -> None:
        self.exp_avg.copy_(sd["exp_avg"].to(self.device))
        self.exp_avg_sq.copy_(sd["exp_avg_sq"].to(self.device))
        self.step = int(sd["step"])
