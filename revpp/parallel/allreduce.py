"""Gradient reduction across pipeline replicas (PP x DP) and data-parallel modes.

* ``NcclReducer``     - one NCCL all-reduce of the stage's flat fp32 gradient, then a
                        1/D scale (the baseline).
* ``ShardedReducer``  - ``--par-mode fsdp``: reduce-scatter of the flat gradient, AdamW on
                        this rank's shard, all-gather of the updated parameters.
* ``FusedP2PReducer`` - the sm_100a kernel that reads the peer replicas' gradient buffers
                        over NVLink (CUDA IPC mappings), sums, scales, clips and applies
                        AdamW in one pass (``revpp.parallel.fused_allreduce``).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from revpp.config import GlobalConfig, ParMode


class NcclReducer:
    fused_update = False
    sharded = False

    def __init__(self, group, replicas: int):
        self.group = group
        self.D = replicas

    def reduce(self, grad: torch.Tensor) -> None:
        dist.all_reduce(grad, op=dist.ReduceOp.SUM, group=self.group)
        grad.mul_(1.0 / self.D)


class ShardedReducer:
    """ZeRO-2-style: each replica owns 1/D of the flat buffers for the optimizer update."""

    fused_update = False
    sharded = True

    def __init__(self, group, replicas: int, rank_in_group: int, numel: int):
        self.group = group
        self.D = replicas
        self.r = rank_in_group
        assert numel % replicas == 0
        self.shard = numel // replicas

    def reduce(self, grad: torch.Tensor) -> None:
        out = grad.narrow(0, self.r * self.shard, self.shard)
        tmp = torch.empty(self.shard, dtype=grad.dtype, device=grad.device)
        dist.reduce_scatter_tensor(tmp, grad, op=dist.ReduceOp.SUM, group=self.group)
        grad.zero_()
        out.copy_(tmp.mul_(1.0 / self.D))

    def sharded_step(self, opt, sumsq: torch.Tensor) -> None:
        # the squared norm of the full gradient: shards are disjoint, so sum over ranks
        local = opt.grad_sumsq()
        dist.all_reduce(local, group=self.group)
        f = opt.flat
        lo, n = self.r * self.shard, self.shard
        views = (f.data, f.grad, f.exp_avg, f.exp_avg_sq, f.shadow)
        full = tuple(views)
        try:
            f.data, f.grad, f.exp_avg, f.exp_avg_sq = (t.narrow(0, lo, n) for t in full[:4])
            if f.shadow is not None:
                f.shadow = full[4].narrow(0, lo, n)
            opt.step(local)
        finally:
            f.data, f.grad, f.exp_avg, f.exp_avg_sq, f.shadow = full
        gathered = torch.empty_like(f.data)
        dist.all_gather_into_tensor(gathered, f.data.narrow(0, lo, n).contiguous(), group=self.group)
        f.data.copy_(gathered)
        f.refresh_shadow()
        f.grad.zero_()


def make_reducer(trainer, cfg: GlobalConfig):
    D = trainer.D
    group = trainer.dp_group
    if cfg.par_mode == ParMode.FSDP:
        pad = (-trainer.flat.numel) % D
        if pad:
            raise ValueError("flat parameter size must be divisible by the replica count for fsdp mode")
        return ShardedReducer(group, D, trainer.replica, trainer.flat.numel)
    use_fused = os.environ.get("REVPP_FUSED_ALLREDUCE", "1") != "0"
    if use_fused and trainer.device.type == "cuda":
        try:
            from .fused_allreduce import FusedP2PReducer

            return FusedP2PReducer(trainer, group)
        except (ImportError, RuntimeError) as e:  # extension without the kernel, or no P2P access
            if trainer.env.main_logger:
                trainer.env.main_logger.warning("fused replica all-reduce unavailable (%s); using NCCL", e)
    return NcclReducer(group, D)
