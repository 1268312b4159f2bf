"""Gradient reduction across pipeline replicas (PP x DP) and data-parallel modes.

* ``NcclReducer``     - one NCCL all-reduce of the stage's flat fp32 gradient, then a
                        1/D scale (the baseline).
* ``ShardedReducer``  - ``--par-mode fsdp`` (ZeRO-2): reduce-scatter of the flat gradient,
                        Adam moments and AdamW of this rank's shard only, all-gather of the
                        updated parameters.
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
    """``--par-mode fsdp`` as ZeRO-2: gradients are reduce-scattered, each replica keeps the
    Adam moments of its 1/D shard only (the full-size moment buffers are released) and
    updates that shard, and the updated parameters are all-gathered.  Parameters stay
    whole on every rank: for these models they are a few GB at most on a 180 GB device,
    while resharding them after every forward (the reference's ``fully_shard(
    reshard_after_forward=True)``, BERT/experiment/base.py:252-254) would add an all-gather
    per block and micro-batch, and another for each block the reversible backward
    recomputes."""

    fused_update = False
    sharded = True

    def __init__(self, group, replicas: int, rank_in_group: int, numel: int, flat=None):
        self.group = group
        self.D = replicas
        self.r = rank_in_group
        assert numel % replicas == 0
        self.shard = numel // replicas
        if flat is not None:
            dev = flat.device
            flat.exp_avg = torch.zeros(self.shard, dtype=torch.float32, device=dev)
            flat.exp_avg_sq = torch.zeros(self.shard, dtype=torch.float32, device=dev)

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
        full = (f.data, f.grad, f.shadow)
        if f.exp_avg.numel() != n:  # moments still full-size (constructed without the flat buffers)
            f.exp_avg = f.exp_avg.narrow(0, lo, n).clone()
            f.exp_avg_sq = f.exp_avg_sq.narrow(0, lo, n).clone()
        try:
            f.data, f.grad = (t.narrow(0, lo, n) for t in full[:2])
            if f.shadow is not None:
                f.shadow = full[2].narrow(0, lo, n)
            opt.step(local)
        finally:
            f.data, f.grad, f.shadow = full
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
        return ShardedReducer(group, D, trainer.replica, trainer.flat.numel, trainer.flat)
    use_fused = os.environ.get("REVPP_FUSED_ALLREDUCE", "1") != "0"
    if use_fused and trainer.device.type == "cuda":
        try:
            from .fused_allreduce import FusedP2PReducer

            return FusedP2PReducer(trainer, group)
        except (ImportError, RuntimeError) as e:  # extension without the kernel, or no P2P access
            if trainer.env.main_logger:
                trainer.env.main_logger.warning("fused replica all-reduce unavailable (%s); using NCCL", e)
    return NcclReducer(group, D)
