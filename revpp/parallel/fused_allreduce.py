"""Fused replica gradient all-reduce + clip + AdamW over NVLink peer memory (PP x DP).

At construction every replica of a stage exports CUDA IPC handles of its flat fp32
parameters, fp32 gradients, bf16 shadow weights and a zeroed flag page, gathers the
peers' handles over the data-parallel process group and maps them *for its own GPU*
(``revpp._C.ipc_open`` runs cudaIpcOpenMemHandle with this rank's device current and lazy
peer access).  Each step then runs one cooperative kernel per GPU
(``revpp._C.dp_reduce_adamw``, csrc/comm.cu): peers' gradient shards are read with plain
loads, averaged, the clip norm is exchanged through the flag pages, AdamW updates this
rank's shard and the updated parameters are stored into every replica.  All waits in the
kernel are bounded and report ``kStatusFlagTimeout``.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist


class FusedP2PReducer:
    fused_update = True
    sharded = False

    def __init__(self, trainer, group):
        from revpp.ops import ext

        self.C = ext()
        self.trainer = trainer
        self.group = group
        self.D = trainer.D
        self.rank_in_group = dist.get_rank(group)
        flat = trainer.flat
        if flat.numel % (4 * self.D) != 0:
            raise RuntimeError("flat buffer size must be a multiple of 4 x replicas")
        if trainer.cfg.global_clip:
            raise RuntimeError("global clipping across stages is not fused; using NCCL")
        dev = flat.device
        self.device = dev
        # a flag page of its own allocation (128 int32 words, padded to its own segment)
        self.flags = torch.zeros(1 << 18, dtype=torch.int32, device=dev)[:128]
        self.scratch = torch.zeros(2, dtype=torch.float32, device=dev)
        torch.cuda.synchronize(dev)
        own = {"grad": flat.grad, "param": flat.data, "shadow": flat.shadow, "flags": self.flags}
        mine = {k: (self.C.ipc_export(t) if t is not None else None) for k, t in own.items()}
        allh = [None] * self.D
        dist.all_gather_object(allh, mine, group=group)
        self._bases = {}  # handle bytes -> mapped base (each peer segment mapped once)
        self.ptrs = {"grad": [], "param": [], "shadow": [], "flags": []}
        with torch.cuda.device(dev):
            for d, h in enumerate(allh):
                for key in ("grad", "param", "shadow", "flags"):
                    if own[key] is None:
                        continue
                    if d == self.rank_in_group:
                        self.ptrs[key].append(own[key].data_ptr())
                        continue
                    handle, off = h[key]
                    if handle not in self._bases:
                        self._bases[handle] = self.C.ipc_open(handle)
                    self.ptrs[key].append(self._bases[handle] + int(off))
        if flat.shadow is None:
            self.ptrs["shadow"] = []
        self.epoch = 0
        self.timeout_s = float(os.environ.get("REVPP_P2P_TIMEOUT_S", "60"))

    def reduce_and_update(self, opt) -> None:
        f = opt.flat
        f.step += 1
        self.C.dp_reduce_adamw(self.ptrs["grad"], self.ptrs["param"], self.ptrs["shadow"], self.ptrs["flags"],
                               f.exp_avg, f.exp_avg_sq, self.scratch, f.numel, self.rank_in_group, self.epoch,
                               opt.lr, opt.beta1, opt.beta2, opt.eps, opt.weight_decay, f.step, opt.max_grad_norm,
                               self.timeout_s, True)
        self.epoch += 1

    def reduce(self, grad) -> None:  # pragma: no cover - the fused path never splits the update
        raise RuntimeError("FusedP2PReducer updates parameters itself; call reduce_and_update")

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        for base in self._bases.values():
            self.C.ipc_close(base)
        self._bases.clear()
