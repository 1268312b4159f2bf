"""Fused replica gradient all-reduce + clip + AdamW over NVLink peer memory (PP x DP).

At construction every replica of a stage exports CUDA IPC handles of its flat fp32
parameters, fp32 gradients, bf16 shadow weights and a zeroed flag page, gathers the
peers' handles over the data-parallel process group and maps them.  Each step then runs
one cooperative kernel per GPU (``revpp._C.dp_reduce_adamw``, csrc/comm.cu): peers' gradient
shards are read with plain loads, averaged, the clip norm is exchanged through the flag
pages, AdamW updates this rank's shard and the updated parameters are stored into every
replica.  All waits in the kernel are bounded and report ``kStatusFlagTimeout``.

torch's CUDA storage sharing (``_share_cuda_`` / ``_new_shared_cuda``) is used only to
export and open the IPC handles; the data movement is the kernel's.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist


def _export(t: torch.Tensor):
    st = t.untyped_storage()
    meta = st._share_cuda_()
    elem_off = t.storage_offset() * t.element_size()
    return meta, elem_off, t.numel(), str(t.dtype)


def _open(meta, elem_off):
    st = torch.UntypedStorage._new_shared_cuda(*meta)
    return st, st.data_ptr() + elem_off


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
        self.flags = torch.zeros(128, dtype=torch.int32, device=dev)
        self.scratch = torch.zeros(2, dtype=torch.float32, device=dev)
        torch.cuda.synchronize(dev)
        mine = {
            "grad": _export(flat.grad),
            "param": _export(flat.data),
            "shadow": _export(flat.shadow) if flat.shadow is not None else None,
            "flags": _export(self.flags),
            "pid": os.getpid(),
        }
        allh = [None] * self.D
        dist.all_gather_object(allh, mine, group=group)
        self._keep = []  # opened storages stay alive for the mappings' lifetime
        self.ptrs = {"grad": [], "param": [], "shadow": [], "flags": []}
        own = {"grad": flat.grad, "param": flat.data, "shadow": flat.shadow, "flags": self.flags}
        for d, h in enumerate(allh):
            for key in ("grad", "param", "shadow", "flags"):
                if key == "shadow" and h["shadow"] is None:
                    continue
                if d == self.rank_in_group:
                    self.ptrs[key].append(own[key].data_ptr())
                else:
                    meta, off, _, _ = h[key]
                    st, ptr = _open(meta, off)
                    self._keep.append(st)
                    self.ptrs[key].append(ptr)
        if flat.shadow is None:
            self.ptrs["shadow"] = []
        # every mapped pointer must be device memory before a kernel touches it
        for key, lst in self.ptrs.items():
            for d, ptr in enumerate(lst):
                kind, _ = self.C.pointer_info(int(ptr))
                if kind != 2:  # cudaMemoryTypeDevice
                    raise RuntimeError(f"replica {d} {key} mapping is not device memory (type {kind})")
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
