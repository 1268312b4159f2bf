"""Replica gradient all-reduce + clip + AdamW: the fused NVLink kernel against NCCL.

    torchrun --nproc-per-node D --master-addr 127.0.0.1 -m revpp.parallel.bench_allreduce --params 168000000

Every rank holds the flat fp32 buffers of one pipeline stage of one replica (n parameters:
fp32 weights, gradients, Adam moments, bf16 shadow weights).  Two ways of finishing a
step are timed with CUDA events between a barrier + synchronize on both sides (maximum
over ranks):

  fused - ``FusedP2PReducer.reduce_and_update``: one cooperative kernel per GPU that reads
          the peers' gradient shards over NVLink, averages them, exchanges the clip norm,
          applies AdamW to its shard and stores the new parameters into every replica;
  nccl  - NCCL all-reduce of the gradient, 1/D scale, squared-norm pass, fused AdamW kernel.

Roofline of the fused kernel (per GPU, per direction of its NVLink port): the peers' shards
of the gradient come in and this shard's parameters (fp32 + bf16) go out to D-1 peers,
while the peers do the same with this GPU's buffers: 10 n (D-1)/D bytes each way.  Local
HBM traffic is about 14 n + 28 n / D bytes.  The target time is the slower of the two at
the measured link (770 GB/s per direction) and copy (6534 GB/s) bandwidths.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
from types import SimpleNamespace

import torch
import torch.distributed as dist

LINK_GBS = 770.0
HBM_GBS = 6534.5


class _Flat:
    """The fields of FlatParams the reducers and the optimizer use, without a module."""

    def __init__(self, n: int, device: torch.device):
        self.numel = n
        self.device = device
        self.data = torch.randn(n, device=device) * 0.02
        self.grad = torch.zeros(n, device=device)
        self.shadow = self.data.to(torch.bfloat16)
        self.exp_avg = torch.zeros(n, device=device)
        self.exp_avg_sq = torch.zeros(n, device=device)
        self.step = 0


def _time(fn, warmup: int, iters: int, dev) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier(device_ids=[dev.index])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    dist.barrier(device_ids=[dev.index])
    t = torch.tensor([e0.elapsed_time(e1) / iters], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--params", type=int, default=168_000_000, help="parameters per stage (rounded to a multiple of 4 x D)")
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iters", type=int, default=10)
    a = p.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    D = dist.get_world_size()
    n = (a.params + 4 * D - 1) // (4 * D) * (4 * D)

    from revpp.optim import FlatAdamW
    from revpp.ops import ext
    from revpp.parallel.allreduce import NcclReducer
    from revpp.parallel.fused_allreduce import FusedP2PReducer

    C = ext()
    flat = _Flat(n, dev)
    opt = FlatAdamW(flat, lr=1e-5, eps=1e-6, weight_decay=0.01, max_grad_norm=1.0)
    trainer = SimpleNamespace(D=D, flat=flat, cfg=SimpleNamespace(global_clip=False), device=dev)
    group = dist.group.WORLD
    fused = FusedP2PReducer(trainer, group)
    nccl = NcclReducer(group, D)

    def run_fused():
        fused.reduce_and_update(opt)

    def run_nccl():
        nccl.reduce(flat.grad)
        opt.step(opt.grad_sumsq())

    flat.grad.normal_()
    t_fused = _time(run_fused, a.warmup, a.iters, dev)
    status = C.status_read_and_clear()
    t_nccl = _time(run_nccl, a.warmup, a.iters, dev)
    link_bytes = 10.0 * n * (D - 1) / D
    hbm_bytes = 14.0 * n + 28.0 * n / D
    roof_ms = max(link_bytes / (LINK_GBS * 1e6), hbm_bytes / (HBM_GBS * 1e6))
    rec = {"op": "replica_allreduce_adamw", "replicas": D, "n": n, "fused_ms": t_fused, "nccl_ms": t_nccl,
           "speedup_vs_nccl": t_nccl / t_fused, "link_bytes_per_direction": link_bytes, "hbm_bytes": hbm_bytes,
           "roofline_ms": roof_ms, "fused_fraction_of_roofline": roof_ms / t_fused,
           "link_gbs_per_direction_achieved": link_bytes / (t_fused * 1e6), "status": status}
    fused.close()
    if dist.get_rank() == 0:
        print(json.dumps(rec), flush=True)
    dist.barrier(device_ids=[dev.index])
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
