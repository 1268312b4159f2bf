"""Process / device / process-group setup (the reference's EnvContext, BERT/src/env.py:10-84).

One process per GPU, launched by torchrun (RANK / LOCAL_RANK / WORLD_SIZE / MASTER_*).
NCCL on CUDA, gloo on CPU (tests).  The process group gets a finite timeout so that a
rank that dies or hangs makes the others fail with an error instead of waiting forever.
The main logger lives on the last rank of the first pipeline, which sees the loss.
"""
from __future__ import annotations

import datetime
import logging
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from revpp.config import GlobalConfig, ParMode

from .logger import build_logger


@dataclass
class EnvContext:
    world_size: int
    rank: int
    local_rank: int
    device: torch.device
    proc_logger: logging.Logger
    node_logger: Optional[logging.Logger]
    main_logger: Optional[logging.Logger]
    pg: Optional[object]
    master_rank: int
    num_stages: int = 1
    replicas: int = 1

    @property
    def stage_index(self) -> int:
        return self.rank % self.num_stages

    @property
    def replica(self) -> int:
        return self.rank // self.num_stages

    def barrier(self) -> None:
        if dist.is_initialized():
            if self.device.type == "cuda":
                dist.barrier(device_ids=[self.device.index])
            else:
                dist.barrier()

    def close(self) -> None:
        if dist.is_initialized():
            try:
                self.barrier()
            finally:
                dist.destroy_process_group()


def pick_device(cfg: GlobalConfig, local_rank: int) -> torch.device:
    want = cfg.device
    if want == "cpu" or (want == "auto" and not torch.cuda.is_available()):
        return torch.device("cpu")
    if not torch.cuda.is_available():
        raise RuntimeError("--device cuda requested but no CUDA device is visible")
    torch.cuda.set_device(local_rank)
    return torch.device("cuda", local_rank)


def init_distributed(device: torch.device, timeout_s: float = 600.0) -> None:
    if dist.is_initialized():
        return
    backend = "nccl" if device.type == "cuda" else "gloo"
    kw = dict(backend=backend, init_method="env://", timeout=datetime.timedelta(seconds=timeout_s))
    if device.type == "cuda":
        kw["device_id"] = device
    dist.init_process_group(**kw)


def build_env(cfg: GlobalConfig, timeout_s: float = 600.0) -> EnvContext:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    device = pick_device(cfg, local_rank)
    if cfg.par_mode != ParMode.NONE or world > 1:
        init_distributed(device, timeout_s)
        world = dist.get_world_size()
        rank = dist.get_rank()
    replicas = cfg.dp if cfg.par_mode == ParMode.PP else 1
    if cfg.par_mode == ParMode.PP and world % replicas != 0:
        raise ValueError(f"world size {world} is not a multiple of --dp {replicas}")
    num_stages = world // replicas if cfg.par_mode == ParMode.PP else 1
    master_rank = num_stages - 1 if cfg.par_mode == ParMode.PP else 0
    log_dir = cfg.log_rdir / cfg.exp_id / cfg.env_id
    proc_logger = build_logger(f"proc{rank}", log_dir / f"proc_{rank}.log", console=False)
    node_logger = build_logger("node", log_dir / "node.log", console=False) if local_rank == 0 else None
    main_logger = build_logger("main", log_dir / "main.log", console=True) if rank == master_rank else None
    return EnvContext(world_size=world, rank=rank, local_rank=local_rank, device=device, proc_logger=proc_logger,
                      node_logger=node_logger, main_logger=main_logger,
                      pg=dist.group.WORLD if dist.is_initialized() else None, master_rank=master_rank,
                      num_stages=num_stages, replicas=replicas)
