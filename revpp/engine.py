"""Assembly and training loop.

``Trainer`` builds one rank's share of the job - its stage module (embedding / blocks /
head), the flat parameter buffers, the math (sm_100a kernels or PyTorch), the stage
runtime (reversible / standard / checkpoint / inverse), the pipeline channels and
executor, and the optimizer - and exposes ``train_step(batch)`` / ``eval_step(batch)``,
the public per-step API (what the reference spreads over Experiment._build_model_and_engine
and Engine._step_pp_{first,middle,last}, BERT/experiment/base.py:101-317,
BERT/src/engine.py:160-323).

Parallel layouts (P pipeline stages x D replicas, rank = replica * P + stage):
  --par-mode none      P = 1, D = 1
  --par-mode ddp       P = 1, D = world: gradients averaged over replicas
  --par-mode fsdp      P = 1, D = world: gradients reduce-scattered, each rank updates its
                       shard of the flat buffers, parameters all-gathered (ZeRO-2 style)
  --par-mode pp        P = world / dp, D = --dp
The reversible stages run their custom backward under every layout (the reference's
DDP/FSDP + reversible path produced no body gradients, reversible_stage_with_pareprop.py:561-575).

``Engine`` is the epoch loop with the reference's hooks (on_batch_start/end,
on_epoch_start/end) and metric tracking.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass, field
from typing import Callable, List, Optional

import torch
import torch.distributed as dist

from revpp.config import GlobalConfig, ParMode
from revpp.data import LoaderBundle
from revpp.metrics import MetricTracker
from revpp.models.blockmath import make_math
from revpp.models.encoder import build_stage_module, make_embed_head, stage_kind
from revpp.models.params import FlatParams
from revpp.optim import FlatAdamW, StepLR
from revpp.parallel.p2p import PipeComms, TensorSpec
from revpp.parallel.schedule import PipelineExecutor
from revpp.parallel.stage import STAGE_TYPES
from revpp.utils.env import EnvContext
from revpp.utils.profiling import annotate


class DeviceWaitError(RuntimeError):
    """A kernel's bounded wait ran out of time (recorded in the device status word)."""


def layout(cfg: GlobalConfig, world: int):
    if cfg.par_mode == ParMode.PP:
        return world // cfg.dp, cfg.dp
    if cfg.par_mode in (ParMode.DDP, ParMode.FSDP):
        return 1, world
    return 1, 1


def runtime_kind(cfg: GlobalConfig) -> str:
    if cfg.reversible:
        return "inverse" if cfg.inverse else "reversible"
    return "checkpoint" if cfg.checkpointing else "standard"


class Trainer:
    def __init__(self, cfg: GlobalConfig, env: EnvContext, eval_actv_err: bool = False):
        self.cfg = cfg
        self.env = env
        world = env.world_size
        self.P, self.D = layout(cfg, world)
        self.rank = env.rank
        self.stage_index = self.rank % self.P
        self.replica = self.rank // self.P
        self.device = env.device
        if cfg.num_microbatches < 1 or cfg.batch_size % self.D != 0:
            raise ValueError("batch_size must be divisible by the number of replicas")
        self.local_batch = cfg.batch_size // self.D
        if self.local_batch % cfg.num_microbatches != 0:
            raise ValueError("local batch must be divisible by num_microbatches")
        self.mbs = self.local_batch // cfg.num_microbatches
        # ---- model
        self.module = build_stage_module(cfg, self.stage_index, self.P, stage_kind(cfg))
        self.module.to(self.device)
        lowp = cfg.autocast_dtype == torch.bfloat16 and self.device.type == "cuda"
        self.flat = FlatParams(self.module, self.device, want_shadow=lowp)
        self.math = make_math(self.flat, cfg.autocast_dtype, cfg.num_attention_heads, self.device)
        self.uses_kernels = self.device.type == "cuda"
        self.eh = make_embed_head(self.module, self.flat, cfg.autocast_dtype, self.device)
        kind = runtime_kind(cfg)
        self.stage = STAGE_TYPES[kind](self.module, self.math, self.eh, self.mbs, cfg.num_microbatches, self.device,
                                       pareprop=cfg.is_pareprop, eval_actv_err=eval_actv_err)
        # ---- communication (collective construction: every rank, same order)
        self.comms: Optional[PipeComms] = None
        self.dp_group = None
        self.pp_group = None
        if dist.is_initialized():
            label_spec = TensorSpec((self.local_batch,), torch.int64)
            # messages into this stage: the previous stage's outputs, and the next stage's
            # backward message for this receiver
            self.comms = PipeComms(self.rank, world, self.P, self.D, self.device, self.stage.fwd_specs(),
                                   self.stage.bwd_specs(self.stage_index), label_spec)
            from revpp.parallel.p2p import _warm_group

            if self.D > 1:
                for s in range(self.P):
                    ranks = [d * self.P + s for d in range(self.D)]
                    g = dist.new_group(ranks)
                    _warm_group(g, ranks, self.device)
                    if s == self.stage_index:
                        self.dp_group = g
            if self.P > 1:
                self.pp_group = self.comms.group
        if self.P > 1 and self.device.type == "cuda":
            from revpp import ops

            if ops.available():
                ops.set_sm_reserve(4)  # room for the NCCL kernels that run next to the GEMMs
        self.executor = PipelineExecutor(self.stage, self.comms, cfg.num_microbatches, cfg.schedule)
        self.opt = FlatAdamW(self.flat, cfg.lr, eps=cfg.adam_eps, weight_decay=cfg.weight_decay,
                             max_grad_norm=cfg.max_grad_norm)
        self.lr_sched = StepLR(self.opt, 1, cfg.gamma)
        self.dp_reducer = None
        if self.D > 1:
            from revpp.parallel.allreduce import make_reducer

            # replicas start from the first replica's weights (DistributedDataParallel does the
            # same broadcast when it wraps the module)
            src = self.stage_index  # replica 0 of this stage
            dist.broadcast(self.flat.data, src=src, group=self.dp_group)
            self.flat.refresh_shadow()
            self.dp_reducer = make_reducer(self, cfg)
        self.step_count = 0

    # ------------------------------------------------------------------ helpers
    @property
    def is_first(self) -> bool:
        return self.stage.is_first

    @property
    def is_last(self) -> bool:
        return self.stage.is_last

    def split_inputs(self, batch: dict):
        """Device micro-batch inputs of the first stage.  BERT passes the attention mask as
        the token-type ids, as the reference engine does (engine.py:180 -> bert_stages.py:188)."""
        n = self.cfg.num_microbatches
        if self.cfg.model == "bert":
            ids = batch["input_ids"].to(self.device, non_blocking=True)
            tt = batch.get("token_type_ids", batch["attention_mask"]).to(self.device, non_blocking=True)
            return list(zip(torch.chunk(ids, n), torch.chunk(tt, n)))
        img = batch["images"].to(self.device, non_blocking=True)
        return [(x,) for x in torch.chunk(img, n)]

    # ------------------------------------------------------------------ steps
    def train_step(self, batch: Optional[dict]) -> Optional[torch.Tensor]:
        """One optimizer step on one global batch.  ``batch`` is required on first stages
        (host tensors, ideally pinned); returns the mean micro-batch loss (a device tensor)
        on last stages, None elsewhere."""
        inputs = labels = None
        if self.is_first:
            with annotate("## dataload ##"):
                inputs = self.split_inputs(batch)
                labels = batch["labels"].to(self.device, non_blocking=True)
        elif self.is_last and self.P == 1:
            labels = batch["labels"].to(self.device, non_blocking=True)
        with annotate("## pipeline_step ##"):
            losses = self.executor.step(inputs, labels, train=True)
        self.finish_step()
        self.step_count += 1
        if self.is_last:
            return torch.stack(losses).mean()
        return None

    def finish_step(self) -> None:
        """Replica gradient reduction, clipping and the optimizer update, then a check of the
        device status word."""
        self._update()
        self.check_device_status()

    def check_device_status(self, sync: bool = False) -> None:
        """Raise if a bounded wait inside one of the extension's kernels gave up (its output
        is then incomplete: an mbarrier wait in a tensor-core kernel, or a peer flag in the
        fused replica all-reduce).  The word lives in mapped host memory, so the read costs
        no device synchronisation; a failure in a kernel still running is seen by a later
        check (``sync=True`` waits for the device first)."""
        if not self.uses_kernels:
            return
        from revpp import ops

        if sync:
            torch.cuda.synchronize(self.device)
        st = ops.check_status(clear=False)
        if st:
            raise DeviceWaitError(f"rank {self.rank}: device status word {st:#x} after step {self.step_count} "
                                  "(a bounded wait inside a kernel gave up; results of this step are incomplete)")

    def _update(self) -> None:
        if self.dp_reducer is not None:
            with annotate("## dp_allreduce ##"):
                if self.dp_reducer.fused_update:
                    self.dp_reducer.reduce_and_update(self.opt)
                    return
                self.dp_reducer.reduce(self.flat.grad)
        with annotate("## clip_grad ##"):
            sumsq = self.opt.grad_sumsq()
            if self.cfg.global_clip and self.pp_group is not None:
                dist.all_reduce(sumsq, group=self.pp_group)
        with annotate("## optimize ##"):
            if self.dp_reducer is not None and self.dp_reducer.sharded:
                self.dp_reducer.sharded_step(self.opt, sumsq)
            else:
                self.opt.step(sumsq)

    def eval_step(self, batch: Optional[dict]):
        inputs = labels = None
        if self.is_first:
            inputs = self.split_inputs(batch)
            labels = batch["labels"].to(self.device, non_blocking=True)
        elif self.is_last and self.P == 1:
            labels = batch["labels"].to(self.device, non_blocking=True)
        with torch.no_grad():
            losses = self.executor.step(inputs, labels, train=False)
        if self.is_last:
            logits = torch.cat(self.stage.logits) if self.stage.logits else None
            lab = torch.cat(self.stage.labels) if self.stage.labels is not None else None
            loss = torch.stack(losses).mean() if losses else None
            return loss, logits, lab
        return None

    def last_labels(self) -> Optional[torch.Tensor]:
        return torch.cat(self.stage.labels) if self.stage.labels is not None else None

    def last_logits(self) -> Optional[torch.Tensor]:
        return torch.cat(self.stage.logits) if self.stage.logits else None

    def close(self) -> None:
        if self.comms is not None:
            self.comms.drain()
        if self.dp_reducer is not None and hasattr(self.dp_reducer, "close"):
            self.dp_reducer.close()
        self.check_device_status(sync=True)


@dataclass
class Engine:
    trainer: Trainer
    loaders: LoaderBundle
    tracker: MetricTracker
    on_batch_start: List[Callable] = field(default_factory=list)
    on_batch_end: List[Callable] = field(default_factory=list)
    on_epoch_start: List[Callable] = field(default_factory=list)
    on_epoch_end: List[Callable] = field(default_factory=list)
    log_every: int = 64

    def _run(self, hooks, *a):
        for h in hooks:
            h(*a)

    def step(self, epoch: int, is_train: bool, batch_limit: Optional[int] = None) -> dict:
        t = self.trainer
        self._run(self.on_epoch_start, epoch, is_train)
        self.tracker.reset("train" if is_train else "valid", epoch)
        n = self.loaders.num_batches_train if is_train else self.loaders.num_batches_val
        loader = (self.loaders.train_loader if is_train else self.loaders.val_loader) if t.is_first else None
        it = iter(loader) if loader is not None else None
        if loader is not None and hasattr(loader, "set_epoch"):
            loader.set_epoch(epoch)
        for bi in range(n):
            if batch_limit is not None and bi >= batch_limit:
                break
            self._run(self.on_batch_start, bi, is_train)
            batch = next(it) if it is not None else None
            if batch is None and t.is_last and t.P == 1:
                raise RuntimeError("single-stage run needs a batch")
            if is_train:
                loss = t.train_step(batch)
                if t.is_last:
                    self.tracker.update(loss, t.last_logits(), t.last_labels())
            else:
                r = t.eval_step(batch)
                if t.is_last and r is not None:
                    self.tracker.update(r[0], r[1], r[2])
            if t.is_last and bi % self.log_every == 0 and is_train:
                lv = float(loss)
                if math.isnan(lv) or math.isinf(lv):
                    if self.tracker.logger:
                        self.tracker.logger.error("loss is %s at batch %d", lv, bi)
                self.tracker.log_batch(bi, n, lv)
            self._run(self.on_batch_end, bi, is_train)
        self._run(self.on_epoch_end, epoch, is_train)
        if t.pp_group is None and t.dp_group is None:
            pass
        summary = self.tracker.summary() if t.is_last else {}
        if t.is_last:
            self.tracker.log_epoch()
        if is_train:
            t.lr_sched.step()
        return summary
