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


class ChunkedStage(torch.nn.Module):
    """The model chunks of one rank under the interleaved schedule (state_dict keys
    ``chunks.<c>.<stage keys>``)."""

    def __init__(self, modules):
        super().__init__()
        self.chunks = torch.nn.ModuleList(modules)

    @property
    def kind(self) -> str:
        return self.chunks[0].kind


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
        # ---- model: v chunks per rank (v > 1 with the interleaved schedule); chunk c is
        # global stage c * P + stage_index of v * P
        self.v = cfg.virtual_stages if cfg.schedule == "interleaved" else 1
        if self.v > 1 and runtime_kind(cfg) == "inverse":
            raise ValueError("the interleaved schedule supports reversible, standard and checkpoint stages")
        G = self.P * self.v
        modules = [build_stage_module(cfg, c * self.P + self.stage_index, G, stage_kind(cfg)) for c in range(self.v)]
        self.module = modules[0] if self.v == 1 else ChunkedStage(modules)
        self.module.to(self.device)
        lowp = cfg.autocast_dtype == torch.bfloat16 and self.device.type == "cuda"
        self.flat = FlatParams(self.module, self.device, want_shadow=lowp)
        self.math = make_math(self.flat, cfg.autocast_dtype, cfg.num_attention_heads, self.device)
        self.uses_kernels = self.device.type == "cuda"
        kind = runtime_kind(cfg)
        self.stages = []
        for mm in modules:
            eh = make_embed_head(mm, self.flat, cfg.autocast_dtype, self.device)
            self.stages.append(STAGE_TYPES[kind](mm, self.math, eh, self.mbs, cfg.num_microbatches, self.device,
                                                 pareprop=cfg.is_pareprop, eval_actv_err=eval_actv_err))
        self.stage = self.stages[0]
        self.eh = self.stage.eh
        self.last_stage = self.stages[-1]
        # ---- communication (collective construction: every rank, same order)
        self.comms: Optional[PipeComms] = None
        self.channels = None
        self.dp_group = None
        self.pp_group = None
        self.p2p = "none"
        if dist.is_initialized():
            self.p2p = self._choose_p2p(cfg)
            if self.v > 1 and self.p2p != "copy":
                raise ValueError("the interleaved schedule runs over copy channels (--p2p copy, one node)")
            if self.p2p == "group":
                label_spec = TensorSpec((self.local_batch,), torch.int64)
                # messages into this stage: the previous stage's outputs, and the next stage's
                # backward message for this receiver
                self.comms = PipeComms(self.rank, world, self.P, self.D, self.device, self.stage.fwd_specs(),
                                       self.stage.bwd_specs(self.stage_index), label_spec)
                if self.P > 1:
                    self.pp_group = self.comms.group
            else:
                for d in range(self.D):
                    g = dist.new_group(list(range(d * self.P, (d + 1) * self.P)))
                    if d == self.replica:
                        self.pp_group = g
                if self.P > 1:
                    self.channels = self._build_channels(cfg, kind)
            from revpp.parallel.p2p import _warm_group

            if self.D > 1:
                for s in range(self.P):
                    ranks = [d * self.P + s for d in range(self.D)]
                    g = dist.new_group(ranks)
                    _warm_group(g, ranks, self.device)
                    if s == self.stage_index:
                        self.dp_group = g
        if self.P > 1 and self.device.type == "cuda" and self.p2p == "group":
            from revpp import ops

            if ops.available():
                ops.set_sm_reserve(4)  # room for the NCCL kernels that run next to the GEMMs
        if self.channels is not None:
            from revpp.parallel.schedule import ChannelExecutor

            names = self._channel_names()
            chans = {role: self.channels.get(name) for role, name in names.items()}
            self.executor = ChannelExecutor(self.stages, chans, cfg.num_microbatches, self.P, self.stage_index,
                                            cfg.schedule, global_rank=self.rank)
        else:
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

    # ------------------------------------------------------------------ p2p set-up
    def _choose_p2p(self, cfg: GlobalConfig) -> str:
        """"copy": copy-engine channels (every rank of the job on one node; shared memory on
        CPU); "group": NCCL / gloo point-to-point groups.  ``auto`` picks copy channels on one
        GPU node and groups otherwise (collective: every rank must agree)."""
        import socket

        want = cfg.p2p
        hosts = [None] * dist.get_world_size()
        dist.all_gather_object(hosts, socket.gethostname())
        one_node = len(set(hosts)) == 1
        if want == "auto":
            want = "copy" if (one_node and self.device.type == "cuda") else "group"
        if want == "copy" and not one_node:
            raise ValueError("--p2p copy needs every rank on one node")
        return want

    def _channel_names(self) -> dict:
        """This rank's channel roles -> channel names (see _build_channels)."""
        P, r, d = self.P, self.stage_index, self.replica
        names = {}
        if r < P - 1 or self.v > 1:
            names["fwd_out"] = f"d{d}:fwd:{r}"
        if r > 0 or self.v > 1:
            names["fwd_in"] = f"d{d}:fwd:{(r - 1) % P}"
        if r > 0 or self.v > 1:
            names["bwd_out"] = f"d{d}:bwd:{r}"
        if r < P - 1 or self.v > 1:
            names["bwd_in"] = f"d{d}:bwd:{(r + 1) % P}"
        names["labels"] = f"d{d}:labels"
        return names

    def _build_channels(self, cfg: GlobalConfig, kind: str):
        """Every pipeline channel of the job, in one order on every rank: per replica, the
        forward channel out of each rank, the backward channel out of each rank, labels."""
        from revpp.parallel.channels import ChannelSet, ChannelSpec
        from revpp.parallel.schedule import min_channel_depth

        P, v = self.P, self.v
        act = TensorSpec((self.mbs, cfg.seq_len, cfg.hidden_size), torch.float32)
        two_stream = kind in ("reversible", "inverse")
        fwd = (act,) * (2 if two_stream else 1)
        depth = min_channel_depth(P, v, cfg.num_microbatches, cfg.schedule) + 1
        specs = []
        for d in range(self.D):
            base = d * P
            for r in range(P):
                if r < P - 1 or v > 1:
                    specs.append(ChannelSpec(f"d{d}:fwd:{r}", base + r, base + (r + 1) % P, fwd, depth))
            for r in range(P):
                if r > 0 or v > 1:
                    recv_stage = r - 1  # v == 1: the receiver is global stage r - 1
                    if kind == "inverse" and recv_stage == 0:
                        bwd = (act,) * 2
                    else:
                        bwd = (act,) * (4 if two_stream else 1)
                    specs.append(ChannelSpec(f"d{d}:bwd:{r}", base + r, base + (r - 1) % P, bwd, depth))
            specs.append(ChannelSpec(f"d{d}:labels", base, base + P - 1,
                                     (TensorSpec((self.local_batch,), torch.int64),), 2))
        return ChannelSet(specs, self.device)

    # ------------------------------------------------------------------ helpers
    @property
    def is_first(self) -> bool:
        return self.stage.is_first

    @property
    def is_last(self) -> bool:
        return self.last_stage.is_last

    @property
    def actv_records(self) -> list:
        return [r for st in self.stages for r in st.actv_records]

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

    def timed_train_step(self, batch: Optional[dict]) -> dict:
        """``train_step`` with a device timeline of the pipeline part: this rank's step,
        compute and idle time and its mean forward / backward action (ms), from CUDA events
        on the compute stream (``revpp.parallel.schedule.StepTimeline``)."""
        from .parallel.schedule import StepTimeline

        self.executor.timeline = StepTimeline()
        try:
            self.train_step(batch)
            out = self.executor.timeline.summary()
        finally:
            self.executor.timeline = None
        out.update({"rank": self.rank, "stage": self.stage_index, "replica": self.replica})
        return out

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
            st = self.last_stage
            logits = torch.cat(st.logits) if st.logits else None
            lab = torch.cat(st.labels) if st.labels is not None else None
            loss = torch.stack(losses).mean() if losses else None
            return loss, logits, lab
        return None

    def last_labels(self) -> Optional[torch.Tensor]:
        st = self.last_stage
        return torch.cat(st.labels) if st.labels is not None else None

    def last_logits(self) -> Optional[torch.Tensor]:
        st = self.last_stage
        return torch.cat(st.logits) if st.logits else None

    def close(self) -> None:
        if self.channels is not None:
            self.channels.close()
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
