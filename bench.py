"""Training-throughput benchmark: reversible BERT-Large (24 x 1024, 16 heads, seq 512, bf16),
pipeline-parallel over N GPUs (PP = N, 1F1B, one rank per GPU), global batch 512,
synthetic data, random init.

Micro-batch size (PaBER: reversible stages hold O(1) activations, so the micro-batch can be
expanded): 64 on a single stage, where there is no pipeline bubble and larger GEMMs run
fuller waves (measured on one B200: 16 -> 527, 64 -> 550, 128 -> 544 samples/s); 16 with
a pipeline, where 32 micro-batches keep the 1F1B bubble at (P-1)/(31+P) of the step.
``--microbatch-size`` overrides it (both implementations use the same value).

    python bench.py --gpus 1 --steps K --warmup W
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N --steps K --warmup W
    ... --impl reference        # the reference implementation on the same config

Secondary workloads (same JSON line; the reference arm covers the headline only):
    --model {bert-base,vit-b16,vit-l16-384}  --seq S (BERT)  --layers L
    --dp D          pipeline replicas: PP = N / D, replicas reduced by the fused NVLink kernel
    --stage {standard,checkpoint}            non-reversible stages for comparison
    --microbatch-size M --global-batch B     micro-batches per replica = B / (M * D)

Reported (rank 0 prints one JSON line):
  value  - samples/s of the whole job: global_batch / step time, where the step time is
           K full training steps (pipeline forward/backward of every micro-batch, gradient
           clipping, AdamW) timed with CUDA events between a barrier + synchronize on both
           sides, the maximum over ranks.
  e2e    - the same steps through Trainer.train_step with this step's inputs copied from
           pinned host memory and the loss read back to the host every step, wall clock,
           maximum over ranks.
  peak_hbm_gib - max over ranks of torch.cuda.max_memory_allocated.
  clocks - median SM clock and active throttle reasons sampled during the timed region.
  gpu_launches - kernels launched by this framework's extension inside the timed region
           (summed over ranks).
The working set (fp32 weights + Adam state of the stage, activations of 16 x 512 x 1024
micro-batches) is far larger than the 126 MB L2, so no flush is inserted between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
METRIC = "train samples/sec + peak HBM/GPU, Rev-BERT-Large PaBER at PP=1/2/4/8 vs ref"
MODEL = dict(hidden=1024, heads=16, layers=24, seq=512, vocab=30522, classes=2)
# defaults of the revpp arm with several pipeline stages
DEFAULT_P2P = "copy"
DEFAULT_SCHEDULE = "interleaved"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=6)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["revpp", "reference"], default="revpp")
    p.add_argument("--global-batch", type=int, default=512)
    p.add_argument("--microbatch-size", type=int, default=None,
                   help="default: 64 with one pipeline stage, 16 with several (PaBER sizing)")
    p.add_argument("--seq", type=int, default=MODEL["seq"])
    p.add_argument("--layers", type=int, default=MODEL["layers"])
    p.add_argument("--pareprop", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--model", choices=["bert-large", "bert-base", "vit-b16", "vit-l16-384"], default="bert-large",
                   help="secondary workloads; the headline is bert-large")
    p.add_argument("--dp", type=int, default=1, help="pipeline replicas: PP = gpus / dp")
    p.add_argument("--stage", choices=["reversible", "standard", "checkpoint"], default="reversible")
    p.add_argument("--schedule", choices=["1f1b", "interleaved"], default=None,
                   help="default: interleaved 1F1B with several pipeline stages (revpp arm), 1f1b otherwise")
    p.add_argument("--virtual-stages", type=int, default=None,
                   help="model chunks per rank with the interleaved schedule (default: one block per chunk "
                        "up to 3 chunks)")
    p.add_argument("--p2p", choices=["auto", "copy", "group"], default=DEFAULT_P2P,
                   help="stage messages: copy-engine channels or NCCL groups (revpp arm)")
    a = p.parse_args()
    if a.model != "bert-large" and a.layers == MODEL["layers"]:
        a.layers = None  # the preset's depth
    if a.gpus % a.dp != 0:
        p.error("--gpus must be a multiple of --dp")
    if a.microbatch_size is None:
        a.microbatch_size = 64 if a.gpus // a.dp == 1 else 16
    P = a.gpus // a.dp
    if a.schedule is None:
        a.schedule = DEFAULT_SCHEDULE if (P > 1 and a.impl == "revpp" and a.p2p != "group") else "1f1b"
    if a.virtual_stages is None:
        a.virtual_stages = default_virtual_stages(a, P)
    if a.schedule != "interleaved":
        a.virtual_stages = 1
    return a


def default_virtual_stages(a, P: int) -> int:
    """Chunks per rank for the interleaved schedule: as many as keep at least one block per
    chunk, at most 3, and a divisor of the blocks per rank."""
    if P <= 1:
        return 1
    from revpp.config import PRESETS

    layers = a.layers or PRESETS[a.model]["num_hidden_layers"]
    per_rank = layers // P
    for v in (3, 2):
        if per_rank % v == 0:
            return v
    return 1


MODEL_NAMES = {"bert-large": "Rev-BERT-Large", "bert-base": "Rev-BERT-Base", "vit-b16": "Rev-ViT-B/16",
               "vit-l16-384": "Rev-ViT-L/16@384"}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", init_method="env://", timeout=datetime.timedelta(seconds=900),
                                device_id=dev)
    return world, rank, local, dev


def barrier(dev):
    if dist.is_initialized():
        dist.barrier(device_ids=[dev.index])


def max_over_ranks(x: float, dev) -> float:
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, dev) -> float:
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def base_record(args, world, impl):
    from revpp.config import PRESETS

    pre = PRESETS[args.model]
    nmb = args.global_batch // (args.microbatch_size * args.dp)
    P = world // args.dp
    name = MODEL_NAMES[args.model]
    if args.stage != "reversible":
        name = name.replace("Rev-", "") + f" ({args.stage} stages)"
    if pre["model"] == "bert":
        seq = args.seq
        data = "synthetic (uniform token ids, all-ones mask, Bernoulli labels), random init"
    else:
        seq = (pre["img_size"] // pre["patch_size"]) ** 2 + 1
        data = "synthetic (i.i.d. N(0,1) pixels, uniform labels), random init"
    par = f"pp{P}" + (f"xdp{args.dp}" if args.dp > 1 else "")
    return {
        "metric": METRIC, "unit": "samples/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": data,
        "impl": impl,
        "config": {"model": name, "layers": args.layers or pre["num_hidden_layers"], "hidden": pre["hidden_size"],
                   "heads": pre["num_attention_heads"], "global_batch": args.global_batch, "seq_len": seq,
                   "microbatch_size": args.microbatch_size, "num_microbatches": nmb,
                   "parallelism": par,
                   "schedule": ("interleaved-1f1b" if args.schedule == "interleaved" else "1f1b"),
                   "virtual_stages": args.virtual_stages,
                   "backward": "pareprop" if args.pareprop else "sequential",
                   "l2": "no flush: per-step working set (weights, Adam state, activations) >> 126 MB L2"},
    }


# ============================================================================ revpp arm
def run_revpp(args):
    sys.path.insert(0, HERE)
    world, rank, local, dev = dist_setup(args.gpus)
    from revpp.config import GlobalConfig, ParMode
    from revpp.data import SyntheticBatches
    from revpp.engine import Trainer
    from revpp.ops import ext
    from revpp.utils.clocks import ClockSampler
    from revpp.utils.env import EnvContext
    from revpp.utils.logger import build_logger
    from revpp.utils.seed import set_seed

    from revpp.config import PRESETS

    C = ext()
    P = world // args.dp
    nmb = args.global_batch // (args.microbatch_size * args.dp)  # per replica
    pre = dict(PRESETS[args.model])
    if args.layers:
        pre["num_hidden_layers"] = args.layers
    if pre["model"] == "bert":
        pre["max_position_embeddings"] = args.seq
    par_mode = ParMode.PP if P > 1 or args.dp > 1 else ParMode.NONE
    cfg = GlobalConfig(par_mode=par_mode, reversible=args.stage == "reversible",
                       checkpointing=args.stage == "checkpoint", is_pareprop=args.pareprop, dp=args.dp,
                       schedule=args.schedule, virtual_stages=args.virtual_stages, p2p=args.p2p,
                       autocast_dtype=torch.bfloat16, batch_size=args.global_batch,
                       microbatch_size=args.microbatch_size, num_microbatches=nmb, lr=1e-5, dataset="synthetic",
                       **pre)
    lg = build_logger(f"bench{rank}", None)
    env = EnvContext(world_size=world, rank=rank, local_rank=local, device=dev, proc_logger=lg, node_logger=None,
                     main_logger=None, pg=dist.group.WORLD if dist.is_initialized() else None,
                     master_rank=world - 1, num_stages=P, replicas=args.dp)
    set_seed(cfg.seed + rank)
    tr = Trainer(cfg, env)
    data = SyntheticBatches(cfg, tr.local_batch, 4, seed=tr.replica)
    batches = [data.make(i) for i in range(4)] if tr.is_first else [None] * 4

    for i in range(args.warmup):
        tr.train_step(batches[i % 4])
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()

    # ---- device-timed region
    sampler = ClockSampler(local)
    barrier(dev)
    torch.cuda.synchronize()
    l0 = C.launch_count()
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    last = None
    for i in range(args.steps):
        last = tr.train_step(batches[i % 4])
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    barrier(dev)
    launches = C.launch_count() - l0
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = max_over_ranks(ms, dev)
    launches_total = sum_over_ranks(float(launches), dev)
    peak = max_over_ranks(torch.cuda.max_memory_allocated() / 2**30, dev)
    status = C.status_read_and_clear()

    # ---- end-to-end: public API, H2D of each step's inputs, D2H of each step's loss
    e2e = None
    if not args.no_e2e:
        h2d = sum(t.numel() * t.element_size() for t in batches[0].values()) if tr.is_first else 0
        barrier(dev)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(args.steps):
            loss = tr.train_step(batches[i % 4])
            if loss is not None:
                float(loss)  # device -> host read of the step's result
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) * 1e3 / args.steps
        barrier(dev)
        wall_max = max_over_ranks(wall, dev)
        h2d_total = sum_over_ranks(float(h2d), dev)
        e2e = {"value": args.global_batch / (wall_max / 1e3), "unit": "samples/s", "ms_per_step": wall_max,
               "h2d_bytes_per_step": int(h2d_total), "d2h_bytes_per_step": 4,
               "api": "revpp.engine.Trainer.train_step"}
    # ---- one more (untimed) step timed on the host: how long the host takes to enqueue a step
    # and how long the device still runs after that (a short drain means the host is the limit)
    torch.cuda.synchronize()
    h0 = time.perf_counter()
    tr.train_step(batches[0])
    h1 = time.perf_counter()
    torch.cuda.synchronize()
    h2 = time.perf_counter()
    host = {"enqueue_ms": round(max_over_ranks((h1 - h0) * 1e3, dev), 2),
            "drain_ms_min_over_ranks": round(-max_over_ranks(-(h2 - h1) * 1e3, dev), 2)}
    # ---- one more (untimed) step with a device timeline per rank: compute / bubble / exposed P2P
    breakdown = None
    if P > 1:
        mine = tr.timed_train_step(batches[0])
        allr = [None] * world
        dist.all_gather_object(allr, mine)
        from revpp.parallel.schedule import pipeline_breakdown

        pipe0 = sorted((r for r in allr if r["replica"] == 0), key=lambda r: r["stage"])
        breakdown = {"replica": 0, "method": "CUDA events around every action's compute on the compute stream; "
                     "bubble = the schedule's simulated idle time with each rank's measured mean action times",
                     "per_stage": [{k: (round(v, 3) if isinstance(v, float) else v) for k, v in d.items()}
                                   for d in pipeline_breakdown(pipe0, P, tr.v, nmb, args.schedule)]}
    loss_val = float(last) if last is not None else None
    tr.close()
    rec = base_record(args, world, "revpp")
    rec.update({"value": args.global_batch / (ms_max / 1e3), "ms_per_step": ms_max, "e2e": e2e,
                "gpu_launches": int(launches_total), "peak_hbm_gib": peak, "clocks": clocks,
                "device_status": status})
    rec["config"]["p2p"] = tr.p2p
    rec["host"] = host
    if breakdown is not None:
        rec["pipeline_breakdown"] = breakdown
    if loss_val is not None:
        rec["final_loss"] = loss_val
    # the loss lives on the last rank; rank 0 prints
    if dist.is_initialized():
        obj = [rec.get("final_loss")]
        dist.broadcast_object_list(obj, src=P - 1)
        rec["final_loss"] = obj[0]
    if rank == 0:
        print(json.dumps(rec), flush=True)
    if dist.is_initialized():
        barrier(dev)
        dist.destroy_process_group()


# ============================================================================ reference arm
REF_BASE = os.path.join(HERE, "baseline", "_ref")


def _ref_modules(args, world, rank, dev):
    """The reference's own stage module for this rank and its pipeline-stage class
    (BERT/experiment/base.py:165-278; Vit/experiment/base.py): reversible stages run in
    RevPipelineStageWithPareprop, standard ones in PipelineStage, activation-checkpoint
    ones in PipelineStageWithCP."""
    from revpp.config import PRESETS

    pre = PRESETS[args.model]
    bert = pre["model"] == "bert"
    sys.path.insert(0, os.path.join(REF_BASE, "BERT" if bert else "Vit"))
    import pipelining as refpp  # noqa: E402

    layers = args.layers or pre["num_hidden_layers"]
    kw = dict(hidden_size=pre["hidden_size"], num_attention_heads=pre["num_attention_heads"],
              num_blocks=layers // world, enable_amp=True, autocast_dtype=torch.bfloat16)
    rev = args.stage == "reversible"
    if rev:
        kw["is_pareprop"] = args.pareprop
    first, last = rank == 0, rank == world - 1
    if bert:
        if rev:
            from models.bert_stages import BertFirstStage as F, BertLastStage as L, BertMidStage as Mid  # noqa: E402
        else:
            from models.normal_bert_stages import (NormalBertFirstStage as F, NormalBertLastStage as L,  # noqa: E402
                                                   NormalBertMidStage as Mid)
        if first:
            model = F(vocab_size=MODEL["vocab"], max_position_embeddings=args.seq, type_vocab_size=2, **kw)
        elif last:
            model = L(num_classes=pre["num_classes"], **kw)
        else:
            model = Mid(**kw)
    else:
        if rev:
            from models.vit_stages import ViTFirstStage as F, ViTLastStage as L, ViTMidStage as Mid  # noqa: E402
        else:
            from models.normal_vit_stages import (NormalViTFirstStage as F, NormalViTLastStage as L,  # noqa: E402
                                                  NormalViTMidStage as Mid)
        img = dict(img_size=pre["img_size"], patch_size=pre["patch_size"], in_chans=3)
        if first:
            model = F(**img, **kw)
        elif last:
            model = L(num_classes=pre["num_classes"], **kw)
        else:
            model = Mid(**kw)
    stage_cls = {"reversible": refpp.RevPipelineStageWithPareprop, "standard": refpp.PipelineStage,
                 "checkpoint": refpp.PipelineStageWithCP}[args.stage]
    return model.to(dev), stage_cls, refpp.Schedule1F1B, pre


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.dp != 1:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference has no pipeline replicas (PP x DP): "
                              "its DDP/FSDP modes and its PP mode share the world group "
                              "(BERT/experiment/base.py:244-299)"}), flush=True)
        return
    if not os.path.isdir(REF_BASE):
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref not installed"}), flush=True)
        return
    if world < 2:
        if args.stage == "reversible":
            why = ("the reference cannot train a reversible model on one GPU: PP=1 builds a first stage without a "
                   "head (BERT/experiment/base.py:166) and its non-PP reversible model computes no body gradients "
                   "(BERT/models/reversible.py:125)")
        elif args.model.startswith("bert"):
            why = ("the reference's single-GPU BERT path fails: its engine passes attention_mask to a stage forward "
                   "that does not take it (BERT/src/engine.py:137 vs BERT/models/bert_stages.py:111)")
        else:
            why = "this arm measures the reference's pipeline path (Schedule1F1B), which needs at least 2 GPUs"
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
        return
    world, rank, local, dev = dist_setup(args.gpus)
    from revpp.utils.clocks import ClockSampler  # timing helper only

    torch.manual_seed(rank)
    nmb = args.global_batch // args.microbatch_size
    model, stage_cls, sched_cls, pre = _ref_modules(args, world, rank, dev)
    bert = pre["model"] == "bert"
    stage = stage_cls(submodule=model, stage_index=rank, num_stages=world, device=dev)
    sched = sched_cls(stage=stage, n_microbatches=nmb, loss_fn=torch.nn.CrossEntropyLoss())
    opt = torch.optim.AdamW(model.parameters(), lr=1e-5, weight_decay=0.01, eps=1e-6)
    g = torch.Generator().manual_seed(0)
    B, S = args.global_batch, args.seq
    if bert:
        host = [dict(ids=torch.randint(0, MODEL["vocab"], (B, S), generator=g).pin_memory(),
                     mask=torch.ones(B, S, dtype=torch.int64).pin_memory(),
                     labels=torch.bernoulli(torch.full((B,), 0.5), generator=g).long().pin_memory()) for _ in range(2)]
    else:
        I = pre["img_size"]
        host = [dict(images=torch.randn(B, 3, I, I, generator=g).pin_memory(),
                     labels=torch.randint(0, pre["num_classes"], (B,), generator=g).pin_memory()) for _ in range(2)]
    labels_buf = torch.zeros(B, dtype=torch.int64, device=dev)

    def step(i):
        # the loop body of the reference Engine (BERT/src/engine.py:160-281, Vit/src/engine.py);
        # its own loop deletes an unbound name after the first batch on rank 0
        # (BERT/src/engine.py:197).  Returns the batch loss on the last rank: the reference's
        # 1F1B turns every micro-batch loss into a host float (loss.item(),
        # schedules.py:778-784), and the engine averages them.
        b = host[i % 2]
        loss = None
        if rank == 0:
            lab = b["labels"].to(dev, non_blocking=True)
            if bert:
                ids = b["ids"].to(dev, non_blocking=True)
                mask = b["mask"].to(dev, non_blocking=True)
                dist.isend(lab, dst=world - 1).wait()
                sched.step(ids, mask)
            else:
                img = b["images"].to(dev, non_blocking=True)
                dist.isend(lab, dst=world - 1).wait()
                sched.step(img)
        elif rank == world - 1:
            dist.irecv(labels_buf, src=0).wait()
            losses = []
            sched.step(target=labels_buf, losses=losses)
            loss = sum(float(x) for x in losses) / len(losses)
        else:
            sched.step()
        for p in model.parameters():
            if p.grad is not None:
                p.grad.div_(nmb)
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        opt.zero_grad()
        return loss

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    sampler = ClockSampler(local)
    barrier(dev)
    torch.cuda.synchronize()
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    barrier(dev)
    ms_max = max_over_ranks(e0.elapsed_time(e1) / args.steps, dev)
    peak = max_over_ranks(torch.cuda.max_memory_allocated() / 2**30, dev)

    # ---- end-to-end, measured as the revpp arm measures it: each step's inputs go host ->
    # device from pinned memory inside the step (rank 0), the batch loss reaches the host
    # (the reference reads every micro-batch loss with .item()), wall clock, max over ranks
    e2e = None
    if not args.no_e2e:
        h2d = sum(t.numel() * t.element_size() for t in host[0].values()) if rank == 0 else 0
        barrier(dev)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(args.steps):
            loss = step(i)
            if loss is not None:
                float(loss)
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) * 1e3 / args.steps
        barrier(dev)
        wall_max = max_over_ranks(wall, dev)
        h2d_total = sum_over_ranks(float(h2d), dev)
        e2e = {"value": args.global_batch / (wall_max / 1e3), "unit": "samples/s", "ms_per_step": wall_max,
               "h2d_bytes_per_step": int(h2d_total), "d2h_bytes_per_step": 4 * nmb,
               "api": "pipelining.Schedule1F1B.step (reference Engine loop body)"}
    rec = base_record(args, world, "reference")
    rec.update({"value": args.global_batch / (ms_max / 1e3), "ms_per_step": ms_max, "e2e": e2e,
                "peak_hbm_gib": peak, "clocks": clocks, "gpu_launches": 0,
                "api": f"pipelining.{stage_cls.__name__} + Schedule1F1B (baseline/_ref/{'BERT' if bert else 'Vit'})"})
    if rank == 0:
        print(json.dumps(rec), flush=True)
    barrier(dev)
    dist.destroy_process_group()


if __name__ == "__main__":
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_revpp(a)
