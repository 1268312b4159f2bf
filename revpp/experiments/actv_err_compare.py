"""Reconstruction error of this framework against the reference's, on the same weights.

    torchrun --nproc-per-node 4 --master-addr 127.0.0.1 -m revpp.experiments.actv_err_compare \
        --layers 24 --microbatch-size 16 --num-microbatches 8 --out actv_err_compare.json

One training step of reversible BERT (hidden 1024, 16 heads, seq 512 by default; bf16) on
PP = world, run twice on the same batch:

1. the installed reference (baseline/_ref/BERT): its ``BertFirst/Mid/LastStage`` modules in
   ``RevPipelineStageWithPareprop(eval_actv_err=True)`` with ``Schedule1F1B``; the stage
   records, for every micro-batch, the per-sample MSE and cosine similarity of the
   reconstructed stage input against the input seen in forward, in fp64, on middle stages
   (BERT/pipelining/reversible_stage_with_pareprop.py:457-560);
2. this framework's ``Trainer`` with ``eval_actv_err`` on the reference's weights (its stage
   ``state_dict()`` loaded strictly), which records the same quantities
   (``ReversibleStage._record_actv_err``).

Rank 0 writes the per-stage distributions (count, max / p99 / median MSE, min / p1 cosine)
of both and whether this framework's worst values stay within the reference's:
``max MSE <= reference max MSE`` and ``min cosine >= reference min cosine``, pooled over
the middle stages.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF = os.path.join(HERE, "baseline", "_ref", "BERT")


def _summary(mse, cos):
    import numpy as np

    if not mse:
        return {"n": 0}
    m, c = np.asarray(mse, dtype=np.float64), np.asarray(cos, dtype=np.float64)
    return {"n": int(m.size), "mse_max": float(m.max()), "mse_p99": float(np.percentile(m, 99)),
            "mse_median": float(np.median(m)), "cos_min": float(c.min()), "cos_p1": float(np.percentile(c, 1)),
            "cos_median": float(np.median(c))}


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--layers", type=int, default=24)
    p.add_argument("--hidden", type=int, default=1024)
    p.add_argument("--heads", type=int, default=16)
    p.add_argument("--seq", type=int, default=512)
    p.add_argument("--microbatch-size", type=int, default=16)
    p.add_argument("--num-microbatches", type=int, default=8)
    p.add_argument("--out", default="actv_err_compare.json")
    a = p.parse_args(argv)
    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    if world < 3:
        raise SystemExit("needs at least 3 pipeline stages: the reference records middle stages only")
    import datetime

    # the reference's pipeline runs on NCCL only (its point-to-point ops hang on gloo)
    cpu = False
    dtype = torch.bfloat16
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    B = a.microbatch_size * a.num_microbatches
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 30522, (B, a.seq), generator=g)
    mask = torch.ones(B, a.seq, dtype=torch.int64)
    labels = torch.bernoulli(torch.full((B,), 0.5), generator=g).long()

    # ---------------------------------------------------------------- the reference
    sys.path.insert(0, REF)
    from models.bert_stages import BertFirstStage, BertLastStage, BertMidStage  # noqa: E402
    from pipelining import RevPipelineStageWithPareprop, Schedule1F1B  # noqa: E402

    torch.manual_seed(1000 + rank)
    kw = dict(hidden_size=a.hidden, num_attention_heads=a.heads, num_blocks=a.layers // world, enable_amp=not cpu,
              autocast_dtype=dtype, is_pareprop=False)
    if rank == 0:
        model = BertFirstStage(vocab_size=30522, max_position_embeddings=a.seq, type_vocab_size=2, **kw)
    elif rank == world - 1:
        model = BertLastStage(num_classes=2, **kw)
    else:
        model = BertMidStage(**kw)
    model = model.to(dev)
    weights = {k: v.detach().cpu().clone() for k, v in model.state_dict().items()}
    stage = RevPipelineStageWithPareprop(submodule=model, stage_index=rank, num_stages=world, device=dev,
                                         eval_actv_err=True)
    sched = Schedule1F1B(stage=stage, n_microbatches=a.num_microbatches, loss_fn=torch.nn.CrossEntropyLoss())
    lab_dev = labels.to(dev)
    if rank == 0:
        sched.step(ids.to(dev), mask.to(dev))
    elif rank == world - 1:
        sched.step(target=lab_dev, losses=[])
    else:
        sched.step()
    if not cpu:
        torch.cuda.synchronize()
    ref = (list(stage.mse_stats), list(stage.cos_stats))
    del sched, stage, model
    if not cpu:
        torch.cuda.empty_cache()
    dist.barrier()

    # ---------------------------------------------------------------- this framework
    sys.path.insert(0, HERE)
    from revpp.ckpt import strip_aliases
    from revpp.config import GlobalConfig, ParMode
    from revpp.engine import Trainer
    from revpp.utils.env import EnvContext
    from revpp.utils.logger import build_logger

    cfg = GlobalConfig(par_mode=ParMode.PP, reversible=True, model="bert", num_hidden_layers=a.layers,
                       hidden_size=a.hidden, num_attention_heads=a.heads, max_position_embeddings=a.seq,
                       num_classes=2, autocast_dtype=dtype, batch_size=B, p2p="copy",
                       microbatch_size=a.microbatch_size, num_microbatches=a.num_microbatches, lr=1e-7)
    env = EnvContext(world_size=world, rank=rank, local_rank=local, device=dev,
                     proc_logger=build_logger(f"ae{rank}", None), node_logger=None, main_logger=None,
                     pg=dist.group.WORLD, master_rank=world - 1, num_stages=world, replicas=1)
    tr = Trainer(cfg, env, eval_actv_err=True)
    missing, unexpected = tr.module.load_state_dict(strip_aliases(weights), strict=False)
    if missing or unexpected:
        raise RuntimeError(f"reference weights do not fit: {missing[:3]} {unexpected[:3]}")
    tr.flat.refresh_shadow()
    batch = {"input_ids": ids, "attention_mask": mask, "labels": labels}
    tr.train_step(batch if tr.is_first else None)
    if not cpu:
        torch.cuda.synchronize()
    mine = ([r["mse"] for r in tr.actv_records], [r["cos"] for r in tr.actv_records])
    tr.close()

    allr = [None] * world
    dist.all_gather_object(allr, (rank, ref, mine))
    if rank == 0:
        middle = [r for r in range(1, world - 1)]
        per = {}
        pooled = {"reference": ([], []), "revpp": ([], [])}
        for rk, rf, mn in allr:
            per[rk] = {"reference": _summary(*rf), "revpp": _summary(*mn)}
            if rk in middle:
                for name, src in (("reference", rf), ("revpp", mn)):
                    pooled[name][0].extend(src[0])
                    pooled[name][1].extend(src[1])
        pr, pm = _summary(*pooled["reference"]), _summary(*pooled["revpp"])
        res = {"config": {"model": "Rev-BERT", "layers": a.layers, "hidden": a.hidden, "heads": a.heads,
                          "seq_len": a.seq, "microbatch_size": a.microbatch_size,
                          "num_microbatches": a.num_microbatches, "pp": world,
                          "dtype": "fp32" if cpu else "bf16",
                          "weights": "the reference's random init, loaded into both"},
               "middle_stages": middle, "per_stage": per, "pooled_middle": {"reference": pr, "revpp": pm},
               "within_reference_bound": bool(pm.get("n", 0) > 0 and pr.get("n", 0) > 0
                                              and pm["mse_max"] <= pr["mse_max"] and pm["cos_min"] >= pr["cos_min"])}
        with open(a.out, "w") as fh:
            json.dump(res, fh, indent=2)
        print(json.dumps({"within_reference_bound": res["within_reference_bound"], "reference": pr, "revpp": pm}),
              flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
