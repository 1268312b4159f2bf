"""Worker for the multi-GPU tests (launched by torchrun from tests/test_multi_gpu.py).

modes:
  pipeline  - reversible BERT on the kernels, PP = world: the pipelined loss of one batch
              equals the loss of the same weights run as one stage on rank 0, and three
              training steps stay finite with a clean device status.
  dp        - PP = 1 x DP = world: the fused NVLink all-reduce + AdamW kernel gives the same
              parameters as the NCCL all-reduce followed by AdamW.
  grads     - reversible BERT on the kernels, PP = world (REVPP_MGPU_ARGS picks the transport
              and the schedule): every parameter's gradient of one pipelined step equals the
              gradient of the same weights run as one stage on rank 0, so the messages across
              stage boundaries (gradients and reconstructed inputs) are right.
  memory    - reversible BERT-Large width, PP = world, 2 blocks per stage: the memory a
              training step allocates on top of what lives between steps, per rank.
"""
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from revpp.config import GlobalConfig, ParMode  # noqa: E402
from revpp.data import SyntheticBatches  # noqa: E402
from revpp.engine import Trainer  # noqa: E402
from revpp.ops import ext  # noqa: E402
from revpp.utils.env import build_env  # noqa: E402
from revpp.utils.seed import set_seed  # noqa: E402


def _extra():
    """REVPP_MGPU_ARGS="p2p=copy,schedule=interleaved,v=2" -> dict."""
    kv = {}
    for item in filter(None, os.environ.get("REVPP_MGPU_ARGS", "").split(",")):
        k, v = item.split("=")
        kv[k] = v
    return kv


def cfg_for(mode, world):
    ex = _extra()
    v = int(ex.get("v", "1"))
    sched = dict(p2p=ex.get("p2p", "auto"), schedule=ex.get("schedule", "1f1b"), virtual_stages=v)
    common = dict(model="bert", reversible=True, num_hidden_layers=2 * world, hidden_size=256,
                  num_attention_heads=4, max_position_embeddings=128, autocast_dtype=torch.bfloat16, lr=1e-3)
    if mode == "grads":
        common["num_hidden_layers"] = 2 * world * v
        return GlobalConfig(par_mode=ParMode.PP, batch_size=16, microbatch_size=2, num_microbatches=8, **common,
                            **sched)
    if mode == "memory":
        common.update(num_hidden_layers=2 * world, hidden_size=1024, num_attention_heads=16,
                      max_position_embeddings=512, lr=1e-5)
        return GlobalConfig(par_mode=ParMode.PP, batch_size=16, microbatch_size=2, num_microbatches=8, **common,
                            **sched)
    if mode == "pipeline":
        return GlobalConfig(par_mode=ParMode.PP, batch_size=16, microbatch_size=2, num_microbatches=8, **common)
    return GlobalConfig(par_mode=ParMode.DDP, batch_size=8 * world, microbatch_size=4, num_microbatches=2, **common)


def _single_name(key, g, per_stage):
    """Stage-local parameter name of global stage g -> name in a single-stage model."""
    if key.startswith("chunks."):
        key = key.split(".", 2)[2]
    if ".layers." in key:
        _, rest = key.split(".layers.", 1)
        i, tail = rest.split(".", 1)
        return f"body.layers.{g * per_stage + int(i)}.{tail}"
    return key


def _grads(cfg, tr, env, out, world):
    from revpp.models.blockmath import make_math
    from revpp.models.encoder import build_stage_module, make_embed_head
    from revpp.models.params import FlatParams
    from revpp.parallel.schedule import PipelineExecutor
    from revpp.parallel.stage import ReversibleStage

    batch = SyntheticBatches(cfg, cfg.batch_size, 1, seed=5).make(0)
    inputs = tr.split_inputs(batch) if tr.is_first else None
    labels = batch["labels"] if tr.is_first else None
    tr.flat.zero_grad()
    losses = tr.executor.step(inputs, labels, train=True)
    torch.cuda.synchronize()
    P, v = tr.P, tr.v
    G = P * v
    per_stage = cfg.num_hidden_layers // G
    mine = {}
    for name, g in tr.flat.named_grads():
        c = int(name.split(".")[1]) if name.startswith("chunks.") else 0
        mine[_single_name(name, c * P + tr.stage_index, per_stage)] = g.detach().cpu()
    weights = {}
    for name, t in tr.module.state_dict().items():
        c = int(name.split(".")[1]) if name.startswith("chunks.") else 0
        weights[_single_name(name, c * P + tr.stage_index, per_stage)] = t.detach().cpu()
    loss = float(torch.stack(losses).mean()) if tr.is_last else None
    gathered = [None] * world
    dist.all_gather_object(gathered, (loss, mine, weights))
    out["p2p"] = tr.p2p
    out["v"] = v
    if env.rank != 0:
        return
    from revpp.config import GlobalConfig as GC

    single = GC(**{**cfg.__dict__, "par_mode": ParMode.NONE, "schedule": "1f1b"})
    merged = {}
    for _, _, w in gathered:
        merged.update(w)
    dev = env.device
    mod = build_stage_module(single, 0, 1, "reversible").to(dev)
    mod.load_state_dict(merged)
    fl = FlatParams(mod, dev, want_shadow=True)
    mth = make_math(fl, torch.bfloat16, cfg.num_attention_heads, dev)
    eh = make_embed_head(mod, fl, torch.bfloat16, dev)
    st = ReversibleStage(mod, mth, eh, cfg.microbatch_size, cfg.num_microbatches, dev)
    ex = PipelineExecutor(st, None, cfg.num_microbatches, "1f1b")
    n = cfg.num_microbatches
    ins = list(zip(torch.chunk(batch["input_ids"].to(dev), n), torch.chunk(batch["attention_mask"].to(dev), n)))
    ref_losses = ex.step(ins, batch["labels"].to(dev), train=True)
    torch.cuda.synchronize()
    ref = {name: g.detach().cpu() for name, g in fl.named_grads()}
    out["pp_loss"] = gathered[-1][0]
    out["single_loss"] = float(torch.stack(ref_losses).mean())
    worst, worst_name, names = 0.0, "", set()
    for _, g, _ in gathered:
        for name, t in g.items():
            names.add(name)
            r = ref[name].double()
            e = (t.double() - r).norm().item() / max(r.norm().item(), 1e-12)
            if e > worst:
                worst, worst_name = e, name
    out["worst_rel"] = worst
    out["worst_name"] = worst_name
    out["missing"] = sorted(set(ref) - names)


def main():
    mode = sys.argv[1]
    world = int(os.environ["WORLD_SIZE"])
    cfg = cfg_for(mode, world)
    env = build_env(cfg, timeout_s=120)
    rank = env.rank
    set_seed(cfg.seed + rank)
    tr = Trainer(cfg, env)
    C = ext()
    out = {"rank": rank}
    if mode == "pipeline":
        batch = SyntheticBatches(cfg, cfg.batch_size, 1, seed=5).make(0)
        inputs = tr.split_inputs(batch) if tr.is_first else None
        labels = batch["labels"] if tr.is_first else None
        losses = tr.executor.step(inputs, labels, train=True)
        tr.flat.zero_grad()
        sd = {k: v.detach().cpu() for k, v in tr.module.state_dict().items()}
        gathered = [None] * world
        dist.all_gather_object(gathered, (float(torch.stack(losses).mean()) if tr.is_last else None, sd))
        if rank == 0:
            # the same weights as one stage: renumber blocks into body.layers.*
            from revpp.config import GlobalConfig as G
            from revpp.engine import Trainer as T
            from revpp.utils.env import EnvContext
            from revpp.utils.logger import build_logger

            single = G(**{**cfg.__dict__, "par_mode": ParMode.NONE})
            env1 = EnvContext(1, 0, 0, env.device, build_logger("one", None), None, None, None, 0)
            t1 = T.__new__(T)
            merged = {}
            off = 0
            for s, (_, sdd) in enumerate(gathered):
                n_here = 0
                for k, v in sdd.items():
                    if ".layers." in k:
                        pre, rest = k.split(".layers.", 1)
                        i, tail = rest.split(".", 1)
                        merged[f"body.layers.{int(i) + off}.{tail}"] = v
                        n_here = max(n_here, int(i) + 1)
                    else:
                        merged[k] = v
                off += n_here
            from revpp.models.blockmath import make_math
            from revpp.models.encoder import build_stage_module, make_embed_head
            from revpp.models.params import FlatParams
            from revpp.models.reversible import rev_forward

            mod = build_stage_module(single, 0, 1, "reversible").to(env.device)
            mod.load_state_dict(merged)
            fl = FlatParams(mod, env.device, want_shadow=True)
            mth = make_math(fl, torch.bfloat16, cfg.num_attention_heads, env.device)
            eh = make_embed_head(mod, fl, torch.bfloat16, env.device)
            ids = batch["input_ids"].to(env.device)
            tt = batch["attention_mask"].to(env.device)
            lab = batch["labels"].to(env.device)
            ls = []
            for i, (a, b, c) in enumerate(zip(torch.chunk(ids, cfg.num_microbatches), torch.chunk(tt, cfg.num_microbatches),
                                               torch.chunk(lab, cfg.num_microbatches))):
                x = eh.embed_fwd((a, b))
                y2, y1 = rev_forward(mth, mod.blocks, x, x)
                loss, _ = eh.head_eval(y2, y1, c)
                ls.append(float(loss))
            out["pp_loss"] = gathered[-1][0]
            out["single_loss"] = sum(ls) / len(ls)
        steps = []
        for i in range(3):
            l = tr.train_step(batch if tr.is_first else None)
            steps.append(float(l) if l is not None else None)
        torch.cuda.synchronize()
        out["losses"] = steps
    elif mode == "grads":
        _grads(cfg, tr, env, out, world)
    elif mode == "memory":
        batch = SyntheticBatches(cfg, cfg.batch_size, 1, seed=5).make(0)
        tr.train_step(batch if tr.is_first else None)
        torch.cuda.synchronize()
        base = torch.cuda.memory_allocated()
        torch.cuda.reset_peak_memory_stats()
        tr.train_step(batch if tr.is_first else None)
        torch.cuda.synchronize()
        out["transient"] = torch.cuda.max_memory_allocated() - base
        out["persistent"] = base
        out["p2p"] = tr.p2p
    else:
        from revpp.parallel.allreduce import NcclReducer

        batch = SyntheticBatches(cfg, tr.local_batch, 1, seed=11 + rank).make(0)
        init = tr.flat.data.clone()
        out["fused"] = type(tr.dp_reducer).__name__
        tr.train_step(batch)
        torch.cuda.synchronize()
        p_fused = tr.flat.data.clone()
        # same step through NCCL + AdamW
        tr.flat.data.copy_(init)
        tr.flat.refresh_shadow()
        tr.flat.exp_avg.zero_()
        tr.flat.exp_avg_sq.zero_()
        tr.flat.step = 0
        tr.flat.zero_grad()
        tr.dp_reducer = NcclReducer(tr.dp_group, tr.D)
        tr.train_step(batch)
        torch.cuda.synchronize()
        p_nccl = tr.flat.data.clone()
        out["max_diff"] = float((p_fused - p_nccl).abs().max())
        out["max_step"] = float((p_nccl - init).abs().max())
        other = p_fused.clone()
        dist.broadcast(other, src=0)
        out["replica_diff"] = float((other - p_fused).abs().max())
    out["status"] = C.status_read_and_clear()
    # one file per rank: concurrent ranks interleave their lines on a shared stdout
    res_dir = os.environ.get("REVPP_MGPU_RESULT_DIR")
    if res_dir:
        with open(os.path.join(res_dir, f"rank{out['rank']}.json"), "w") as fh:
            json.dump(out, fh)
    print("RESULT " + json.dumps(out), flush=True)
    tr.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
