"""Pipeline runtime on CPU / gloo against a plain-autograd oracle.

Tiny reversible BERT, 2 pipeline stages x 2 reversible layers, fp32, global batch 16 in 4
micro-batches of 4, token ids uniform in [0, 30522), all-ones mask, Bernoulli labels: the
gradients of every parameter and the loss must match ordinary autograd through the same
network (which stores every activation) to 1e-5.  The same harness checks the standard,
activation-checkpoint, inverse and PaReprop variants and the 1F1B / GPipe schedules.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as Fn

from revpp.config import build_global_config, parse_args
from revpp.data import SyntheticBatches
from revpp.engine import Trainer, runtime_kind
from revpp.models.blockmath import TorchMath
from revpp.models.encoder import TorchEmbedHead, build_stage_module, stage_kind
from revpp.models.params import FlatParams
from revpp.utils.env import build_env
from revpp.utils.seed import set_seed


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg(extra: str, world: int):
    if "--model vit" in extra:
        base = ("--model vit --hidden-size 128 --num-attention-heads 2 --img-size 32 --patch-size 8 "
                "--num-classes 10 ")
    else:
        base = "--preset tiny-bert "
    args = parse_args((base + "--num-hidden-layers 4 --par-mode pp --batch-size 16 "
                       "--microbatch-size 4 --num-microbatches 4 --device cpu --lr 1e-3 " + extra).split())
    return build_global_config(args)


def _oracle(cfg, P, batch, v=1):
    """Full network with ordinary autograd; returns (loss, {rank: {name: grad}}).  With
    ``v`` chunks per rank, rank r builds global stages c * P + r (c = 0..v-1) in that order
    after seeding, as the Trainer does, and its gradient names carry the chunk prefix."""
    G = P * v
    mods = [None] * G
    for r in range(P):
        set_seed(cfg.seed + r)
        for c in range(v):
            mods[c * P + r] = build_stage_module(cfg, c * P + r, G, stage_kind(cfg))
    flats = [FlatParams(m, "cpu", want_shadow=False) for m in mods]
    maths = [TorchMath(f, torch.float32, cfg.num_attention_heads) for f in flats]
    eh0 = TorchEmbedHead(mods[0], flats[0], torch.float32)
    ehl = TorchEmbedHead(mods[-1], flats[-1], torch.float32)
    n = cfg.num_microbatches
    if cfg.model == "bert":
        inputs = list(zip(torch.chunk(batch["input_ids"], n), torch.chunk(batch["attention_mask"], n)))
    else:
        inputs = [(x,) for x in torch.chunk(batch["images"], n)]
    labels = torch.chunk(batch["labels"], n)
    total = 0.0
    for i in range(n):
        x = eh0._embed(inputs[i])
        reversible = cfg.reversible
        x2, x1 = x, x
        for s in range(G):
            for blk in mods[s].blocks:
                if reversible:
                    y1 = x1 + maths[s].attn(blk.F, x2).float()
                    y2 = x2 + maths[s].mlp(blk.G, y1).float()
                    x2, x1 = y2, y1
                else:
                    x2 = x2 + maths[s].attn(blk.F, x2).float()
                    x2 = x2 + maths[s].mlp(blk.G, x2).float()
        logits = ehl._head(x2, x1 if reversible else None)
        total = total + Fn.cross_entropy(logits.float(), labels[i]) / n
    total.backward()
    grads = [{} for _ in range(P)]
    for g, m in enumerate(mods):
        prefix = "" if v == 1 else f"chunks.{g // P}."
        for name, p in m.named_parameters():
            if p.grad is not None:
                grads[g % P][prefix + name] = p.grad.clone()
    return float(total), grads


def _worker(rank, world, port, extra, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        cfg = _cfg(extra, world)
        env = build_env(cfg, timeout_s=120)
        set_seed(cfg.seed + rank)
        tr = Trainer(cfg, env)
        # each pipeline replica reads its own local batch
        batch = SyntheticBatches(cfg, tr.local_batch, 1, seed=123 + tr.replica).make(0)
        inputs = tr.split_inputs(batch) if tr.is_first else None
        labels = batch["labels"] if tr.is_first else None
        losses = tr.executor.step(inputs, labels, train=True)
        if tr.dp_reducer is not None:
            tr.dp_reducer.reduce(tr.flat.grad)
        grads = {name: g.clone() for name, g in tr.flat.named_grads()}
        loss = float(torch.stack(losses).mean()) if tr.is_last else None
        if tr.dp_reducer is not None:
            # the optimizer step must leave every replica with the same parameters
            tr.opt.step(tr.opt.grad_sumsq())
            grads["__params__"] = tr.flat.data.clone()
        gathered = [None] * world
        dist.all_gather_object(gathered, (loss, grads))
        tr.close()
        if rank == 0:
            # numpy arrays pickle by value (tensors would go through shared-memory handles
            # that die with this process)
            q.put(("ok", [(l, {k: v.numpy() for k, v in g.items()}) for l, g in gathered]))
        env.close()
    except Exception as e:  # noqa: BLE001
        import traceback

        q.put(("err", f"rank {rank}: {traceback.format_exc()}"))
        raise


def _run(extra: str, world: int = 2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, extra, q)) for r in range(world)]
    for p in procs:
        p.start()
    status, payload = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
    assert status == "ok", payload
    return [(l, {k: torch.from_numpy(v) for k, v in g.items()}) for l, g in payload]


@pytest.mark.parametrize("extra", [
    "--reversible",
    "--reversible --model vit",
    "--reversible --schedule gpipe",
    "--reversible --is_pareprop",
    "--reversible --inverse",
    "",
    "--checkpointing",
])
def test_pipeline_matches_autograd(extra):
    world = 2
    gathered = _run(extra, world)
    cfg = _cfg(extra, world)
    batch = SyntheticBatches(cfg, cfg.batch_size, 1, seed=123).make(0)
    ref_loss, ref_grads = _oracle(cfg, world, batch)
    loss = gathered[-1][0]
    assert abs(loss - ref_loss) <= 1e-5 * max(1.0, abs(ref_loss)), (loss, ref_loss)
    for s in range(world):
        got = gathered[s][1]
        assert set(got) == set(ref_grads[s]), (sorted(got)[:5], sorted(ref_grads[s])[:5])
        for name, g in got.items():
            r = ref_grads[s][name]
            err = (g - r).abs().max().item()
            scale = r.abs().max().item()
            assert err <= 1e-5 * max(scale, 1e-3), f"stage {s} {name}: err {err:.3e} scale {scale:.3e}"


def test_four_stage_reversible():
    gathered = _run("--reversible --num-hidden-layers 4", world=4)
    cfg = _cfg("--reversible --num-hidden-layers 4", 4)
    batch = SyntheticBatches(cfg, cfg.batch_size, 1, seed=123).make(0)
    ref_loss, ref_grads = _oracle(cfg, 4, batch)
    assert abs(gathered[-1][0] - ref_loss) <= 1e-5 * max(1.0, abs(ref_loss))
    for s in range(4):
        for name, g in gathered[s][1].items():
            r = ref_grads[s][name]
            assert (g - r).abs().max().item() <= 1e-5 * max(r.abs().max().item(), 1e-3), (s, name)


def test_pipeline_replicas_average_gradients():
    """PP = 2 x DP = 2 on 4 gloo ranks: after the replica all-reduce every stage holds the
    mean of the two replicas' gradients (each replica on its own local batch), and the
    optimizer step leaves both replicas with identical parameters."""
    extra = "--reversible --dp 2 --microbatch-size 2"
    world = 4
    gathered = _run(extra, world)
    cfg = _cfg(extra, world)
    P = 2
    local = cfg.batch_size // 2
    refs = [_oracle(cfg, P, SyntheticBatches(cfg, local, 1, seed=123 + d).make(0)) for d in range(2)]
    for d in range(2):
        assert abs(gathered[d * P + P - 1][0] - refs[d][0]) <= 1e-5 * max(1.0, abs(refs[d][0]))
    for s in range(P):
        g0, g1 = gathered[s][1], gathered[P + s][1]
        assert torch.equal(g0.pop("__params__"), g1.pop("__params__")), f"stage {s}: replicas diverged"
        for name, g in g0.items():
            r = 0.5 * (refs[0][1][s][name] + refs[1][1][s][name])
            scale = r.abs().max().item()
            assert (g - r).abs().max().item() <= 1e-5 * max(scale, 1e-3), (s, name)
            assert torch.equal(g, g1[name]), (s, name)


def _check(gathered, cfg, P, v=1):
    batch = SyntheticBatches(cfg, cfg.batch_size, 1, seed=123).make(0)
    ref_loss, ref_grads = _oracle(cfg, P, batch, v)
    loss = gathered[P - 1][0]
    assert abs(loss - ref_loss) <= 1e-5 * max(1.0, abs(ref_loss)), (loss, ref_loss)
    for r in range(P):
        got = gathered[r][1]
        assert set(got) == set(ref_grads[r]), (sorted(got)[:5], sorted(ref_grads[r])[:5])
        for name, g in got.items():
            ref = ref_grads[r][name]
            scale = ref.abs().max().item()
            assert (g - ref).abs().max().item() <= 1e-5 * max(scale, 1e-3), f"rank {r} {name}"


@pytest.mark.parametrize("extra,world", [
    ("--reversible --p2p copy", 2),
    ("--reversible --p2p copy --is_pareprop", 2),
    ("--p2p copy --checkpointing", 2),
    ("--reversible --p2p copy", 4),
    ("--reversible --p2p copy --schedule interleaved --virtual-stages 2", 2),
    ("--reversible --p2p copy --schedule interleaved --virtual-stages 2 --num-hidden-layers 8", 4),
    ("--p2p copy --schedule interleaved --virtual-stages 2", 2),
])
def test_copy_channels_match_autograd(extra, world):
    """Copy channels (shared-memory slots on CPU, the protocol of the GPU's copy-engine
    channels) with 1F1B and interleaved 1F1B: same loss and gradients as autograd."""
    gathered = _run(extra, world)
    cfg = _cfg(extra, world)
    v = cfg.virtual_stages if cfg.schedule == "interleaved" else 1
    _check(gathered, cfg, world, v)


def _train_worker(rank, world, port, extra, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        args = parse_args(("--preset tiny-bert --num-hidden-layers 2 --batch-size 8 --microbatch-size 4 "
                           "--num-microbatches 2 --device cpu --lr 1e-2 --reversible " + extra).split())
        cfg = build_global_config(args)
        env = build_env(cfg, timeout_s=120)
        set_seed(cfg.seed)
        tr = Trainer(cfg, env)
        batch = SyntheticBatches(cfg, tr.local_batch, 1, seed=300 + rank).make(0)
        for _ in range(2):
            tr.train_step(batch)
        out = (tr.flat.data.clone().numpy(), int(tr.flat.exp_avg.numel()), int(tr.flat.numel))
        gathered = [None] * world
        dist.all_gather_object(gathered, out)
        if rank == 0:
            q.put(("ok", gathered))
        env.close()
    except Exception:  # noqa: BLE001
        import traceback

        q.put(("err", f"rank {rank}: {traceback.format_exc()}"))
        raise


def _run_train(extra, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_train_worker, args=(r, world, port, extra, q)) for r in range(world)]
    for p in procs:
        p.start()
    status, payload = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
    assert status == "ok", payload
    return payload


def test_fsdp_shards_adam_state_and_matches_ddp():
    """--par-mode fsdp (ZeRO-2): each rank holds Adam moments of its half only, and two
    steps leave the same parameters as --par-mode ddp, identical on both ranks."""
    fsdp = _run_train("--par-mode fsdp")
    ddp = _run_train("--par-mode ddp")
    for (p, n_m, n), (pd, n_md, _) in zip(fsdp, ddp):
        assert n_m == n // 2 and n_md == n
        assert abs(p - pd).max() < 1e-5, abs(p - pd).max()
    assert (fsdp[0][0] == fsdp[1][0]).all()
