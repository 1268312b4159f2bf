"""Run configuration: enums, the frozen GlobalConfig, presets and the CLI parser.

Same flags and invariants as the reference CLI (BERT/args.py:4-166, Vit/args.py:82-99,
BERT/src/config.py:9-143): ``microbatch_size * num_microbatches == batch_size`` and
``--is_pareprop`` requires ``--reversible``.  Additions: ``--model {bert,vit}`` (one entry
point for both families), ``--dataset synthetic``, ``--dp`` (pipeline replicas),
``--schedule``, ``--preset``, ``--global-clip`` and ``--ref-compat``.
"""
from __future__ import annotations

import argparse
import enum
import os
from dataclasses import dataclass, field, replace
from pathlib import Path

import torch


class ExpMode(enum.Enum):
    TRAINING = "training"
    PROFILING = "profiling"
    ACTV_ERR = "actv-err"
    ACC = "acc"


class ParMode(enum.Enum):
    NONE = "none"
    DDP = "ddp"
    FSDP = "fsdp"
    PP = "pp"


DATASET_ALIASES = {"cifar-10": "cifar10", "cifar-100": "cifar100"}

DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}
DTYPE_NAMES = {v: k for k, v in DTYPES.items()}

# Model presets (hidden, heads, layers, seq/img).  BERT vocab and type vocab come from
# bert-base-uncased (30522, 2).
PRESETS = {
    "tiny-bert": dict(model="bert", hidden_size=128, num_attention_heads=2, num_hidden_layers=4,
                      max_position_embeddings=128, num_classes=2),
    "bert-base": dict(model="bert", hidden_size=768, num_attention_heads=12, num_hidden_layers=12,
                      max_position_embeddings=512, num_classes=2),
    "bert-large": dict(model="bert", hidden_size=1024, num_attention_heads=16, num_hidden_layers=24,
                       max_position_embeddings=512, num_classes=2),
    "vit-b16": dict(model="vit", hidden_size=768, num_attention_heads=12, num_hidden_layers=12,
                    img_size=224, patch_size=16, num_classes=1000),
    "vit-l16-384": dict(model="vit", hidden_size=1024, num_attention_heads=16, num_hidden_layers=24,
                        img_size=384, patch_size=16, num_classes=1000),
}


@dataclass(frozen=True)
class GlobalConfig:
    # experiment / parallelism
    exp_mode: ExpMode = ExpMode.TRAINING
    par_mode: ParMode = ParMode.NONE
    is_pareprop: bool = False
    reversible: bool = False
    inverse: bool = False
    checkpointing: bool = False
    schedule: str = "1f1b"
    virtual_stages: int = 2
    p2p: str = "auto"
    dp: int = 1
    # model
    model: str = "bert"
    num_hidden_layers: int = 12
    hidden_size: int = 768
    num_attention_heads: int = 12
    max_position_embeddings: int = 512
    vocab_size: int = 30522
    type_vocab_size: int = 2
    img_size: int = 224
    patch_size: int = 16
    num_channels: int = 3
    num_classes: int = 2
    mlp_ratio: int = 4
    # data / training
    autocast_dtype: torch.dtype = torch.float32
    dataset: str = "synthetic"
    debug_subset: bool = False
    batch_size: int = 256
    microbatch_size: int = 64
    num_microbatches: int = 4
    num_epochs: int = 1
    lr: float = 0.01
    gamma: float = 1.0
    weight_decay: float = 0.01
    adam_eps: float = 1e-6
    max_grad_norm: float = 1.0
    global_clip: bool = False
    num_workers: int = 8
    seed: int = 0
    synthetic_batches: int = 8
    # paths
    dataset_rdir: Path = Path("/dataset")
    log_rdir: Path = Path("logs")
    checkpoint_rdir: Path = Path("checkpoints")
    profile_rdir: Path = Path("profiles")
    load_checkpoint: bool = False
    save_checkpoint: bool = False
    # behaviour switches
    ref_compat: bool = False  # reproduce reference quirks (see docs)
    device: str = "auto"      # auto | cuda | cpu
    # ids
    exp_id: str = ""
    env_id: str = ""

    @property
    def seq_len(self) -> int:
        if self.model == "vit":
            return (self.img_size // self.patch_size) ** 2 + 1
        return self.max_position_embeddings

    @property
    def intermediate_size(self) -> int:
        return self.hidden_size * self.mlp_ratio

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    def with_(self, **kw) -> "GlobalConfig":
        return replace(self, **kw)


def make_exp_id(exp_mode: str, par_mode: str, reversible: bool, is_pareprop: bool, inverse: bool,
                checkpointing: bool, dtype_name: str, dataset: str, seed: int, layers: int) -> str:
    """Experiment id in the reference's format (BERT/src/config.py:86-105)."""
    s = f"{exp_mode}_{par_mode}_"
    if reversible:
        if is_pareprop:
            s += "pareprop_"
        elif inverse:
            s += "inverse"
        else:
            s += "rev-seq_"
    elif checkpointing:
        s += "wcp_"
    else:
        s += "std_"
    return s + f"{dtype_name}_{dataset}_seed{seed:04d}numLayer{layers}"


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="revpp: reversible pipeline-parallel Transformer training")
    p.add_argument("--exp-mode", "-e", choices=[e.value for e in ExpMode], default=ExpMode.TRAINING.value)
    p.add_argument("--par-mode", choices=[e.value for e in ParMode], default=ParMode.NONE.value)
    p.add_argument("--reversible", action="store_true", default=False)
    p.add_argument("--inverse", action="store_true", default=False)
    p.add_argument("--is_pareprop", "--is-pareprop", dest="is_pareprop", action="store_true", default=False)
    p.add_argument("--checkpointing", action="store_true", default=False)
    p.add_argument("--dataset", default="synthetic",
                   choices=["synthetic", "imdb", "debug", "cifar10", "cifar100", "cinic10", "imagenet",
                            "cifar-10", "cifar-100"],
                   help="cifar-10 / cifar-100 are the reference's spellings of cifar10 / cifar100")
    p.add_argument("--model", choices=["bert", "vit"], default=None)
    p.add_argument("--preset", choices=sorted(PRESETS), default=None)
    p.add_argument("--num-hidden-layers", type=int, default=None)
    p.add_argument("--hidden-size", type=int, default=None)
    p.add_argument("--num-attention-heads", type=int, default=None)
    p.add_argument("--max-position-embeddings", type=int, default=None)
    p.add_argument("--img-size", type=int, default=None)
    p.add_argument("--patch-size", type=int, default=None)
    p.add_argument("--num-classes", type=int, default=None)
    p.add_argument("--autocast-dtype", choices=list(DTYPES), default="fp32")
    p.add_argument("--batch-size", type=int, default=256)
    p.add_argument("--microbatch-size", type=int, default=64)
    p.add_argument("--num-microbatches", type=int, default=4)
    p.add_argument("--lr", type=float, default=0.01)
    p.add_argument("--gamma", type=float, default=1.0)
    p.add_argument("--num-epochs", type=int, default=1)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--load-checkpoint", action="store_true", default=False)
    p.add_argument("--save-checkpoint", action="store_true", default=False)
    p.add_argument("--debug-subset", action="store_true", default=False)
    # additions
    p.add_argument("--dp", type=int, default=1, help="pipeline replicas (PP x DP)")
    p.add_argument("--schedule", choices=["1f1b", "gpipe", "interleaved"], default="1f1b",
                   help="interleaved: interleaved 1F1B with --virtual-stages model chunks per rank")
    p.add_argument("--virtual-stages", type=int, default=2,
                   help="model chunks per rank under --schedule interleaved")
    p.add_argument("--p2p", choices=["auto", "copy", "group"], default="auto",
                   help="stage messages: copy-engine channels (one node) or NCCL/gloo groups")
    p.add_argument("--global-clip", action="store_true", default=False,
                   help="clip by the norm over all stages instead of per stage")
    p.add_argument("--ref-compat", action="store_true", default=False,
                   help="reproduce reference quirks (num-epochs 1 trains nothing, ...)")
    p.add_argument("--synthetic-batches", type=int, default=8)
    p.add_argument("--device", choices=["auto", "cuda", "cpu"], default="auto")
    p.add_argument("--log-dir", default="logs")
    p.add_argument("--checkpoint-dir", default="checkpoints")
    p.add_argument("--profile-dir", default="profiles")
    p.add_argument("--dataset-dir", default="/dataset")
    return p


def parse_args(argv=None) -> argparse.Namespace:
    return build_parser().parse_args(argv)


def build_global_config(args: argparse.Namespace) -> GlobalConfig:
    """Namespace -> GlobalConfig with the reference's validation rules."""
    # the reference's invariant (BERT/src/config.py:77-82); with pipeline replicas the batch
    # is the global one, split evenly over the replicas
    if args.microbatch_size * args.num_microbatches * max(args.dp, 1) != args.batch_size:
        raise ValueError("batch_size must equal microbatch_size * num_microbatches * dp")
    if args.is_pareprop and not args.reversible:
        raise ValueError("is_pareprop=True requires reversible=True")
    if args.inverse and not args.reversible:
        raise ValueError("inverse=True requires reversible=True")
    base: dict = {}
    if args.preset:
        base.update(PRESETS[args.preset])
    model = args.model or base.get("model", "bert")
    base["model"] = model
    defaults = dict(num_hidden_layers=12, hidden_size=768, num_attention_heads=12, max_position_embeddings=512,
                    img_size=224, patch_size=16, num_classes=2 if model == "bert" else 1000)
    for k, dv in defaults.items():
        v = getattr(args, k, None)
        if v is not None:
            base[k] = v
        else:
            base.setdefault(k, dv)
    if base["hidden_size"] % base["num_attention_heads"] != 0:
        raise ValueError("hidden_size must be divisible by num_attention_heads")
    if args.dp < 1:
        raise ValueError("--dp must be >= 1")
    if args.schedule == "interleaved" and args.virtual_stages < 1:
        raise ValueError("--virtual-stages must be >= 1")
    dtype_name = args.autocast_dtype
    exp_id = make_exp_id(args.exp_mode, args.par_mode, args.reversible, args.is_pareprop, args.inverse,
                         args.checkpointing, dtype_name, args.dataset, args.seed, base["num_hidden_layers"])
    env_id = os.environ.get("SLURM_JOB_PARTITION", "UNKNOWN")
    return GlobalConfig(
        exp_mode=ExpMode(args.exp_mode), par_mode=ParMode(args.par_mode), is_pareprop=args.is_pareprop,
        reversible=args.reversible, inverse=args.inverse, checkpointing=args.checkpointing,
        schedule=args.schedule, virtual_stages=args.virtual_stages, p2p=args.p2p, dp=args.dp,
        autocast_dtype=DTYPES[dtype_name], dataset=DATASET_ALIASES.get(args.dataset, args.dataset),
        debug_subset=args.debug_subset,
        batch_size=args.batch_size, microbatch_size=args.microbatch_size, num_microbatches=args.num_microbatches,
        num_epochs=args.num_epochs, lr=args.lr, gamma=args.gamma, global_clip=args.global_clip, seed=args.seed,
        synthetic_batches=args.synthetic_batches,
        dataset_rdir=Path(args.dataset_dir), log_rdir=Path(args.log_dir), checkpoint_rdir=Path(args.checkpoint_dir),
        profile_rdir=Path(args.profile_dir), load_checkpoint=args.load_checkpoint,
        save_checkpoint=args.save_checkpoint, ref_compat=args.ref_compat, device=args.device,
        exp_id=exp_id, env_id=env_id, **base,
    )
