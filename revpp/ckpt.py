"""Checkpoint I/O with the reference's per-stage layout (BERT/src/ckpt_io.py:15-78).

  checkpoints/{par}_{rev|std}_{autocast dtype}_{dataset}_{seed:04d}/latest_rank{r}.pth   (pp / fsdp)
  checkpoints/{par}_{rev|std}_{autocast dtype}_{dataset}_{seed:04d}/latest.pth           (none / ddp)

The file holds the stage module's ``state_dict`` (torch.save).  The reference wraps each
reversible block in ParePropReversibleBlockWrapper, which registers the block three times
(``block``, ``F``, ``G``), so its files carry every block parameter twice:
``...layers.{i}.block.F.*`` and ``...layers.{i}.F.*``.  Saving writes both spellings; loading
accepts either and checks that every parameter is present (strict).  The dtype segment is
``str(torch.dtype)`` (e.g. ``torch.bfloat16``) as in the reference.

Optimizer moments, step count, learning rate and epoch go to a sibling
``*.optim.pth`` so the reference layout stays untouched; resume restores them when present.
"""
from __future__ import annotations

import re
from pathlib import Path
from typing import Optional

import torch

from revpp.config import GlobalConfig, ParMode

_ALIAS = re.compile(r"^(.*\.layers\.\d+)\.(F|G)\.(.*)$")
_ALIASED = re.compile(r"^(.*\.layers\.\d+)\.block\.(F|G)\.(.*)$")


def ckpt_dir(cfg: GlobalConfig) -> Path:
    tag = "rev" if cfg.reversible else "std"
    return cfg.checkpoint_rdir / f"{cfg.par_mode.value}_{tag}_{cfg.autocast_dtype}_{cfg.dataset}_{cfg.seed:04d}"


def file_name(cfg: GlobalConfig, rank: int) -> str:
    if cfg.par_mode in (ParMode.PP, ParMode.FSDP):
        return f"latest_rank{rank}.pth"
    return "latest.pth"


def with_aliases(sd: dict, kind: str) -> dict:
    """Add the wrapper-alias keys the reference writes for reversible blocks."""
    out = dict(sd)
    if kind != "reversible":
        return out
    for k, v in sd.items():
        m = _ALIAS.match(k)
        if m:
            out[f"{m.group(1)}.block.{m.group(2)}.{m.group(3)}"] = v
    return out


def strip_aliases(sd: dict) -> dict:
    out = {}
    for k, v in sd.items():
        m = _ALIASED.match(k)
        if m:
            canon = f"{m.group(1)}.{m.group(2)}.{m.group(3)}"
            out.setdefault(canon, v)
        else:
            out[k] = v
    return out


def save_checkpoint(trainer, cfg: GlobalConfig, rank: int, epoch: int = 0, extra: Optional[dict] = None) -> Path:
    d = ckpt_dir(cfg)
    d.mkdir(parents=True, exist_ok=True)
    path = d / file_name(cfg, rank)
    if cfg.par_mode in (ParMode.NONE, ParMode.DDP) and rank != 0:
        return path
    sd = {k: v.detach().cpu().clone() for k, v in trainer.module.state_dict().items()}
    torch.save(with_aliases(sd, trainer.module.kind), path)
    opt = {"optimizer": trainer.opt.state_dict(), "epoch": epoch, "lr_epoch": trainer.lr_sched.epoch,
           "step_count": trainer.step_count}
    if extra:
        opt.update(extra)
    torch.save(opt, path.with_suffix(".optim.pth"))
    return path


def load_checkpoint(trainer, cfg: GlobalConfig, rank: int, strict: bool = True) -> Optional[dict]:
    path = ckpt_dir(cfg) / file_name(cfg, rank)
    sd = torch.load(path, map_location="cpu")
    sd = strip_aliases(sd)
    missing, unexpected = trainer.module.load_state_dict(sd, strict=False)
    if strict and (missing or unexpected):
        raise RuntimeError(f"checkpoint {path} does not match the stage: missing {missing[:5]}, "
                           f"unexpected {unexpected[:5]}")
    if trainer.flat.shadow is not None:
        trainer.flat.refresh_shadow()
    opath = path.with_suffix(".optim.pth")
    if opath.exists():
        st = torch.load(opath, map_location="cpu")
        trainer.opt.load_state_dict(st["optimizer"])
        trainer.lr_sched.epoch = int(st.get("lr_epoch", 0))
        trainer.step_count = int(st.get("step_count", 0))
        return st
    return None
