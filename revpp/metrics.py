"""Loss / accuracy tracking (BERT/src/metric_tracker.py:7-195).

Per-epoch loss, top-1 / top-5 accuracy and per-class accuracy (mean / max / min), reduced
over ranks at epoch end and appended to ``metrics.csv`` next to the main log.  Updates
stay on the device; the only host reads are at logging points.
"""
from __future__ import annotations

import csv
import logging
from pathlib import Path
from typing import Optional, Sequence

import torch
import torch.distributed as dist


def topk_correct_per_class(logits: torch.Tensor, labels: torch.Tensor, num_classes: int, k: int) -> torch.Tensor:
    k = min(k, logits.shape[-1])
    top = logits.topk(k, dim=-1).indices
    hit = (top == labels[:, None]).any(dim=-1).to(torch.float32)
    out = torch.zeros(num_classes, dtype=torch.float32, device=logits.device)
    return out.index_add_(0, labels, hit)


class MetricTracker:
    def __init__(self, num_classes: int, topk: Sequence[int] = (1, 5), num_epochs: int = 1,
                 device: torch.device = torch.device("cpu"), logger: Optional[logging.Logger] = None,
                 csv_path: Optional[Path] = None):
        self.num_classes = num_classes
        self.topk = tuple(topk)
        self.num_epochs = num_epochs
        self.device = device
        self.logger = logger
        self.csv_path = csv_path
        self.reset("train", 0)

    def reset(self, split: str, epoch: int) -> None:
        self.split = split
        self.epoch = epoch
        self.loss_sum = torch.zeros((), dtype=torch.float32, device=self.device)
        self.count = torch.zeros((), dtype=torch.int64, device=self.device)
        self.class_count = torch.zeros(self.num_classes, dtype=torch.float32, device=self.device)
        self.correct = {k: torch.zeros(self.num_classes, dtype=torch.float32, device=self.device) for k in self.topk}
        self.batches = 0

    def update(self, loss: torch.Tensor, logits: Optional[torch.Tensor], labels: Optional[torch.Tensor]) -> None:
        self.batches += 1
        if labels is None:
            return
        n = labels.shape[0]
        self.loss_sum += loss.detach().float() * n
        self.count += n
        self.class_count.index_add_(0, labels, torch.ones_like(labels, dtype=torch.float32))
        if logits is not None:
            for k in self.topk:
                self.correct[k] += topk_correct_per_class(logits, labels, self.num_classes, k)

    def sync(self, group=None) -> None:
        if dist.is_available() and dist.is_initialized():
            for t in [self.loss_sum, self.count, self.class_count] + list(self.correct.values()):
                dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)

    def summary(self) -> dict:
        n = max(int(self.count.item()), 1)
        out = {"split": self.split, "epoch": self.epoch, "loss": float(self.loss_sum.item()) / n, "samples": n}
        cc = self.class_count.clamp(min=1)
        for k in self.topk:
            out[f"top{k}"] = float(self.correct[k].sum().item()) / n
            per = (self.correct[k] / cc)[self.class_count > 0]
            if per.numel():
                out[f"top{k}_class_mean"] = float(per.mean())
                out[f"top{k}_class_max"] = float(per.max())
                out[f"top{k}_class_min"] = float(per.min())
        return out

    def log_batch(self, batch_idx: int, num_batches: int, loss: Optional[float] = None) -> None:
        if self.logger:
            self.logger.info("[%s epoch %d] batch %d/%d%s", self.split, self.epoch, batch_idx, num_batches,
                             "" if loss is None else f" loss {loss:.6f}")

    def log_epoch(self) -> dict:
        s = self.summary()
        if self.logger:
            self.logger.info("[%s epoch %d] %s", self.split, self.epoch,
                             ", ".join(f"{k}={v:.5f}" if isinstance(v, float) else f"{k}={v}" for k, v in s.items()))
        if self.csv_path is not None and self.logger is not None:
            new = not self.csv_path.exists()
            self.csv_path.parent.mkdir(parents=True, exist_ok=True)
            with open(self.csv_path, "a", newline="") as fh:
                w = csv.DictWriter(fh, fieldnames=sorted(s))
                if new:
                    w.writeheader()
                w.writerow(s)
        return s
