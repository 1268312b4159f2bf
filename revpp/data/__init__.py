"""Datasets and loaders (BERT/src/dataset_factory.py, dataset_registry.py, dataloader.py;
Vit/src/dataset_factory.py).

* ``synthetic`` - the benchmark data: BERT token ids uniform in [0, vocab), an all-ones
  attention mask, Bernoulli(0.5) labels; ViT pixels i.i.d. N(0, 1), labels uniform in
  [0, classes).  Batches are generated from (seed, batch index) so every run sees the
  same data, into pinned host memory.
* ``imdb`` / ``debug`` (BERT) and ``cifar10`` / ``cifar100`` / ``cinic10`` / ``imagenet`` (ViT)
  read pre-staged copies under ``--dataset-dir`` (no network).  The vocabulary size and
  token-type count are fixed to bert-base-uncased's (30522, 2) instead of being fetched.

In pipeline mode only the first stage of each pipeline loads data, with local batch =
global batch / replicas; the batch count is broadcast so every stage runs the same
number of steps (dataloader.py:100-105).
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Callable, Dict, Iterator, List, Optional

import torch
import torch.distributed as dist

from revpp.config import GlobalConfig, ParMode


@dataclass
class DatasetSpec:
    name: str
    kind: str  # "text" | "image"
    num_classes: int
    vocab_size: int = 30522
    type_vocab_size: int = 2


REGISTRY: Dict[str, DatasetSpec] = {
    "synthetic": DatasetSpec("synthetic", "any", 0),
    "imdb": DatasetSpec("imdb", "text", 2),
    "debug": DatasetSpec("debug", "text", 2),
    "cifar10": DatasetSpec("cifar10", "image", 10),
    "cifar100": DatasetSpec("cifar100", "image", 100),
    "cinic10": DatasetSpec("cinic10", "image", 10),
    "imagenet": DatasetSpec("imagenet", "image", 1000),
}


class SyntheticBatches:
    """Deterministic synthetic batches of the configured shape (pinned host tensors)."""

    def __init__(self, cfg: GlobalConfig, batch_size: int, num_batches: int, seed: int, split: str = "train"):
        self.cfg = cfg
        self.batch_size = batch_size
        self.num_batches = num_batches
        self.seed = seed + (0 if split == "train" else 7919)
        self.pin = torch.cuda.is_available()

    def __len__(self) -> int:
        return self.num_batches

    def make(self, i: int) -> dict:
        cfg = self.cfg
        g = torch.Generator().manual_seed(self.seed * 1000003 + i)
        B = self.batch_size
        if cfg.model == "bert":
            S = cfg.max_position_embeddings
            batch = {
                "input_ids": torch.randint(0, cfg.vocab_size, (B, S), generator=g, dtype=torch.int64),
                "attention_mask": torch.ones(B, S, dtype=torch.int64),
                "labels": torch.bernoulli(torch.full((B,), 0.5), generator=g).to(torch.int64),
            }
        else:
            batch = {
                "images": torch.randn(B, cfg.num_channels, cfg.img_size, cfg.img_size, generator=g),
                "labels": torch.randint(0, cfg.num_classes, (B,), generator=g, dtype=torch.int64),
            }
        if self.pin:
            batch = {k: v.pin_memory() for k, v in batch.items()}
        return batch

    def __iter__(self) -> Iterator[dict]:
        for i in range(self.num_batches):
            yield self.make(i)


class TensorBatches:
    """Batches drawn from in-memory tensors (pre-staged real datasets)."""

    def __init__(self, tensors: Dict[str, torch.Tensor], batch_size: int, shuffle: bool, seed: int,
                 drop_last: bool = True):
        self.t = tensors
        self.batch_size = batch_size
        self.shuffle = shuffle
        self.seed = seed
        self.epoch = 0
        n = next(iter(tensors.values())).shape[0]
        self.n = n
        self.num_batches = n // batch_size if drop_last else (n + batch_size - 1) // batch_size

    def __len__(self) -> int:
        return self.num_batches

    def set_epoch(self, e: int) -> None:
        self.epoch = e

    def __iter__(self):
        idx = torch.randperm(self.n, generator=torch.Generator().manual_seed(self.seed + self.epoch)) \
            if self.shuffle else torch.arange(self.n)
        for b in range(self.num_batches):
            sel = idx[b * self.batch_size:(b + 1) * self.batch_size]
            yield {k: v[sel] for k, v in self.t.items()}


# ------------------------------------------------------------------ pre-staged real datasets
def _load_imdb(cfg: GlobalConfig, split: str) -> Dict[str, torch.Tensor]:
    root = cfg.dataset_rdir / "imdb_tokenized"
    f = root / f"{split}.pt"
    if not f.exists():
        raise FileNotFoundError(
            f"IMDb needs a pre-tokenized copy at {f} (dict of input_ids / attention_mask / labels tensors); "
            "there is no network access to download it.  Use --dataset synthetic for benchmarks.")
    return torch.load(f)


_DEBUG_SENTENCES = [
    "this movie was great", "terrible plot and acting", "i loved every minute", "a waste of time",
    "brilliant performances all round", "boring and predictable", "an instant classic", "i fell asleep",
    "the soundtrack was wonderful", "worst film of the year",
]


def _load_debug(cfg: GlobalConfig, split: str) -> Dict[str, torch.Tensor]:
    """Tiny sentiment set tokenised with a hash vocabulary (no tokenizer download)."""
    S = cfg.max_position_embeddings
    ids, labels = [], []
    for i, s in enumerate(_DEBUG_SENTENCES * 3):
        toks = [101] + [1000 + (hash(w) % (cfg.vocab_size - 1000)) for w in s.split()][: S - 2] + [102]
        toks = toks + [0] * (S - len(toks))
        ids.append(toks)
        labels.append(i % 2)
    ids_t = torch.tensor(ids, dtype=torch.int64)
    return {"input_ids": ids_t, "attention_mask": (ids_t != 0).to(torch.int64),
            "labels": torch.tensor(labels, dtype=torch.int64)}


def _load_cifar(cfg: GlobalConfig, split: str, name: str) -> Dict[str, torch.Tensor]:
    import pickle

    import numpy as np

    root = cfg.dataset_rdir / {"cifar10": "cifar-10-batches-py", "cifar100": "cifar-100-python"}[name]
    if not root.exists():
        raise FileNotFoundError(f"{name} needs the python-pickle release under {root} (no network access)")
    files = ([f"data_batch_{i}" for i in range(1, 6)] if split == "train" else ["test_batch"]) \
        if name == "cifar10" else (["train"] if split == "train" else ["test"])
    xs, ys = [], []
    for fn in files:
        with open(root / fn, "rb") as fh:
            d = pickle.load(fh, encoding="latin1")
        xs.append(np.asarray(d["data"], dtype=np.uint8).reshape(-1, 3, 32, 32))
        ys.extend(d["labels"] if "labels" in d else d["fine_labels"])
    x = torch.from_numpy(np.concatenate(xs)).float().div_(255.0)
    mean = torch.tensor([0.4914, 0.4822, 0.4465]).view(1, 3, 1, 1)
    std = torch.tensor([0.2470, 0.2435, 0.2616]).view(1, 3, 1, 1)
    x = (x - mean) / std
    if cfg.img_size != 32 and name == "cifar10":
        # the reference resizes CIFAR-10 to 224 (Vit/src/dataset_factory.py:31-57)
        x = torch.nn.functional.interpolate(x, size=(cfg.img_size, cfg.img_size), mode="bilinear",
                                            align_corners=False)
    return {"images": x, "labels": torch.tensor(ys, dtype=torch.int64)}


def load_split(cfg: GlobalConfig, split: str) -> Dict[str, torch.Tensor]:
    if cfg.dataset == "imdb":
        return _load_imdb(cfg, split)
    if cfg.dataset == "debug":
        return _load_debug(cfg, split)
    if cfg.dataset in ("cifar10", "cifar100"):
        return _load_cifar(cfg, split, cfg.dataset)
    raise FileNotFoundError(f"dataset {cfg.dataset} has no offline copy in {cfg.dataset_rdir}")


@dataclass
class LoaderBundle:
    train_loader: Optional[object]
    val_loader: Optional[object]
    num_batches_train: int
    num_batches_val: int
    local_batch: int


def build_loaders(cfg: GlobalConfig, rank: int, world: int, num_stages: int, device: torch.device,
                  loads_data: bool) -> LoaderBundle:
    replicas = max(1, world // max(1, num_stages)) if cfg.par_mode == ParMode.PP else max(1, world)
    if cfg.batch_size % replicas != 0:
        raise ValueError(f"batch_size {cfg.batch_size} not divisible by {replicas} data-parallel replicas")
    local_batch = cfg.batch_size // replicas
    seed = cfg.seed + (rank // max(1, num_stages) if cfg.par_mode == ParMode.PP else rank)
    train = val = None
    nt = nv = 0
    if loads_data:
        if cfg.dataset == "synthetic":
            nb = cfg.synthetic_batches if not cfg.debug_subset else min(2, cfg.synthetic_batches)
            train = SyntheticBatches(cfg, local_batch, nb, seed, "train")
            val = SyntheticBatches(cfg, local_batch, max(1, nb // 4), seed, "val")
        else:
            tr = load_split(cfg, "train")
            va = load_split(cfg, "test")
            if cfg.debug_subset:
                tr = {k: v[: 8 * local_batch] for k, v in tr.items()}
                va = {k: v[: 2 * local_batch] for k, v in va.items()}
            train = TensorBatches(tr, local_batch, True, seed)
            val = TensorBatches(va, local_batch, False, seed)
        nt, nv = len(train), len(val)
    if dist.is_initialized() and cfg.par_mode == ParMode.PP:
        t = torch.tensor([nt, nv], dtype=torch.int64, device=device)
        # every pipeline's first stage holds the counts and the replicas agree by construction,
        # so global rank 0 (the first stage of replica 0) speaks for all of them
        dist.broadcast(t, src=0)
        nt, nv = int(t[0]), int(t[1])
    return LoaderBundle(train, val, nt, nv, local_batch)
