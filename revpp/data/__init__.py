"""Datasets and loaders (BERT/src/dataset_factory.py, dataset_registry.py, dataloader.py;
Vit/src/dataset_factory.py).

* ``synthetic`` - the benchmark data: BERT token ids uniform in [0, vocab), an all-ones
  attention mask, Bernoulli(0.5) labels; ViT pixels i.i.d. N(0, 1), labels uniform in
  [0, classes).  Batches are generated from (seed, batch index) so every run sees the
  same data, into pinned host memory.
* ``imdb`` / ``debug`` (BERT) read a raw or tokenised copy under ``--dataset-dir`` and
  tokenise with a local BERT tokenizer directory; ``cifar10`` / ``cifar100`` / ``cinic10`` /
  ``imagenet`` (ViT) read the reference's on-disk layouts through torchvision with the
  reference's transforms (no network).  The vocabulary size and token-type count are fixed
  to bert-base-uncased's (30522, 2) instead of being fetched.

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
def _tokenize(texts: List[str], labels: List[int], tokenizer_dir: Path, max_length: int) -> Dict[str, torch.Tensor]:
    """BERT word-piece tokenisation with the reference's settings (special tokens, padding
    and truncation to max_length; BERT/src/dataset_factory.py:44-67), from a local tokenizer
    directory (no download)."""
    from transformers import BertTokenizerFast

    tok = BertTokenizerFast.from_pretrained(str(tokenizer_dir))
    enc = tok(texts, add_special_tokens=True, max_length=max_length, padding="max_length", truncation=True,
              return_tensors="pt")
    return {"input_ids": enc["input_ids"].to(torch.int64), "attention_mask": enc["attention_mask"].to(torch.int64),
            "labels": torch.tensor(labels, dtype=torch.int64)}


def _imdb_texts(root: Path, split: str):
    """(texts, labels) of an IMDb split from a raw copy: the HF ``save_to_disk`` layout the
    reference's prepare script writes (imdb_raw/), or the original aclImdb text folders."""
    raw = root / "imdb_raw"
    if raw.exists():
        from datasets import load_from_disk

        d = load_from_disk(str(raw))[split]
        return list(d["text"]), [int(x) for x in d["label"]]
    acl = root / "aclImdb" / split
    if acl.exists():
        texts, labels = [], []
        for lab, sub in ((0, "neg"), (1, "pos")):
            for f in sorted((acl / sub).glob("*.txt")):
                texts.append(f.read_text(encoding="utf-8", errors="replace"))
                labels.append(lab)
        return texts, labels
    return None


def _load_imdb(cfg: GlobalConfig, split: str) -> Dict[str, torch.Tensor]:
    """IMDb, in this order: a tokenised tensor cache (imdb_tokenized/{split}.pt), else the raw
    text (imdb_raw/ or aclImdb/) tokenised with the local tokenizer/ directory (written to the
    cache when the directory is writable)."""
    root = cfg.dataset_rdir
    S = cfg.max_position_embeddings
    cache = root / "imdb_tokenized" / f"{split}.pt"
    if cache.exists():
        d = torch.load(cache)
        if d["input_ids"].shape[1] == S:
            return d
    raw = _imdb_texts(root, split)
    tok_dir = root / "tokenizer"
    if raw is None or not tok_dir.exists():
        raise FileNotFoundError(
            f"IMDb needs {cache}, or a raw copy ({root / 'imdb_raw'} or {root / 'aclImdb'}) and a BERT tokenizer "
            f"directory {tok_dir}; there is no network access (python -m revpp.data.prepare stages them). "
            "Use --dataset synthetic for benchmarks.")
    d = _tokenize(raw[0], raw[1], tok_dir, S)
    try:
        cache.parent.mkdir(parents=True, exist_ok=True)
        torch.save(d, cache)
    except OSError:
        pass
    return d


_DEBUG_SENTENCES = [
    "this movie was great", "terrible plot and acting", "i loved every minute", "a waste of time",
    "brilliant performances all round", "boring and predictable", "an instant classic", "i fell asleep",
    "the soundtrack was wonderful", "worst film of the year",
]


def _load_debug(cfg: GlobalConfig, split: str) -> Dict[str, torch.Tensor]:
    """Tiny sentiment set (30 sentences, the same for train and validation as in the
    reference's debug set); tokenised with the local tokenizer directory when there is one,
    else with a hash vocabulary."""
    S = cfg.max_position_embeddings
    sents = _DEBUG_SENTENCES * 3
    labels = [i % 2 for i in range(len(sents))]
    tok_dir = cfg.dataset_rdir / "tokenizer"
    if tok_dir.exists():
        return _tokenize(sents, labels, tok_dir, S)
    ids = []
    for s in sents:
        toks = [101] + [1000 + (hash(w) % (cfg.vocab_size - 1000)) for w in s.split()][: S - 2] + [102]
        ids.append(toks + [0] * (S - len(toks)))
    ids_t = torch.tensor(ids, dtype=torch.int64)
    return {"input_ids": ids_t, "attention_mask": (ids_t != 0).to(torch.int64),
            "labels": torch.tensor(labels, dtype=torch.int64)}


def _load_cifar_pickle(cfg: GlobalConfig, split: str, name: str) -> Dict[str, torch.Tensor]:
    """CIFAR from the python-pickle release unpacked directly under the dataset directory."""
    import pickle

    import numpy as np

    root = cfg.dataset_rdir / {"cifar10": "cifar-10-batches-py", "cifar100": "cifar-100-python"}[name]
    files = ([f"data_batch_{i}" for i in range(1, 6)] if split == "train" else ["test_batch"]) \
        if name == "cifar10" else (["train"] if split == "train" else ["test"])
    xs, ys = [], []
    for fn in files:
        with open(root / fn, "rb") as fh:
            d = pickle.load(fh, encoding="latin1")
        xs.append(np.asarray(d["data"], dtype=np.uint8).reshape(-1, 3, 32, 32))
        ys.extend(d["labels"] if "labels" in d else d["fine_labels"])
    x = torch.from_numpy(np.concatenate(xs)).float().div_(255.0)
    mean, std = _NORM[name]
    x = (x - torch.tensor(mean).view(1, 3, 1, 1)) / torch.tensor(std).view(1, 3, 1, 1)
    if cfg.img_size != 32 and name == "cifar10":
        # the reference resizes CIFAR-10 to 224 (Vit/src/dataset_factory.py:31-57)
        x = torch.nn.functional.interpolate(x, size=(cfg.img_size, cfg.img_size), mode="bilinear",
                                            align_corners=False)
    return {"images": x, "labels": torch.tensor(ys, dtype=torch.int64)}


# normalisation constants of the reference's transforms (Vit/src/dataset_factory.py)
_NORM = {
    "cifar10": ([0.4914, 0.4822, 0.4465], [0.2023, 0.1994, 0.2010]),
    "cinic10": ([0.4914, 0.4822, 0.4465], [0.2023, 0.1994, 0.2010]),
    "cifar100": ([0.5071, 0.4865, 0.4409], [0.2673, 0.2564, 0.2761]),
    "imagenet": ([0.485, 0.456, 0.406], [0.229, 0.224, 0.225]),
}


def image_dataset(cfg: GlobalConfig, split: str):
    """A torchvision dataset of (image, label) with the reference's transforms
    (Vit/src/dataset_factory.py:5-109), read from its on-disk layout under --dataset-dir:

      cifar10   cifar-10/  (torchvision CIFAR10 files)   224 x 224: resize, crop pad 4, flip
      cifar100  cifar-100/ (torchvision CIFAR100 files)  32 x 32: crop pad 4, flip
      cinic10   CINIC-10/{train,valid}/<class>/*.png     32 x 32: crop pad 4, flip
      imagenet  ImageNet-1K/{train,val}/<class>/*.JPEG   train: random-resized crop 224 (scale
                0.2-1, bicubic), flip; val: resize 256, centre crop 224
    Returns None when the layout is absent."""
    from torchvision import datasets as tvd
    from torchvision import transforms as T

    name, root, train = cfg.dataset, cfg.dataset_rdir, split == "train"
    norm = T.Normalize(*_NORM[name])
    if name == "cifar10":
        size = cfg.img_size
        tf = T.Compose(([T.Resize((size, size)), T.RandomCrop(size, padding=4), T.RandomHorizontalFlip()] if train
                        else [T.Resize((size, size))]) + [T.ToTensor(), norm])
        d = root / "cifar-10"
        if not (d / "cifar-10-batches-py").exists():
            return None
        return tvd.CIFAR10(str(d), train=train, transform=tf, download=False)
    if name == "cifar100":
        tf = T.Compose(([T.RandomCrop(32, padding=4), T.RandomHorizontalFlip()] if train else []) + [T.ToTensor(), norm])
        d = root / "cifar-100"
        if not (d / "cifar-100-python").exists():
            return None
        return tvd.CIFAR100(str(d), train=train, transform=tf, download=False)
    if name == "cinic10":
        tf = T.Compose(([T.RandomCrop(32, padding=4), T.RandomHorizontalFlip()] if train else []) + [T.ToTensor(), norm])
        d = root / "CINIC-10" / ("train" if train else "valid")
        return tvd.ImageFolder(str(d), tf) if d.exists() else None
    if name == "imagenet":
        size = cfg.img_size
        if train:
            tf = T.Compose([T.RandomResizedCrop(size, scale=(0.2, 1.0), interpolation=T.InterpolationMode.BICUBIC),
                            T.RandomHorizontalFlip(), T.ToTensor(), norm])
        else:
            tf = T.Compose([T.Resize(int(size * 256 / 224)), T.CenterCrop(size), T.ToTensor(), norm])
        d = root / "ImageNet-1K" / ("train" if train else "val")
        return tvd.ImageFolder(str(d), tf) if d.exists() else None
    return None


class ImageBatches:
    """Batches {"images", "labels"} from a torchvision dataset through a DataLoader with
    workers; replicas read disjoint shards (DistributedSampler over the replicas)."""

    def __init__(self, ds, batch_size: int, train: bool, replicas: int, replica: int, seed: int, workers: int):
        from torch.utils.data import DataLoader, DistributedSampler

        self.sampler = DistributedSampler(ds, num_replicas=replicas, rank=replica, shuffle=train, seed=seed,
                                          drop_last=True)
        self.loader = DataLoader(ds, batch_size=batch_size, sampler=self.sampler, num_workers=workers,
                                 pin_memory=torch.cuda.is_available(), drop_last=True,
                                 persistent_workers=workers > 0)

    def __len__(self) -> int:
        return len(self.loader)

    def set_epoch(self, e: int) -> None:
        self.sampler.set_epoch(e)

    def __iter__(self):
        for x, y in self.loader:
            yield {"images": x, "labels": y}


def load_split(cfg: GlobalConfig, split: str) -> Dict[str, torch.Tensor]:
    """In-memory tensors of a split (text datasets and CIFAR from the pickle release)."""
    if cfg.dataset == "imdb":
        return _load_imdb(cfg, split)
    if cfg.dataset == "debug":
        return _load_debug(cfg, split)
    if cfg.dataset in ("cifar10", "cifar100"):
        pick = cfg.dataset_rdir / {"cifar10": "cifar-10-batches-py", "cifar100": "cifar-100-python"}[cfg.dataset]
        if pick.exists():
            return _load_cifar_pickle(cfg, split, cfg.dataset)
    raise FileNotFoundError(
        f"dataset {cfg.dataset} has no offline copy under {cfg.dataset_rdir} (see revpp.data.image_dataset for "
        "the layouts; python -m revpp.data.prepare stages them)")


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
            replica = rank // max(1, num_stages) if cfg.par_mode == ParMode.PP else rank
            ds_tr = image_dataset(cfg, "train") if REGISTRY[cfg.dataset].kind == "image" else None
            if ds_tr is not None:
                ds_va = image_dataset(cfg, "val")
                if cfg.debug_subset:
                    from torch.utils.data import Subset

                    ds_tr = Subset(ds_tr, range(min(len(ds_tr), 8 * local_batch * replicas)))
                    ds_va = Subset(ds_va, range(min(len(ds_va), 2 * local_batch * replicas)))
                train = ImageBatches(ds_tr, local_batch, True, replicas, replica, cfg.seed, cfg.num_workers)
                val = ImageBatches(ds_va, local_batch, False, replicas, replica, cfg.seed, cfg.num_workers)
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
