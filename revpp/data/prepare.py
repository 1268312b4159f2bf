"""Stage datasets under a dataset directory in the layouts ``revpp.data`` reads
(the counterpart of BERT/scripts/prepare_dataset.py and Vit/scripts/prepare_dataset.py).

    python -m revpp.data.prepare --outdir /dataset --dataset imdb [--tokenizer bert-base-uncased]
    python -m revpp.data.prepare --outdir /dataset --dataset cifar-10
    python -m revpp.data.prepare --outdir /dataset --dataset cifar-100
    python -m revpp.data.prepare --outdir /dataset --dataset cinic10     # checks a copied layout
    python -m revpp.data.prepare --outdir /dataset --dataset imagenet    # checks a copied layout

imdb: saves the tokenizer (tokenizer/) and the raw dataset (imdb_raw/, HF save_to_disk) when
the hub is reachable; with both present (downloaded here or copied from elsewhere) it also
writes the tokenised tensors (imdb_tokenized/{train,test}.pt at --max-length) that training
loads directly.  CIFAR downloads through torchvision when the network allows.  CINIC-10 and
ImageNet have no downloader (as in the reference): the script checks the copied ImageFolder
layout and reports its class and image counts.
"""
from __future__ import annotations

import argparse
import os
from pathlib import Path


def _imdb(out: Path, tokenizer: str, max_length: int, download: bool) -> None:
    tok_dir, raw_dir = out / "tokenizer", out / "imdb_raw"
    if download and not tok_dir.exists():
        from transformers import BertTokenizer

        BertTokenizer.from_pretrained(tokenizer).save_pretrained(str(tok_dir))
    if download and not raw_dir.exists():
        from datasets import load_dataset

        load_dataset("imdb").save_to_disk(str(raw_dir))
    if not tok_dir.exists() or not (raw_dir.exists() or (out / "aclImdb").exists()):
        raise SystemExit(f"{out} needs tokenizer/ and imdb_raw/ (or aclImdb/); run with network access or copy them")
    from revpp.data import _imdb_texts, _tokenize

    dst = out / "imdb_tokenized"
    dst.mkdir(parents=True, exist_ok=True)
    import torch

    for split in ("train", "test"):
        texts, labels = _imdb_texts(out, split)
        d = _tokenize(texts, labels, tok_dir, max_length)
        torch.save(d, dst / f"{split}.pt")
        print(f"imdb {split}: {len(labels)} reviews -> {dst / (split + '.pt')} (max_length {max_length})")


def _cifar(out: Path, name: str) -> None:
    from torchvision import datasets

    root = out / name
    root.mkdir(parents=True, exist_ok=True)
    cls = datasets.CIFAR10 if name == "cifar-10" else datasets.CIFAR100
    for train in (True, False):
        ds = cls(root=str(root), train=train, download=True)
        print(f"{name} {'train' if train else 'test'}: {len(ds)} images under {root}")


def _image_folder(out: Path, name: str) -> None:
    sub = {"cinic10": ("CINIC-10", ("train", "valid", "test")), "imagenet": ("ImageNet-1K", ("train", "val"))}[name]
    base = out / sub[0]
    found = False
    for split in sub[1]:
        d = base / split
        if not d.exists():
            continue
        found = True
        classes = sorted(p for p in d.iterdir() if p.is_dir())
        n = sum(1 for c in classes for f in c.iterdir() if f.is_file())
        print(f"{name} {split}: {len(classes)} classes, {n} images under {d}")
    if not found:
        raise SystemExit(f"copy the {name} ImageFolder layout to {base}/<split>/<class>/<image> first")


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--outdir", required=True)
    p.add_argument("--dataset", choices=["imdb", "cifar-10", "cifar-100", "cinic10", "imagenet"], default="imdb")
    p.add_argument("--tokenizer", default="bert-base-uncased")
    p.add_argument("--max-length", type=int, default=512)
    p.add_argument("--no-download", action="store_true", help="only convert what is already there")
    a = p.parse_args(argv)
    out = Path(a.outdir)
    os.makedirs(out, exist_ok=True)
    if a.dataset == "imdb":
        _imdb(out, a.tokenizer, a.max_length, not a.no_download)
    elif a.dataset in ("cifar-10", "cifar-100"):
        _cifar(out, a.dataset)
    else:
        _image_folder(out, a.dataset)


if __name__ == "__main__":
    main()
