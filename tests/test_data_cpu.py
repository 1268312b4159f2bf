"""Dataset loaders on small on-disk fixtures (no network): IMDb from aclImdb text folders and
from an HF ``save_to_disk`` copy with a local BERT tokenizer, the tokenised cache, the prepare
script, and the CINIC-10 / ImageNet ImageFolder layouts with the reference's transforms."""

import pytest
import torch

from revpp.config import build_global_config, parse_args


def _tokenizer_dir(path):
    from transformers import BertTokenizerFast

    words = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]", "great", "movie", "bad", "film", "this", "was", "a",
             "boring", "loved", "it"]
    path.mkdir(parents=True, exist_ok=True)
    (path / "vocab.txt").write_text("\n".join(words) + "\n")
    BertTokenizerFast(vocab_file=str(path / "vocab.txt")).save_pretrained(str(path))
    return path


def _cfg(tmp_path, extra):
    args = parse_args((f"--dataset-dir {tmp_path} --device cpu --batch-size 4 --microbatch-size 2 "
                       f"--num-microbatches 2 " + extra).split())
    return build_global_config(args)


def test_imdb_from_acl_text_folders_and_cache(tmp_path):
    from revpp.data import _load_imdb

    _tokenizer_dir(tmp_path / "tokenizer")
    for split in ("train", "test"):
        for sub, text in (("pos", "this movie was great"), ("neg", "a boring bad film")):
            d = tmp_path / "aclImdb" / split / sub
            d.mkdir(parents=True)
            for i in range(3):
                (d / f"{i}.txt").write_text(text)
    cfg = _cfg(tmp_path, "--dataset imdb --preset tiny-bert --max-position-embeddings 16")
    d = _load_imdb(cfg, "train")
    assert d["input_ids"].shape == (6, 16)
    assert d["labels"].tolist() == [0, 0, 0, 1, 1, 1]
    assert int(d["input_ids"][0, 0]) == 2  # [CLS]
    assert d["attention_mask"].sum(1).tolist()[0] == 6  # [CLS] a boring bad film [SEP]
    assert (tmp_path / "imdb_tokenized" / "train.pt").exists()
    again = _load_imdb(cfg, "train")  # from the cache
    assert torch.equal(again["input_ids"], d["input_ids"])


def test_imdb_from_hf_save_to_disk_and_prepare_script(tmp_path):
    from datasets import Dataset, DatasetDict

    from revpp.data import _load_imdb
    from revpp.data.prepare import main as prepare

    _tokenizer_dir(tmp_path / "tokenizer")
    dd = DatasetDict({s: Dataset.from_dict({"text": ["loved it", "bad movie", "great film"], "label": [1, 0, 1]})
                      for s in ("train", "test")})
    dd.save_to_disk(str(tmp_path / "imdb_raw"))
    cfg = _cfg(tmp_path, "--dataset imdb --preset tiny-bert --max-position-embeddings 8")
    d = _load_imdb(cfg, "test")
    assert d["input_ids"].shape == (3, 8) and d["labels"].tolist() == [1, 0, 1]
    prepare(["--outdir", str(tmp_path), "--dataset", "imdb", "--no-download", "--max-length", "8"])
    cached = torch.load(tmp_path / "imdb_tokenized" / "train.pt")
    assert cached["input_ids"].shape == (3, 8)


def _image_folder(root, classes, n, size, ext):
    from PIL import Image

    for c in classes:
        d = root / c
        d.mkdir(parents=True)
        for i in range(n):
            Image.new("RGB", (size, size), color=(10 * i, 50, 200)).save(d / f"{i}.{ext}")


@pytest.mark.parametrize("name,sub,size,ext,img", [
    ("cinic10", ("CINIC-10", "train", "valid"), 32, "png", 32),
    ("imagenet", ("ImageNet-1K", "train", "val"), 300, "JPEG", 224),
])
def test_image_folder_datasets(tmp_path, name, sub, size, ext, img):
    from revpp.config import ParMode
    from revpp.data import build_loaders

    for split in sub[1:]:
        _image_folder(tmp_path / sub[0] / split, ["a", "b"], 4, size, ext)
    extra = f"--dataset {name} --model vit --img-size {img} --patch-size 16 --num-classes 2"
    cfg = _cfg(tmp_path, extra)
    cfg = cfg.__class__(**{**cfg.__dict__, "num_workers": 0, "par_mode": ParMode.NONE})
    lb = build_loaders(cfg, rank=0, world=1, num_stages=1, device=torch.device("cpu"), loads_data=True)
    assert lb.num_batches_train == 2 and lb.num_batches_val == 2
    b = next(iter(lb.train_loader))
    assert b["images"].shape == (4, 3, img, img) and b["labels"].shape == (4,)
    assert set(b["labels"].tolist()) <= {0, 1}


def test_prepare_checks_image_folder_layout(tmp_path, capsys):
    from revpp.data.prepare import main as prepare

    _image_folder(tmp_path / "CINIC-10" / "train", ["cat", "dog"], 3, 32, "png")
    prepare(["--outdir", str(tmp_path), "--dataset", "cinic10"])
    assert "2 classes, 6 images" in capsys.readouterr().out
    with pytest.raises(SystemExit):
        prepare(["--outdir", str(tmp_path / "none"), "--dataset", "imagenet"])


