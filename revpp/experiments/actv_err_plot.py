"""Per-stage boxplots of the reconstruction error (BERT/experiment/actv_err/plot.py:25-91).
Needs matplotlib, which is optional."""
from __future__ import annotations

import csv
from pathlib import Path


def boxplot(out_dir: Path, num_stages: int) -> None:
    import matplotlib

    matplotlib.use("Agg")
    import matplotlib.pyplot as plt

    data, labels = [], []
    for s in range(num_stages):
        p = Path(out_dir) / f"actv_err_{s}.csv"
        if not p.exists():
            continue
        with open(p) as fh:
            rows = list(csv.DictReader(fh))
        if rows:
            data.append([float(r["mse"]) for r in rows])
            labels.append(f"stage {s}")
    if not data:
        return
    fig, ax = plt.subplots(figsize=(6, 4))
    ax.boxplot(data, labels=labels)
    ax.set_yscale("log")
    ax.set_ylabel("reconstruction MSE")
    fig.tight_layout()
    fig.savefig(Path(out_dir) / "actv_err.png")
    fig.savefig(Path(out_dir) / "actv_err.pdf")
    plt.close(fig)
