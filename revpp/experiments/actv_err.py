"""Activation-error experiment (BERT/experiment/actv_err/main.py:11-124).

Needs ``--par-mode pp --reversible``.  Runs one training step with reconstruction checks
on: each middle stage compares the input it reconstructs in backward with the input it
received in forward (per-sample MSE and cosine similarity in fp64) and writes
``actv_err_{stage}.csv``; rank 0 then writes a per-stage summary.  (The reference calls
dist.barrier() after destroying the process group, actv_err/main.py:31,57; here the
barrier comes first.)
"""
from __future__ import annotations

import csv
import json
import statistics

import torch.distributed as dist

from revpp.config import ParMode

from .base import Experiment


class ActvErrExperiment(Experiment):
    eval_actv_err = True

    def __init__(self, cfg, env):
        if cfg.par_mode != ParMode.PP or not cfg.reversible:
            raise ValueError("actv-err needs --par-mode pp --reversible")
        super().__init__(cfg, env)

    def run(self) -> None:
        cfg, env, t = self.cfg, self.env, self.trainer
        self.engine.step(0, is_train=True, batch_limit=1)
        out_dir = cfg.log_rdir / cfg.exp_id / cfg.env_id
        out_dir.mkdir(parents=True, exist_ok=True)
        recs = t.stage.actv_records
        path = out_dir / f"actv_err_{t.stage_index}.csv"
        with open(path, "w", newline="") as fh:
            w = csv.DictWriter(fh, fieldnames=["stage", "mb", "sample", "tensor", "mse", "cos"])
            w.writeheader()
            w.writerows(recs)
        if dist.is_initialized():
            dist.barrier()
        if env.rank == 0:
            summary = {}
            for s in range(t.P):
                p = out_dir / f"actv_err_{s}.csv"
                if not p.exists():
                    continue
                with open(p) as fh:
                    rows = list(csv.DictReader(fh))
                if not rows:
                    continue
                mse = [float(r["mse"]) for r in rows]
                cos = [float(r["cos"]) for r in rows]
                summary[s] = {"n": len(rows), "mse_median": statistics.median(mse), "mse_max": max(mse),
                              "cos_min": min(cos), "cos_median": statistics.median(cos)}
            (out_dir / "actv_err_summary.json").write_text(json.dumps(summary, indent=2))
            try:
                import matplotlib  # noqa: F401  (optional: the boxplot needs matplotlib)

                from .actv_err_plot import boxplot

                boxplot(out_dir, t.P)
            except ImportError:
                pass
