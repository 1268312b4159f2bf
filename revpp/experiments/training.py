"""Training experiment (BERT/experiment/training/main.py:4-11): evaluate, then train and
evaluate each epoch.  The reference's loop runs epochs 1..num_epochs-1, so ``--num-epochs 1``
trains nothing; that behaviour is kept only under ``--ref-compat``."""
from __future__ import annotations

from .base import Experiment


class TrainingExperiment(Experiment):
    def run(self) -> None:
        eng = self.engine
        eng.step(self.start_epoch, is_train=False)
        if self.cfg.ref_compat:
            epochs = range(self.start_epoch + 1, self.start_epoch + self.cfg.num_epochs)
        else:
            epochs = range(self.start_epoch + 1, self.start_epoch + self.cfg.num_epochs + 1)
        for ep in epochs:
            eng.step(ep, is_train=True)
            eng.step(ep, is_train=False)
