"""Experiment registry (BERT/experiment/__init__.py:8-28): training, profiling, actv-err."""
from __future__ import annotations

from typing import Callable, Dict

EXP_REGISTRY: Dict[str, Callable] = {}


def register(name: str):
    def deco(cls):
        EXP_REGISTRY[name] = cls
        return cls

    return deco


def _populate() -> None:
    from .actv_err import ActvErrExperiment
    from .profiling import ProfilingExperiment
    from .training import TrainingExperiment

    register("training")(TrainingExperiment)
    register("profiling")(ProfilingExperiment)
    register("actv-err")(ActvErrExperiment)


_populate()
