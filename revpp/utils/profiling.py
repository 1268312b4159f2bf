"""Trace annotations and device timers.

``annotate(name)`` marks a host range for torch.profiler (``record_function``) and NVTX,
with the reference's ``## name ##`` vocabulary (BERT/src/engine.py:129-270,
reversible_stage_with_pareprop.py:418,479) so traces stay comparable.

``DeviceTimer`` times a region with CUDA events on the current stream; ``max_over_ranks``
reduces a measured time to the slowest rank (multi-GPU numbers are the max over ranks).
"""
from __future__ import annotations

import contextlib
import os

import torch
import torch.distributed as dist

_ENABLED = os.environ.get("REVPP_ANNOTATE", "1") != "0"


@contextlib.contextmanager
def annotate(name: str):
    if not _ENABLED:
        yield
        return
    with torch.profiler.record_function(name):
        if torch.cuda.is_available() and torch.cuda.is_initialized():
            torch.cuda.nvtx.range_push(name)
            try:
                yield
            finally:
                torch.cuda.nvtx.range_pop()
        else:
            yield


class DeviceTimer:
    """Elapsed milliseconds between ``start()`` and ``stop()`` measured on the device."""

    def __init__(self, device: torch.device):
        self.cuda = device.type == "cuda"
        self.t0 = self.t1 = None
        if self.cuda:
            self.e0 = torch.cuda.Event(enable_timing=True)
            self.e1 = torch.cuda.Event(enable_timing=True)

    def start(self) -> None:
        if self.cuda:
            torch.cuda.synchronize()
            self.e0.record()
        else:
            import time

            self.t0 = time.perf_counter()

    def stop(self) -> float:
        if self.cuda:
            self.e1.record()
            torch.cuda.synchronize()
            return float(self.e0.elapsed_time(self.e1))
        import time

        return (time.perf_counter() - self.t0) * 1e3


def max_over_ranks(value: float, device: torch.device, group=None) -> float:
    if not (dist.is_available() and dist.is_initialized()):
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
