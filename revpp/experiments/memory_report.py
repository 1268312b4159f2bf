"""Peak-memory breakdowns for ``timeline_peak_stats.json``.

* ``profiler_peak_breakdown`` follows the reference's report
  (BERT/experiment/profiling/_plot.py:62-90): read the torch memory timeline export
  (timestamps, bytes per category in the profiler's category order, constants.py:3), find
  the time of the largest total over the plotted categories and report each category's
  bytes there.
* ``framework_breakdown`` is this framework's own accounting of one rank's device memory:
  the flat buffers it owns (fp32 parameters and bf16 shadow, Adam moments, fp32
  gradients), the stage-to-stage receive buffers, the kernels' reusable scratch, and the
  rest of the allocator's peak (activations and temporaries of the step).  The torch
  profiler cannot attribute the flat buffers or the kernels' outputs to categories, so this
  is the breakdown that says where the memory goes.
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Dict, Optional, Sequence

# category order of torch's memory timeline export (the reference's BASE_CATS)
BASE_CATS = ["CATEGORY_0", "PARAMETER", "OPTIMIZER_STATE", "INPUT", "TEMPORARY", "ACTIVATION", "GRADIENT",
             "AUTOGRAD_DETAIL", "Unknown"]
DEFAULT_ORDER = ["PARAMETER", "OPTIMIZER_STATE", "INPUT", "GRADIENT", "AUTOGRAD_DETAIL", "ACTIVATION", "TEMPORARY",
                 "Unknown"]
GIB = float(1 << 30)


def profiler_peak_breakdown(json_path: Path, order: Optional[Sequence[str]] = None) -> Optional[dict]:
    """Peak of the memory timeline and its per-category split (GiB), or None without data."""
    try:
        with open(json_path) as fh:
            timestamps, sizes = json.load(fh)
    except (OSError, ValueError):
        return None
    if not timestamps:
        return None
    order = list(order or DEFAULT_ORDER)
    idx = [BASE_CATS.index(c) for c in order if c in BASE_CATS]
    best, best_i = -1.0, 0
    for i, row in enumerate(sizes):
        tot = sum(row[j] for j in idx if j < len(row))
        if tot > best:
            best, best_i = tot, i
    row = sizes[best_i]
    return {
        "peak_total_gib": best / GIB,
        "timestamp_ms": (timestamps[best_i] - timestamps[0]) / 1e3,
        "profiler_peak_breakdown_gib": {BASE_CATS[j]: row[j] / GIB for j in idx if j < len(row) and row[j] > 0},
    }


def _bytes(t) -> int:
    return 0 if t is None else t.numel() * t.element_size()


def framework_breakdown(trainer, peak_allocated: int) -> Dict[str, float]:
    """Where one rank's peak device memory goes (GiB), from the framework's own buffers."""
    f = trainer.flat
    parts = {
        "PARAMETER": _bytes(f.data) + _bytes(f.shadow),
        "OPTIMIZER_STATE": _bytes(f.exp_avg) + _bytes(f.exp_avg_sq),
        "GRADIENT": _bytes(f.grad),
    }
    inp = 0
    if getattr(trainer, "channels", None) is not None:
        for ch in trainer.channels.mine.values():
            inp += _bytes(getattr(ch, "buf", None)) if ch.is_receiver else 0
    comms = getattr(trainer, "comms", None)
    if comms is not None:
        for ring in (comms.fwd_ring, comms.bwd_ring):
            if ring is not None and ring._slots is not None:
                inp += sum(_bytes(t) for slot in ring._slots for t in slot)
    parts["INPUT"] = inp
    scratch = getattr(trainer.math, "_scratch", None)
    parts["TEMPORARY"] = sum(_bytes(t) for t in scratch.values()) if scratch else 0
    accounted = sum(parts.values())
    parts["ACTIVATION"] = max(0, int(peak_allocated) - accounted)
    return {k: v / GIB for k, v in parts.items()}


__all__ = ["BASE_CATS", "DEFAULT_ORDER", "profiler_peak_breakdown", "framework_breakdown"]
