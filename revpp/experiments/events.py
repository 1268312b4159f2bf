"""Annotation vocabulary and Chrome-trace span parsing (BERT/experiment/profiling/constants.py,
events.py:1-89).

Spans are the host ranges opened with ``revpp.utils.profiling.annotate("## name ##")``;
``parse_event_spans`` reads them back from a torch.profiler Chrome trace ("X" complete
events and "B"/"E" pairs of category user_annotation) as zero-based milliseconds.
"""
from __future__ import annotations

import json
import re
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, List

# memory categories of torch's memory profiler, in plotting order
BASE_CATS = ["PARAMETER", "OPTIMIZER_STATE", "INPUT", "TEMPORARY", "ACTIVATION", "GRADIENT", "AUTOGRAD_DETAIL",
             "UNKNOWN"]
DEFAULT_ORDER = BASE_CATS

EVENT_SPECS = {
    "dataload": re.compile(r"^## dataload ##$"),
    "send_labels": re.compile(r"^## send_labels ##$"),
    "recv_labels": re.compile(r"^## recv_labels ##$"),
    "pipeline_step": re.compile(r"^## pipeline_step ##$"),
    "forward_one_chunk": re.compile(r"^## forward_one_chunk ##$"),
    "backward_one_chunk": re.compile(r"^## backward_one_chunk ##$"),
    "dp_allreduce": re.compile(r"^## dp_allreduce ##$"),
    "clip_grad": re.compile(r"^## clip_grad ##$"),
    "optimize": re.compile(r"^## optimize ##$"),
    "step": re.compile(r"^## step \d+ ##$"),
}


@dataclass
class EventSpan:
    label: str
    name: str
    start_ms: float
    end_ms: float

    @property
    def duration_ms(self) -> float:
        return self.end_ms - self.start_ms


def parse_event_spans(trace_path: Path | str) -> List[EventSpan]:
    with open(trace_path) as fh:
        data = json.load(fh)
    events = data["traceEvents"] if isinstance(data, dict) else data
    raw = []
    open_b: Dict[tuple, float] = {}
    for ev in events:
        if ev.get("cat") not in ("user_annotation", "gpu_user_annotation"):
            continue
        if ev.get("cat") == "gpu_user_annotation":
            continue
        name = ev.get("name", "")
        ph = ev.get("ph")
        if ph == "X":
            raw.append((name, float(ev["ts"]), float(ev["ts"]) + float(ev.get("dur", 0.0))))
        elif ph == "B":
            open_b[(name, ev.get("tid"))] = float(ev["ts"])
        elif ph == "E":
            key = (name, ev.get("tid"))
            if key in open_b:
                raw.append((name, open_b.pop(key), float(ev["ts"])))
    if not raw:
        return []
    t0 = min(s for _, s, _ in raw)
    spans = []
    for name, s, e in raw:
        for label, rx in EVENT_SPECS.items():
            if rx.match(name):
                spans.append(EventSpan(label, name, (s - t0) / 1e3, (e - t0) / 1e3))
                break
    spans.sort(key=lambda sp: sp.start_ms)
    return spans


def span_stats(spans: List[EventSpan]) -> Dict[str, dict]:
    out: Dict[str, dict] = {}
    for sp in spans:
        d = out.setdefault(sp.label, {"count": 0, "total_ms": 0.0, "max_ms": 0.0})
        d["count"] += 1
        d["total_ms"] += sp.duration_ms
        d["max_ms"] = max(d["max_ms"], sp.duration_ms)
    for d in out.values():
        d["mean_ms"] = d["total_ms"] / max(d["count"], 1)
    return out
