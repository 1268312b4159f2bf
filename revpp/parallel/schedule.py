"""Pipeline schedules as explicit per-rank action lists, and their executor.

``one_f_one_b(stage, P, n)`` gives the reference's Schedule1F1B order
(BERT/pipelining/schedules.py:677-852): min(P - s, n) warm-up forwards, then
alternating forward / backward, then the remaining backwards.  ``gpipe`` is all forwards
then all backwards (ScheduleGPipe, schedules.py:591-673); ``forward_only`` is the
evaluation schedule (_ScheduleForwardOnly, schedules.py:538-588).

Labels travel from the first to the last stage once per step, as in the reference engine
(BERT/src/engine.py:174-176, 238-240).
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from .p2p import PipeComms

Action = Tuple[str, int]


def one_f_one_b(stage: int, num_stages: int, n: int) -> List[Action]:
    """1F1B as Schedule1F1B runs it (BERT/pipelining/schedules.py:708-852): min(n, P - s)
    warm-up forwards, then alternate one backward and one forward (1B1F), then the
    remaining backwards."""
    warmup = min(num_stages - stage, n)
    acts: List[Action] = [("F", i) for i in range(warmup)]
    f, b = warmup, 0
    while b < n:
        acts.append(("B", b))
        b += 1
        if f < n:
            acts.append(("F", f))
            f += 1
    return acts


def gpipe(stage: int, num_stages: int, n: int) -> List[Action]:
    return [("F", i) for i in range(n)] + [("B", i) for i in range(n)]


def forward_only(stage: int, num_stages: int, n: int) -> List[Action]:
    return [("F", i) for i in range(n)]


SCHEDULES = {"1f1b": one_f_one_b, "gpipe": gpipe}


def simulate(num_stages: int, n: int, schedule: str = "1f1b", t_f: float = 1.0, t_b: float = 2.0,
             events: list | None = None):
    """Event simulation of a schedule: returns (makespan, per-stage busy time).  Used to
    check schedules without GPUs and to predict bubble fractions.  With ``events`` given,
    every simulated action is appended as (stage, kind, micro-batch, start, end)."""
    fn = SCHEDULES[schedule]
    acts = [fn(s, num_stages, n) for s in range(num_stages)]
    pos = [0] * num_stages
    t = [0.0] * num_stages
    f_done = [[None] * n for _ in range(num_stages)]
    b_done = [[None] * n for _ in range(num_stages)]
    busy = [0.0] * num_stages
    progress = True
    while progress:
        progress = False
        for s in range(num_stages):
            if pos[s] >= len(acts[s]):
                continue
            kind, i = acts[s][pos[s]]
            if kind == "F":
                dep = 0.0 if s == 0 else f_done[s - 1][i]
                if dep is None:
                    continue
                start = max(t[s], dep)
                t[s] = start + t_f
                f_done[s][i] = t[s]
                busy[s] += t_f
                if events is not None:
                    events.append((s, "F", i, start, t[s]))
            else:
                dep = f_done[s][i] if s == num_stages - 1 else b_done[s + 1][i]
                if dep is None or f_done[s][i] is None:
                    continue
                start = max(t[s], dep)
                t[s] = start + t_b
                b_done[s][i] = t[s]
                busy[s] += t_b
                if events is not None:
                    events.append((s, "B", i, start, t[s]))
            pos[s] += 1
            progress = True
    if any(p < len(a) for p, a in zip(pos, acts)):
        raise RuntimeError("schedule deadlocks")
    return max(t), busy


def dump_chrometrace(num_stages: int, n: int, path, schedule: str = "1f1b", t_f: float = 1.0,
                     t_b: float = 2.0) -> float:
    """Write the simulated schedule as a Chrome trace (one row per stage, one slice per
    forward / backward of a micro-batch, times in the units of ``t_f`` / ``t_b`` read as
    milliseconds), the counterpart of the reference's schedule trace dump
    (BERT/pipelining/schedules.py:2585).  Returns the makespan."""
    import json

    events: list = []
    makespan, _ = simulate(num_stages, n, schedule, t_f, t_b, events)
    trace = [{"name": "process_name", "ph": "M", "pid": 0, "args": {"name": f"{schedule} schedule"}}]
    trace += [{"name": "thread_name", "ph": "M", "pid": 0, "tid": s, "args": {"name": f"stage {s}"}}
              for s in range(num_stages)]
    for s, kind, i, start, end in events:
        trace.append({"name": f"{kind}{i}", "cat": "forward" if kind == "F" else "backward", "ph": "X", "pid": 0,
                      "tid": s, "ts": start * 1e3, "dur": (end - start) * 1e3})
    with open(path, "w") as fh:
        json.dump({"traceEvents": trace}, fh)
    return makespan


class PipelineExecutor:
    """Runs a schedule on one rank.  Communication follows the reference's grouping
    (BERT/pipelining/schedules.py:700-852) on a single process group per pipeline:

      warm-up (min(n, P - s) forwards): receive input -> forward -> send output; the last
        warm-up send is held back and grouped with the first backward receive;
      steady state: [forward send + backward receive] -> backward ->
                    [backward send + forward receive] -> forward;
      cool-down: backward receive -> backward -> backward send.

    Waits are stream-level on NCCL.  Receive buffers come from the rings in ``PipeComms``."""

    def __init__(self, stage, comms: Optional[PipeComms], num_microbatches: int, schedule: str = "1f1b"):
        self.stage = stage
        self.comms = comms
        self.n = num_microbatches
        self.schedule = schedule
        self.P = stage.num_stages
        self.s = stage.stage_index

    # ---------------------------------------------------------------- helpers
    def _rank(self) -> int:
        return dist.get_rank() if dist.is_initialized() else 0

    def _recv_fwd(self):
        if self.stage.is_first:
            return [], None
        return self.comms.recv_fwd()

    def _recv_bwd(self):
        if self.stage.is_last:
            return [], None
        return self.comms.recv_bwd()

    def _forward(self, i, meta, inputs, train):
        from .faults import before_forward

        before_forward(self._rank(), i)
        x = inputs[i] if meta is None else meta[2]
        out = self.stage.forward(i, x, train)
        if meta is not None:
            meta[0].release(meta[1])
        return out

    def _backward(self, i, meta):
        g = self.stage.backward(i, None if meta is None else meta[2])
        if meta is not None:
            meta[0].release(meta[1])
        return g

    def _send_fwd(self, out):
        if out is None or self.stage.is_last or self.comms is None:
            return [], []
        return self.comms.send_fwd(out)

    def _send_bwd(self, g):
        if g is None or self.stage.is_first or self.comms is None:
            return [], []
        return self.comms.send_bwd(g)

    def _run(self, ops, keep=()):
        cm = self.comms
        if cm is None or not ops:
            return
        cm.wait(cm.issue(ops, list(keep)))

    # ---------------------------------------------------------------- entry
    def step(self, inputs: Optional[Sequence] = None, labels: Optional[torch.Tensor] = None,
             train: bool = True):
        """Run one global batch through the pipeline.  ``inputs``: per-micro-batch inputs of the
        first stage.  ``labels``: full-batch labels on the first stage (sent to the last).
        Returns the list of per-micro-batch losses on the last stage."""
        st = self.stage
        cm = self.comms
        st.clear()
        if self.P > 1 and cm is not None:
            ops, buf = cm.labels_ops(labels, st.is_first, st.is_last)
            self._run(ops, [buf] if buf is not None else [])
            if st.is_last:
                labels = buf
        if st.is_last:
            st.labels = list(torch.tensor_split(labels, self.n)) if labels is not None else None
        if not train:
            self._forward_pass(inputs, train=False)
        elif self.schedule == "gpipe":
            self._forward_pass(inputs, train=True)
            self._backward_pass()
        else:
            self._one_f_one_b(inputs)
        return st.losses

    def _forward_pass(self, inputs, train: bool):
        cm = self.comms
        send_h = None
        for i in range(self.n):
            ops, meta = self._recv_fwd()
            self._run(ops)
            out = self._forward(i, meta, inputs, train)
            if cm is not None:
                cm.wait(send_h)
                sops, keep = self._send_fwd(out)
                send_h = cm.issue(sops, keep)
        if cm is not None:
            cm.wait(send_h)

    def _backward_pass(self):
        cm = self.comms
        send_h = None
        for i in range(self.n):
            ops, meta = self._recv_bwd()
            self._run(ops)
            g = self._backward(i, meta)
            if cm is not None:
                cm.wait(send_h)
                sops, keep = self._send_bwd(g)
                send_h = cm.issue(sops, keep)
        if cm is not None:
            cm.wait(send_h)

    def _one_f_one_b(self, inputs):
        cm = self.comms
        n = self.n
        warmup = min(n, self.P - self.s)
        fi = bi = 0
        send_h = None
        fsend_ops, fsend_keep = [], []
        for _ in range(warmup):
            ops, meta = self._recv_fwd()
            self._run(ops)
            out = self._forward(fi, meta, inputs, True)
            if cm is not None:
                cm.wait(send_h)
                send_h = None
            fsend_ops, fsend_keep = self._send_fwd(out)
            if fi != warmup - 1 and cm is not None:
                send_h = cm.issue(fsend_ops, fsend_keep)
                fsend_ops, fsend_keep = [], []
            fi += 1
        bsend_ops, bsend_keep = [], []
        while True:
            ops, meta = self._recv_bwd()
            self._run(fsend_ops + ops, fsend_keep)
            fsend_ops, fsend_keep = [], []
            g = self._backward(bi, meta)
            bsend_ops, bsend_keep = self._send_bwd(g)
            bi += 1
            if fi == n:
                break
            ops, meta = self._recv_fwd()
            self._run(bsend_ops + ops, bsend_keep)
            bsend_ops, bsend_keep = [], []
            out = self._forward(fi, meta, inputs, True)
            fsend_ops, fsend_keep = self._send_fwd(out)
            fi += 1
        send_h = cm.issue(bsend_ops, bsend_keep) if cm is not None else None
        while bi < n:
            ops, meta = self._recv_bwd()
            self._run(ops)
            g = self._backward(bi, meta)
            if cm is not None:
                cm.wait(send_h)
            bsend_ops, bsend_keep = self._send_bwd(g)
            send_h = cm.issue(bsend_ops, bsend_keep) if cm is not None else None
            bi += 1
        if cm is not None:
            cm.wait(send_h)
