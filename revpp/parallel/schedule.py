"""Pipeline schedules as explicit per-rank action lists, and their executor.

``one_f_one_b(stage, P, n)`` gives the reference's Schedule1F1B order
(BERT/pipelining/schedules.py:677-852): min(P - s - 1, n) warm-up forwards, then
alternating forward / backward, then the remaining backwards.  ``gpipe`` is all forwards
then all backwards (ScheduleGPipe, schedules.py:591-673); ``forward_only`` is the
evaluation schedule (_ScheduleForwardOnly, schedules.py:538-588).

The executor posts receives ahead of use (depth-2 ring per channel), so the transfer
of micro-batch k+1 overlaps the compute of micro-batch k; each wait is a stream-level
dependency, not a host block.  Labels travel from the first to the last stage once per
step, as in the reference engine (BERT/src/engine.py:174-176, 238-240).
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from .p2p import PipeComms

Action = Tuple[str, int]


def one_f_one_b(stage: int, num_stages: int, n: int) -> List[Action]:
    warmup = min(num_stages - stage - 1, n)
    acts: List[Action] = [("F", i) for i in range(warmup)]
    f, b = warmup, 0
    while f < n:
        acts.append(("F", f))
        f += 1
        acts.append(("B", b))
        b += 1
    while b < n:
        acts.append(("B", b))
        b += 1
    return acts


def gpipe(stage: int, num_stages: int, n: int) -> List[Action]:
    return [("F", i) for i in range(n)] + [("B", i) for i in range(n)]


def forward_only(stage: int, num_stages: int, n: int) -> List[Action]:
    return [("F", i) for i in range(n)]


SCHEDULES = {"1f1b": one_f_one_b, "gpipe": gpipe}


def simulate(num_stages: int, n: int, schedule: str = "1f1b", t_f: float = 1.0, t_b: float = 2.0):
    """Event simulation of a schedule: returns (makespan, per-stage busy time).  Used to
    check schedules without GPUs and to predict bubble fractions."""
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
            else:
                dep = f_done[s][i] if s == num_stages - 1 else b_done[s + 1][i]
                if dep is None or f_done[s][i] is None:
                    continue
                start = max(t[s], dep)
                t[s] = start + t_b
                b_done[s][i] = t[s]
                busy[s] += t_b
            pos[s] += 1
            progress = True
    if any(p < len(a) for p, a in zip(pos, acts)):
        raise RuntimeError("schedule deadlocks")
    return max(t), busy


class PipelineExecutor:
    def __init__(self, stage, comms: Optional[PipeComms], num_microbatches: int, schedule: str = "1f1b"):
        self.stage = stage
        self.comms = comms
        self.n = num_microbatches
        self.schedule = schedule
        self.P = stage.num_stages
        self.s = stage.stage_index

    def _top_up(self, ch, remaining: List[int]) -> None:
        """Keep up to ``depth`` receives posted on a channel."""
        if ch is None:
            return
        while remaining[0] > 0 and ch.posted < ch.depth and not ch._slot_busy[ch._next_slot]:
            ch.post_recv()
            remaining[0] -= 1

    def step(self, inputs: Optional[Sequence] = None, labels: Optional[torch.Tensor] = None,
             train: bool = True):
        """Run one global batch through the pipeline.  ``inputs``: per-micro-batch inputs of the
        first stage.  ``labels``: full-batch labels on the first stage (sent to the last).
        Returns the list of per-micro-batch losses on the last stage."""
        st = self.stage
        cm = self.comms
        st.clear()
        # labels: first -> last
        if self.P > 1 and cm is not None and cm.labels is not None:
            if st.is_first and labels is not None:
                cm.labels.send([labels])
            if st.is_last:
                (lab,), slot = cm.labels.recv()
                labels = lab.clone()
                cm.labels.release(slot)
        if st.is_last:
            st.labels = list(torch.tensor_split(labels, self.n)) if labels is not None else None
        fn = SCHEDULES[self.schedule] if train else forward_only
        acts = fn(self.s, self.P, self.n)
        fwd_in = cm.fwd_in if cm is not None else None
        bwd_in = cm.bwd_in if (cm is not None and train) else None
        rem_f = [self.n if fwd_in is not None else 0]
        rem_b = [self.n if bwd_in is not None else 0]
        self._top_up(fwd_in, rem_f)
        self._top_up(bwd_in, rem_b)
        from .faults import before_forward

        rank = dist.get_rank() if dist.is_initialized() else 0
        for kind, i in acts:
            if kind == "F":
                before_forward(rank, i)
                if st.is_first:
                    out = st.forward(i, inputs[i], train)
                else:
                    msg, slot = fwd_in.recv()
                    out = st.forward(i, msg, train)
                    fwd_in.release(slot)
                    self._top_up(fwd_in, rem_f)
                if out is not None and cm is not None and cm.fwd_out is not None:
                    cm.fwd_out.send(out)
            else:
                if st.is_last:
                    g = st.backward(i, None)
                else:
                    msg, slot = bwd_in.recv()
                    g = st.backward(i, msg)
                    bwd_in.release(slot)
                    self._top_up(bwd_in, rem_b)
                if g is not None and cm is not None and cm.bwd_out is not None:
                    cm.bwd_out.send(g)
        return st.losses
