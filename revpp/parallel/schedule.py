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

from typing import Dict, List, Optional, Sequence, Tuple

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


class StepTimeline:
    """Device timeline of one pipeline step on one rank: CUDA events on the compute stream
    at the step's ends and around the compute of every action (recorded after the stream
    waits for the action's input, so the gap before an action is the time its rank sat idle:
    schedule bubble, transfer or synchronisation)."""

    def __init__(self):
        self.marks: List[tuple] = []  # (kind, start event, end event)
        self.t0 = self.t1 = None
        self._open = None

    @staticmethod
    def _ev():
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def begin(self):
        self.marks, self._open = [], None
        self.t0 = self._ev()

    def start(self):
        self._open = self._ev()

    def stop(self, kind: str):
        if self._open is not None:
            self.marks.append((kind, self._open, self._ev()))
            self._open = None

    def end(self):
        self.t1 = self._ev()

    def summary(self) -> dict:
        """Step time, compute time, idle time and the mean forward / backward action (ms)."""
        self.t1.synchronize()
        step = self.t0.elapsed_time(self.t1)
        per = {"F": [], "B": []}
        for kind, a, b in self.marks:
            per[kind].append(a.elapsed_time(b))
        comp = sum(per["F"]) + sum(per["B"])
        mean = lambda xs: sum(xs) / len(xs) if xs else 0.0  # noqa: E731
        return {"step_ms": step, "compute_ms": comp, "idle_ms": max(0.0, step - comp),
                "fwd_action_ms": mean(per["F"]), "bwd_action_ms": mean(per["B"]),
                "n_fwd": len(per["F"]), "n_bwd": len(per["B"])}


def pipeline_breakdown(rank_summaries: Sequence[dict], num_stages: int, chunks: int, n: int,
                       schedule: str) -> List[dict]:
    """Split every rank's idle time into the schedule's own bubble and the rest.  The bubble
    is what ``simulate_virtual`` gives for this schedule with every rank's measured mean
    action times and instant transfers; the rest of the idle time is exposed transfer and
    synchronisation.  ``rank_summaries[r]`` is ``StepTimeline.summary()`` of pipeline rank r."""
    tf = [s["fwd_action_ms"] for s in rank_summaries]
    tb = [s["bwd_action_ms"] for s in rank_summaries]
    sched = "interleaved" if chunks > 1 else schedule
    span, busy = simulate_virtual(num_stages, chunks, n, sched, t_f=tf, t_b=tb)
    out = []
    for r, s in enumerate(rank_summaries):
        bubble = span - busy[r]
        out.append({"stage": r, "step_ms": s["step_ms"], "compute_ms": s["compute_ms"],
                    "bubble_ms": min(bubble, s["idle_ms"]), "exposed_p2p_ms": max(0.0, s["idle_ms"] - bubble),
                    "fwd_action_ms": s["fwd_action_ms"], "bwd_action_ms": s["bwd_action_ms"]})
    return out


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
        self.timeline: Optional[StepTimeline] = None  # set to record one step's device timeline

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
        tl = self.timeline
        if tl is not None:
            tl.start()
        out = self.stage.forward(i, x, train)
        if tl is not None:
            tl.stop("F")
        if meta is not None:
            meta[0].release(meta[1])
        return out

    def _backward(self, i, meta):
        tl = self.timeline
        if tl is not None:
            tl.start()
        g = self.stage.backward(i, None if meta is None else meta[2])
        if tl is not None:
            tl.stop("B")
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
        if self.timeline is not None:
            self.timeline.begin()
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
        if self.timeline is not None:
            self.timeline.end()
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


# ============================================================================ virtual pipelines
# A rank may hold several model chunks ("virtual stages").  Chunk c of rank r is global stage
# g = c * P + r of G = v * P; its forward output goes to global stage g + 1 (rank r + 1, or
# rank 0's next chunk when r = P - 1) and its backward message to g - 1.  Actions are
# (kind, chunk, micro-batch).

VAction = Tuple[str, int, int]


def interleaved_1f1b(rank: int, num_stages: int, chunks: int, n: int) -> List[VAction]:
    """Interleaved 1F1B (BERT/pipelining/schedules.py:1954, ScheduleInterleaved1F1B; the
    Megatron-LM order): micro-batches go through the chunks in groups of P; the k-th forward
    is chunk (k // P) % v of micro-batch (k // (P v)) P + k % P, the k-th backward the same
    with the chunk order reversed.  Rank r runs 2 (P - r - 1) + (v - 1) P warm-up forwards,
    then alternates one forward and one backward, then drains the backwards.  With v = 1
    this is the ordinary 1F1B order."""
    P, v = num_stages, chunks
    if v == 1:
        return [(k, 0, m) for k, m in one_f_one_b(rank, P, n)]
    if n % P != 0:
        raise ValueError(f"interleaved 1F1B needs the number of micro-batches ({n}) to be a multiple of "
                         f"the pipeline depth ({P})")
    total = n * v

    def fwd(k):
        return (k // P) % v, (k // (P * v)) * P + k % P

    def bwd(k):
        c, m = fwd(k)
        return v - 1 - c, m

    warm = total if n == P else min((P - rank - 1) * 2 + (v - 1) * P, total)
    acts: List[VAction] = [("F",) + fwd(k) for k in range(warm)]
    for k in range(total - warm):
        acts.append(("F",) + fwd(warm + k))
        acts.append(("B",) + bwd(k))
    acts += [("B",) + bwd(k) for k in range(total - warm, total)]
    return acts


def virtual_actions(schedule: str, rank: int, num_stages: int, chunks: int, n: int, train: bool = True):
    if not train:
        if chunks == 1:
            return [("F", 0, m) for m in range(n)]
        return [a for a in interleaved_1f1b(rank, num_stages, chunks, n) if a[0] == "F"]
    if schedule == "interleaved" or chunks > 1:
        return interleaved_1f1b(rank, num_stages, chunks, n)
    return [(k, 0, m) for k, m in SCHEDULES[schedule](rank, num_stages, n)]


def _route(kind: str, rank: int, chunk: int, P: int):
    """(peer rank, peer chunk) that the output of (kind, rank, chunk) goes to."""
    if kind == "F":
        return (rank + 1) % P, chunk + (1 if rank == P - 1 else 0)
    return (rank - 1) % P, chunk - (1 if rank == 0 else 0)


def simulate_virtual(num_stages: int, chunks: int, n: int, schedule: str = "interleaved", t_f: float = 1.0,
                     t_b: float = 3.0, t_comm: float = 0.0, events: list | None = None):
    """Timeline of a (virtual) pipeline schedule: every action of rank r starts when the rank
    is free and its input has arrived (``t_comm`` after the producer finished; transfers run
    beside compute).  ``t_f`` / ``t_b`` are per chunk, one value or one per rank.  Returns
    (makespan, per-rank busy).
    Raises if the action orders deadlock."""
    P, v = num_stages, chunks
    G = P * v
    tf = list(t_f) if isinstance(t_f, (list, tuple)) else [t_f] * P
    tb = list(t_b) if isinstance(t_b, (list, tuple)) else [t_b] * P
    acts = [virtual_actions(schedule, r, P, v, n) for r in range(P)]
    pos = [0] * P
    t = [0.0] * P
    busy = [0.0] * P
    fdone: Dict = {}
    bdone: Dict = {}
    progress = True
    while progress:
        progress = False
        for r in range(P):
            while pos[r] < len(acts[r]):
                kind, c, m = acts[r][pos[r]]
                g = c * P + r
                if kind == "F":
                    if g == 0:
                        ready = 0.0
                    else:
                        src = fdone.get((g - 1, m))
                        if src is None:
                            break
                        ready = src + t_comm
                    dur = tf[r]
                else:
                    if g == G - 1:
                        src = fdone.get((g, m))
                        ready = src if src is not None else None
                    else:
                        src = bdone.get((g + 1, m))
                        ready = None if src is None else src + t_comm
                    if ready is None or (g, m) not in fdone:
                        break
                    dur = tb[r]
                start = max(t[r], ready)
                t[r] = start + dur
                busy[r] += dur
                (fdone if kind == "F" else bdone)[(g, m)] = t[r]
                if events is not None:
                    events.append((r, kind, c, m, start, t[r]))
                pos[r] += 1
                progress = True
    if any(p < len(a) for p, a in zip(pos, acts)):
        raise RuntimeError("schedule deadlocks")
    return max(t), busy


def host_deadlock_free(num_stages: int, chunks: int, n: int, schedule: str, depth: int, early_bwd_claim: bool = True,
                       steps: int = 2) -> bool:
    """Run the hosts of every rank of one pipeline through ``steps`` training steps with the
    channel protocol (revpp.parallel.channels): an action waits for its input message to be
    committed; the input is released after the action; sending message k on a channel waits
    until the receiver released message k - depth.  With ``early_bwd_claim`` a backward claims
    its output slot before releasing its input (the reconstructed stage input is sent before
    the gradients are complete).  Returns False if some host would wait forever."""
    P, v = num_stages, chunks
    G = P * v
    acts = [virtual_actions(schedule, r, P, v, n) for r in range(P)] if P > 1 else [[]]
    # channel state: committed / released counts per (kind, src rank)
    committed: Dict = {}
    released: Dict = {}
    # FIFO order check: the messages of a channel in sending order
    sent_seq: Dict = {}
    recv_seq: Dict = {}
    for r in range(P):
        for kind, c, m in acts[r]:
            g = c * P + r
            if kind == "F" and g < G - 1:
                sent_seq.setdefault(("F", r), []).append(m * G + g + 1)
            if kind == "B" and g > 0:
                sent_seq.setdefault(("B", r), []).append(m * G + g - 1)
            if kind == "F" and g > 0:
                recv_seq.setdefault(("F", (r - 1) % P), []).append(m * G + g)
            if kind == "B" and g < G - 1:
                recv_seq.setdefault(("B", (r + 1) % P), []).append(m * G + g)
    for key in sent_seq:
        if sent_seq[key] != recv_seq.get(key):
            raise RuntimeError(f"channel {key} is not consumed in sending order")
    # per rank: (step, action index, phase) ; phase 0 = waiting input, 1 = waiting output slot
    state = [[0, 0, 0] for _ in range(P)]
    total = len(acts[0]) if P > 0 else 0
    recv_count: Dict = {}
    send_count: Dict = {}

    def ch_in(kind, r):
        return (kind, (r - 1) % P) if kind == "F" else (kind, (r + 1) % P)

    progress = True
    while progress:
        progress = False
        for r in range(P):
            st = state[r]
            while st[0] < steps:
                if st[1] >= len(acts[r]):
                    st[0], st[1], st[2] = st[0] + 1, 0, 0
                    continue
                kind, c, m = acts[r][st[1]]
                g = c * P + r
                needs_in = (kind == "F" and g > 0) or (kind == "B" and g < G - 1)
                has_out = (kind == "F" and g < G - 1) or (kind == "B" and g > 0)
                cin = ch_in(kind, r)
                cout = (kind, r)
                if st[2] == 0:
                    if needs_in:
                        k = recv_count.get(cin, 0)
                        if committed.get(cin, 0) < k + 1:
                            break
                    st[2] = 1
                    if not (early_bwd_claim and kind == "B") and needs_in:
                        recv_count[cin] = recv_count.get(cin, 0) + 1
                        released[cin] = recv_count[cin]
                if st[2] == 1:
                    if has_out:
                        k = send_count.get(cout, 0)
                        if released.get(cout, 0) < k - depth + 1:
                            break
                        send_count[cout] = k + 1
                    if early_bwd_claim and kind == "B" and needs_in:
                        recv_count[cin] = recv_count.get(cin, 0) + 1
                        released[cin] = recv_count[cin]
                    if has_out:
                        committed[cout] = send_count[cout]
                    st[1], st[2] = st[1] + 1, 0
                    progress = True
    del total
    return all(s[0] >= steps for s in state)


def min_channel_depth(num_stages: int, chunks: int, n: int, schedule: str, early_bwd_claim: bool = True,
                      limit: int = 64) -> int:
    """Smallest receive-ring depth with which the hosts cannot deadlock (at least 2)."""
    for d in range(2, limit + 1):
        if host_deadlock_free(num_stages, chunks, n, schedule, d, early_bwd_claim):
            return d
    raise RuntimeError("no ring depth up to %d avoids a deadlock for this schedule" % limit)


class ChannelExecutor:
    """Runs a (virtual) pipeline schedule on one rank over copy channels
    (revpp.parallel.channels): every forward / backward sends its message as soon as it is
    enqueued, and waits only for the message it consumes, so transfers overlap compute on
    both GPUs.  A reversible backward sends the reconstructed stage input (X2, X1) as soon as
    it exists and the gradients when they are done.

    ``stages[c]`` is the runtime of chunk c; ``chans`` maps "fwd_in", "fwd_out", "bwd_in",
    "bwd_out", "labels" to this rank's channels (absent where the rank has none)."""

    def __init__(self, stages, chans: Dict[str, object], num_microbatches: int, num_stages: int, rank_in_pipe: int,
                 schedule: str = "1f1b", early_x: bool = True, global_rank: int = 0):
        self.stages = list(stages)
        self.v = len(self.stages)
        self.chans = chans
        self.n = num_microbatches
        self.P = num_stages
        self.r = rank_in_pipe
        self.schedule = schedule
        self.early_x = early_x
        self.global_rank = global_rank
        self.train_actions = virtual_actions(schedule, self.r, self.P, self.v, self.n, train=True)
        self.eval_actions = virtual_actions(schedule, self.r, self.P, self.v, self.n, train=False)
        self.first = self.stages[0]
        self.last = self.stages[-1]
        # compatibility with the single-chunk executor
        self.stage = self.first
        self.timeline: Optional[StepTimeline] = None  # set to record one step's device timeline

    def step(self, inputs: Optional[Sequence] = None, labels: Optional[torch.Tensor] = None, train: bool = True):
        from .channels import ChannelError

        for st in self.stages:
            st.clear()
        tl = self.timeline
        if tl is not None:
            tl.begin()
        try:
            lab_ch = self.chans.get("labels")
            if lab_ch is not None:
                if self.first.is_first:
                    lab_ch.send([labels.to(self.first.device, non_blocking=True)])
                if self.last.is_last:
                    labels = lab_ch.recv()[0].clone()
                    lab_ch.release()
            if self.last.is_last:
                self.last.labels = list(torch.tensor_split(labels, self.n)) if labels is not None else None
            for kind, c, m in (self.train_actions if train else self.eval_actions):
                if kind == "F":
                    self._fwd(c, m, inputs, train)
                else:
                    self._bwd(c, m)
            if tl is not None:
                tl.end()
        except ChannelError:
            raise
        except BaseException:
            chs = [ch for ch in self.chans.values() if ch is not None]
            if chs:
                chs[0].counters.abort()  # the other ranks' next wait raises instead of timing out
            raise
        return self.last.losses

    def _fwd(self, c, m, inputs, train):
        from .faults import before_forward

        st = self.stages[c]
        if c == 0:
            before_forward(self.global_rank, m)
        cin = None
        if st.is_first:
            x = inputs[m]
        else:
            cin = self.chans["fwd_in"]
            x = cin.recv()
        tl = self.timeline
        if tl is not None:
            tl.start()
        out = st.forward(m, x, train)
        if tl is not None:
            tl.stop("F")
        if cin is not None:
            cin.release()
        if out is not None and not st.is_last:
            self.chans["fwd_out"].send(out)

    def _bwd(self, c, m):
        st = self.stages[c]
        msg = None
        cin = None
        if not st.is_last:
            cin = self.chans["bwd_in"]
            msg = cin.recv()
        cout = None if st.is_first else self.chans["bwd_out"]
        hook = None
        if cout is not None and self.early_x and getattr(st, "kind", "") == "reversible":
            def hook(x2, x1, _c=cout):
                _c.put(2, x2)
                _c.put(3, x1)
        tl = self.timeline
        if tl is not None:
            tl.start()
        g = st.backward(m, msg, on_input=hook) if hook is not None else st.backward(m, msg)
        if tl is not None:
            tl.stop("B")
        if cin is not None:
            cin.release()
        if g is not None and cout is not None:
            if hook is not None:
                cout.put(0, g[0])
                cout.put(1, g[1])
                cout.commit()
            else:
                cout.send(g)
