"""Stage-to-stage messages.

All point-to-point traffic of one pipeline runs on one process group (one NCCL
communicator, hence one NCCL stream per rank).  The executor groups the operations of a
schedule step exactly as the reference's Schedule1F1B does (BERT/pipelining/schedules.py:
700-852): forward-send with backward-receive, backward-send with forward-receive, each
group issued as one ``batch_isend_irecv`` in the same order on both sides of a stage pair.
With a single NCCL stream per rank this ordering is deadlock-free.  (A design with one
communicator per direction and receives posted ahead deadlocked on 2 GPUs: NCCL kernels of
different streams can share a hardware queue, so a send could wait behind a receive whose
data that very send unblocks on the peer.)

Receive buffers are preallocated rings (depth 2) per message kind.  Each slot carries a
generation counter; reusing a slot whose previous message was never consumed raises
(host-side race check).  Waiting on a group is a stream-level wait on NCCL; on gloo (CPU
tests) it is a host wait bounded by REVPP_P2P_HOST_TIMEOUT_S, so a lost message or a dead
peer becomes an error.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


@dataclass
class TensorSpec:
    shape: Tuple[int, ...]
    dtype: torch.dtype


class RingSlotError(RuntimeError):
    pass


class RecvRing:
    """Preallocated receive buffers for one message kind."""

    def __init__(self, name: str, specs: Sequence[TensorSpec], device: torch.device, depth: int = 2):
        self.name = name
        self.specs = list(specs)
        self.device = device
        self.depth = depth
        self._slots: Optional[List[List[torch.Tensor]]] = None
        self.gen = [0] * depth
        self.busy = [False] * depth
        self.next = 0

    def acquire(self) -> Tuple[int, List[torch.Tensor]]:
        if self._slots is None:
            self._slots = [[torch.empty(s.shape, dtype=s.dtype, device=self.device) for s in self.specs]
                           for _ in range(self.depth)]
        slot = self.next
        if self.busy[slot]:
            raise RingSlotError(f"{self.name}: ring slot {slot} (generation {self.gen[slot]}) reused before its "
                                "message was consumed")
        self.busy[slot] = True
        self.gen[slot] += 1
        self.next = (slot + 1) % self.depth
        return slot, self._slots[slot]

    def release(self, slot: int) -> None:
        self.busy[slot] = False


def _warm_group(group, ranks, device) -> None:
    """Create the group's NCCL communicator (and, for a pair, its point-to-point
    connections) now, at start-up, in a fixed order on every member: NCCL otherwise builds
    them on first use, blocking the host until the peer joins."""
    me = dist.get_rank()
    if me not in ranks:
        return
    t = torch.zeros(1, device=device)
    dist.all_reduce(t, group=group)
    if len(ranks) == 2:
        peer = ranks[1] if me == ranks[0] else ranks[0]
        out = torch.zeros(1, device=device)
        inp = torch.empty(1, device=device)
        works = dist.batch_isend_irecv([dist.P2POp(dist.isend, out, peer, group),
                                        dist.P2POp(dist.irecv, inp, peer, group)])
        for w in works:
            w.wait()


def _warm_pipeline_p2p(group, ranks, device) -> None:
    """Establish every neighbour connection of a pipeline group: even pairs then odd pairs,
    each a symmetric send + receive, so no rank blocks on a peer that is busy elsewhere."""
    me = dist.get_rank()
    if me not in ranks:
        return
    i = ranks.index(me)
    for parity in (0, 1):
        for a in range(parity, len(ranks) - 1, 2):
            if i in (a, a + 1):
                peer = ranks[a + 1] if i == a else ranks[a]
                out = torch.zeros(1, device=device)
                inp = torch.empty(1, device=device)
                works = dist.batch_isend_irecv([dist.P2POp(dist.isend, out, peer, group),
                                                dist.P2POp(dist.irecv, inp, peer, group)])
                for w in works:
                    w.wait()


class PipeComms:
    """Point-to-point plumbing of one rank: its pipeline's process group, neighbour ranks,
    receive rings and message checks.  Groups are created collectively (every rank, same
    order) for every pipeline replica."""

    def __init__(self, rank: int, world: int, num_stages: int, replicas: int, device: torch.device,
                 fwd_specs, bwd_specs_in, label_spec: Optional[TensorSpec], depth: int = 2):
        self.rank = rank
        self.P = num_stages
        self.replica = rank // num_stages
        self.stage = rank % num_stages
        self.device = device
        base = self.replica * num_stages
        self.first_rank = base
        self.last_rank = base + num_stages - 1
        self.prev = rank - 1 if self.stage > 0 else None
        self.next = rank + 1 if self.stage < num_stages - 1 else None
        self.group = None
        backend = dist.get_backend()
        for d in range(replicas):
            ranks = list(range(d * num_stages, (d + 1) * num_stages))
            g = dist.new_group(ranks, backend=backend)
            _warm_group(g, ranks, device)
            _warm_pipeline_p2p(g, ranks, device)
            if d == self.replica:
                self.group = g
        if num_stages > 1:
            # the label message first -> last
            for d in range(replicas):
                ranks = list(range(d * num_stages, (d + 1) * num_stages))
                if self.rank in (ranks[0], ranks[-1]) and d == self.replica:
                    peer = ranks[-1] if self.rank == ranks[0] else ranks[0]
                    if abs(ranks[-1] - ranks[0]) > 1:
                        out = torch.zeros(1, device=device)
                        inp = torch.empty(1, device=device)
                        works = dist.batch_isend_irecv([dist.P2POp(dist.isend, out, peer, self.group),
                                                        dist.P2POp(dist.irecv, inp, peer, self.group)])
                        for w in works:
                            w.wait()
        self.fwd_specs = list(fwd_specs)
        self.fwd_ring = RecvRing("fwd", fwd_specs, device, depth) if self.prev is not None else None
        self.bwd_ring = RecvRing("bwd", bwd_specs_in, device, depth) if self.next is not None else None
        self.label_spec = label_spec
        self.host_wait = backend == "gloo"
        self.timeout = datetime.timedelta(seconds=float(os.environ.get("REVPP_P2P_HOST_TIMEOUT_S", "30")))
        self.sent = {"fwd": 0, "bwd": 0}

    # -------------------------------------------------------------- op builders
    def recv_fwd(self):
        slot, bufs = self.fwd_ring.acquire()
        return [dist.P2POp(dist.irecv, t, self.prev, self.group) for t in bufs], (self.fwd_ring, slot, bufs)

    def recv_bwd(self):
        slot, bufs = self.bwd_ring.acquire()
        return [dist.P2POp(dist.irecv, t, self.next, self.group) for t in bufs], (self.bwd_ring, slot, bufs)

    def _check(self, tensors, specs, what):
        for t, s in zip(tensors, specs):
            if tuple(t.shape) != tuple(s.shape) or t.dtype != s.dtype:
                raise ValueError(f"{what}: message {tuple(t.shape)}/{t.dtype} does not match "
                                 f"{tuple(s.shape)}/{s.dtype}")

    def send_fwd(self, tensors):
        from .faults import should_drop

        ts = [t.contiguous() for t in tensors]
        self._check(ts, self.fwd_specs, "forward send")
        idx = self.sent["fwd"]
        self.sent["fwd"] += 1
        if should_drop(f"fwd{self.stage}->{self.stage + 1}", idx):
            return [], ts
        return [dist.P2POp(dist.isend, t, self.next, self.group) for t in ts], ts

    def send_bwd(self, tensors):
        from .faults import should_drop

        ts = [t.contiguous() for t in tensors]
        idx = self.sent["bwd"]
        self.sent["bwd"] += 1
        if should_drop(f"bwd{self.stage}->{self.stage - 1}", idx):
            return [], ts
        return [dist.P2POp(dist.isend, t, self.prev, self.group) for t in ts], ts

    # -------------------------------------------------------------- issue / wait
    def issue(self, ops: list, keep: list):
        """Issue one group of operations; returns a handle for ``wait`` that also keeps the
        send buffers alive until then."""
        if not ops:
            return None
        return (dist.batch_isend_irecv(ops), keep)

    def wait(self, handle) -> None:
        if handle is None:
            return
        works, _ = handle
        for w in works:
            if self.host_wait:
                if not w.wait(self.timeout):
                    raise RuntimeError(f"pipeline message not completed within {self.timeout}")
            else:
                w.wait()

    def labels_ops(self, labels: Optional[torch.Tensor], is_first: bool, is_last: bool):
        """Labels travel once per step from the first to the last stage."""
        if self.P == 1:
            return [], None
        if is_first:
            lab = labels.to(self.device, non_blocking=True).contiguous()
            return [dist.P2POp(dist.isend, lab, self.last_rank, self.group)], lab
        if is_last:
            buf = torch.empty(self.label_spec.shape, dtype=self.label_spec.dtype, device=self.device)
            return [dist.P2POp(dist.irecv, buf, self.first_rank, self.group)], buf
        return [], None

