"""Stage-to-stage message channels.

A ``Channel`` carries one kind of message (forward activations s -> s+1, or backward
gradients + reconstructed inputs s+1 -> s) in one direction, over its own two-rank
process group.  Because every channel has its own communicator (and so its own NCCL
stream) and messages inside a channel are matched strictly in order, the forward and
backward traffic of a stage pair can never block each other; the 1F1B send/recv pairing
of the reference (BERT/pipelining/schedules.py:725-849, one fused batch_isend_irecv per
step, waited synchronously) becomes free-running FIFO queues.

Receives are posted ahead of use into a ring of ``depth`` preallocated slots; waiting on
a receive makes the *current stream* wait for the NCCL stream (no host block on NCCL).
Each slot carries a generation counter: reusing a slot whose previous message was never
consumed raises (host-side race check).
"""
from __future__ import annotations

import datetime
import os
from collections import deque
from dataclasses import dataclass, field
from typing import Deque, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


@dataclass
class TensorSpec:
    shape: Tuple[int, ...]
    dtype: torch.dtype


@dataclass
class _Pending:
    slot: int
    gen: int
    works: list
    tensors: List[torch.Tensor]


class RingSlotError(RuntimeError):
    pass


class Channel:
    def __init__(self, name: str, src: int, dst: int, group, specs: Sequence[TensorSpec], device: torch.device,
                 depth: int = 2):
        self.name = name
        self.src = src
        self.dst = dst
        self.group = group
        self.specs = list(specs)
        self.device = device
        self.depth = depth
        self.rank = dist.get_rank()
        self._slots: Optional[List[List[torch.Tensor]]] = None
        self._slot_gen: List[int] = [0] * depth
        self._slot_busy: List[bool] = [False] * depth
        self._next_slot = 0
        self._posted: Deque[_Pending] = deque()
        self._send_inflight: Deque[Tuple[list, List[torch.Tensor]]] = deque()
        self.sent = 0
        self.received = 0
        # gloo point-to-point waits have no timeout of their own: bound them here so a lost
        # message or a dead peer surfaces as an error.  NCCL waits stay stream-level; its
        # watchdog enforces the process-group timeout.
        self.host_wait = dist.get_backend(group) == "gloo"
        self.timeout = datetime.timedelta(seconds=float(os.environ.get("REVPP_P2P_HOST_TIMEOUT_S", "30")))

    # -------------------------------------------------------------- receive side
    def _alloc(self):
        if self._slots is None:
            self._slots = [[torch.empty(s.shape, dtype=s.dtype, device=self.device) for s in self.specs]
                           for _ in range(self.depth)]

    def post_recv(self) -> None:
        """Post the receive of the next message into the next free ring slot."""
        assert self.rank == self.dst, f"{self.name}: only rank {self.dst} receives"
        self._alloc()
        slot = self._next_slot
        if self._slot_busy[slot]:
            raise RingSlotError(f"{self.name}: ring slot {slot} (gen {self._slot_gen[slot]}) reused before its "
                                f"message was consumed")
        self._slot_busy[slot] = True
        self._slot_gen[slot] += 1
        bufs = self._slots[slot]
        ops = [dist.P2POp(dist.irecv, t, self.src, self.group) for t in bufs]
        works = dist.batch_isend_irecv(ops)
        self._posted.append(_Pending(slot, self._slot_gen[slot], works, bufs))
        self._next_slot = (slot + 1) % self.depth

    @property
    def posted(self) -> int:
        return len(self._posted)

    def recv(self) -> Tuple[List[torch.Tensor], int]:
        """Oldest posted message.  The current stream waits for it; returns (tensors, slot)."""
        if not self._posted:
            self.post_recv()
        p = self._posted.popleft()
        for w in p.works:
            self._wait(w)
        self.received += 1
        return p.tensors, p.slot

    def _wait(self, w) -> None:
        if self.host_wait:
            if not w.wait(self.timeout):
                raise RuntimeError(f"{self.name}: message not received within {self.timeout}")
        else:
            w.wait()

    def release(self, slot: int) -> None:
        """The consumer is done with a slot (its reads are enqueued on the current stream)."""
        self._slot_busy[slot] = False

    # -------------------------------------------------------------- send side
    def send(self, tensors: Sequence[torch.Tensor]) -> None:
        assert self.rank == self.src, f"{self.name}: only rank {self.src} sends"
        ts = [t.contiguous() for t in tensors]
        for t, s in zip(ts, self.specs):
            if tuple(t.shape) != tuple(s.shape) or t.dtype != s.dtype:
                raise ValueError(f"{self.name}: message {tuple(t.shape)}/{t.dtype} does not match "
                                 f"{tuple(s.shape)}/{s.dtype}")
        from .faults import should_drop

        if should_drop(self.name, self.sent):
            self.sent += 1  # injected loss: the receiver must time out, not hang
            return
        ops = [dist.P2POp(dist.isend, t, self.dst, self.group) for t in ts]
        works = dist.batch_isend_irecv(ops)
        self._send_inflight.append((works, ts))
        self.sent += 1
        self._reap()

    def _reap(self, keep: int = 4) -> None:
        # keep the last few sends' tensors alive; older ones are complete once waited
        while len(self._send_inflight) > keep:
            works, _ = self._send_inflight.popleft()
            for w in works:
                self._wait(w)

    def drain(self) -> None:
        while self._send_inflight:
            works, _ = self._send_inflight.popleft()
            for w in works:
                self._wait(w)


def _warm_group(group, ranks, device) -> None:
    """Create the group's communicator and, for a two-rank group, its point-to-point
    connections now.  NCCL builds both on first use, and building them blocks the host
    until the peer joins; left lazy, stage s would block on its first (early-posted)
    backward receive before sending its first forward message, while stage s+1 touches
    the backward channel only after that message arrives.  Warming every group in
    creation order, with a symmetric send + receive for pairs, cannot deadlock."""
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


class PipeComms:
    """All channels of one rank: forward/backward to both neighbours plus the label channel.

    Process groups are created collectively by every rank in the same order (a requirement
    of ``new_group``), for every pipeline replica, and their communicators are created
    eagerly in that order (see ``_warm_group``)."""

    def __init__(self, rank: int, world: int, num_stages: int, replicas: int, device: torch.device,
                 fwd_specs, bwd_specs, label_spec: Optional[TensorSpec], depth: int = 2):
        self.rank = rank
        self.P = num_stages
        self.replica = rank // num_stages
        self.stage = rank % num_stages
        base = self.replica * num_stages
        self.fwd_in = self.fwd_out = self.bwd_in = self.bwd_out = self.labels = None
        backend = dist.get_backend()
        for d in range(replicas):
            b = d * num_stages
            for s in range(num_stages - 1):
                a, c = b + s, b + s + 1
                g_f = dist.new_group([a, c], backend=backend)
                _warm_group(g_f, (a, c), device)
                g_b = dist.new_group([a, c], backend=backend)
                _warm_group(g_b, (a, c), device)
                if d == self.replica:
                    if self.stage == s:
                        self.fwd_out = Channel(f"fwd{s}->{s+1}", a, c, g_f, fwd_specs, device, depth)
                        self.bwd_in = Channel(f"bwd{s+1}->{s}", c, a, g_b, bwd_specs, device, depth)
                    if self.stage == s + 1:
                        self.fwd_in = Channel(f"fwd{s}->{s+1}", a, c, g_f, fwd_specs, device, depth)
                        self.bwd_out = Channel(f"bwd{s+1}->{s}", c, a, g_b, bwd_specs, device, depth)
            if num_stages > 1 and label_spec is not None:
                g_l = dist.new_group([b, b + num_stages - 1], backend=backend)
                _warm_group(g_l, (b, b + num_stages - 1), device)
                if d == self.replica and self.stage in (0, num_stages - 1):
                    self.labels = Channel("labels", b, b + num_stages - 1, g_l, [label_spec], device, depth)
        self.first_rank = base
        self.last_rank = base + num_stages - 1

    def drain(self) -> None:
        for ch in (self.fwd_out, self.bwd_out, self.labels):
            if ch is not None and ch.rank == ch.src:
                ch.drain()
