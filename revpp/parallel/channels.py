"""Stage-to-stage message channels over copy engines (one node).

A channel is one directed stream of messages of one kind (forward activations, backward
gradients + reconstructed inputs, labels) from a sender rank to a receiver rank.  The
receiver owns a ring of ``depth`` slots in its own memory; the sender writes message k into
slot k % depth with plain copies and the receiver reads it in place:

* **GPU** (``CudaIpcChannel``): the slots are one device buffer that the sender maps through
  CUDA IPC; each message is copied with ``cudaMemcpyAsync`` on a copy stream of the sender's
  own (a DMA copy over NVLink: no SMs, no NCCL kernel, so it runs under the GEMMs of both
  GPUs).  Ordering on the devices uses interprocess events: ``ready[s]`` is recorded by the
  sender after the copy into slot s, and the receiver's compute stream waits on it;
  ``free[s]`` is recorded by the receiver after the work that reads slot s, and the
  sender's copy stream waits on it before refilling the slot.
* **CPU** (``HostChannel``): the slots are a shared file mapped by both processes; copies
  are synchronous, so no events are needed.  The CPU tests run the same protocol.

Host ordering uses two monotonic counters per channel in a page of shared memory:
``committed`` (messages fully written and their ``ready`` event recorded, advanced by the
sender) and ``released`` (messages consumed and their ``free`` event recorded, advanced by
the receiver).  The receiver waits for ``committed > k`` before it waits on ``ready[s]``;
the sender waits for ``released > k - depth`` before it waits on ``free[s]``.  So every
event wait comes after the record it refers to, and every device dependency is created by
a host call made after its source was enqueued: the hosts' order of calls is a topological
order of the device work, and the device cannot deadlock if the hosts do not (which
``revpp.parallel.schedule.host_deadlock_free`` checks for a schedule and a ring depth).

Every host wait is bounded (``REVPP_P2P_HOST_TIMEOUT_S``); a rank that fails raises the
shared abort word, and every other rank's next wait raises instead of waiting out its
limit.  Messages of a channel are consumed in the order they are sent (checked by the
executor's plan).
"""
from __future__ import annotations

import mmap
import os
import time
import uuid
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist

from .p2p import TensorSpec

_ALIGN = 256


def _host_timeout() -> float:
    return float(os.environ.get("REVPP_P2P_HOST_TIMEOUT_S", "300"))


class ChannelError(RuntimeError):
    pass


@dataclass(frozen=True)
class ChannelSpec:
    """One directed channel: ``name`` is unique and the same on every rank."""

    name: str
    src: int
    dst: int
    specs: Tuple[TensorSpec, ...]
    depth: int


def _layout(specs: Sequence[TensorSpec]) -> Tuple[List[int], int]:
    """Byte offsets of the tensors of one slot, and the slot size (256-byte aligned)."""
    offs, off = [], 0
    for s in specs:
        offs.append(off)
        n = int(np.prod(s.shape)) * torch.tensor([], dtype=s.dtype).element_size()
        off += (n + _ALIGN - 1) // _ALIGN * _ALIGN
    return offs, max(off, _ALIGN)


class SharedCounters:
    """A page of int64 words in /dev/shm shared by every rank of the job: word 0 is the
    abort flag, then (committed, released) per channel, one cache line apart."""

    STRIDE = 8  # int64 words per counter (64 bytes)

    def __init__(self, n_channels: int, group=None):
        words = (1 + 2 * n_channels) * self.STRIDE
        nbytes = max(4096, words * 8)
        name = None
        if dist.get_rank() == 0:
            name = f"/dev/shm/revpp-ch-{uuid.uuid4().hex}"
            with open(name, "wb") as fh:
                fh.truncate(nbytes)
        obj = [name]
        dist.broadcast_object_list(obj, src=0)
        name = obj[0]
        fd = os.open(name, os.O_RDWR)
        try:
            self._mm = mmap.mmap(fd, nbytes, mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE)
        finally:
            os.close(fd)
        self.words = np.frombuffer(self._mm, dtype=np.int64, count=nbytes // 8)
        dist.barrier()
        if dist.get_rank() == 0:
            os.unlink(name)  # the mappings keep the page alive; nothing is left behind

    def _idx(self, ch: int, which: int) -> int:
        return (1 + 2 * ch + which) * self.STRIDE

    def get(self, ch: int, which: int) -> int:
        return int(self.words[self._idx(ch, which)])

    def set(self, ch: int, which: int, v: int) -> None:
        self.words[self._idx(ch, which)] = v

    @property
    def aborted(self) -> bool:
        return bool(self.words[0])

    def abort(self) -> None:
        self.words[0] = 1

    def wait_at_least(self, ch: int, which: int, v: int, what: str) -> None:
        if self.get(ch, which) >= v:
            return
        t0 = time.monotonic()
        limit = _host_timeout()
        spins = 0
        while self.get(ch, which) < v:
            if self.aborted:
                raise ChannelError(f"{what}: another rank aborted")
            if time.monotonic() - t0 > limit:
                self.abort()
                raise ChannelError(f"{what}: not reached within {limit:.0f} s (peer gone or stuck)")
            spins += 1
            time.sleep(0 if spins < 64 else 5e-5)


class _ChannelBase:
    COMMITTED, RELEASED = 0, 1

    def __init__(self, spec: ChannelSpec, index: int, counters: SharedCounters, rank: int):
        self.spec = spec
        self.index = index
        self.counters = counters
        self.rank = rank
        self.is_sender = rank == spec.src
        self.is_receiver = rank == spec.dst
        self.offs, self.slot_bytes = _layout(spec.specs)
        self.sent = 0        # next message index (sender)
        self.received = 0    # next message index (receiver)
        self._open_slot: Optional[int] = None  # sender: slot of the message being written
        self._cur: Optional[int] = None        # receiver: slot of the message being consumed

    # ---------------------------------------------------------------- sender
    def _begin(self) -> int:
        if self._open_slot is None:
            k = self.sent
            self.counters.wait_at_least(self.index, self.RELEASED, k - self.spec.depth + 1,
                                        f"channel {self.spec.name}: slot for message {k}")
            self._open_slot = k % self.spec.depth
            self._on_slot_free(self._open_slot, k)
        return self._open_slot

    def put(self, i: int, t: torch.Tensor) -> None:
        """Write tensor ``i`` of the current message (the first put claims a slot)."""
        s = self._begin()
        sp = self.spec.specs[i]
        if tuple(t.shape) != tuple(sp.shape) or t.dtype != sp.dtype:
            raise ValueError(f"channel {self.spec.name}: tensor {i} is {tuple(t.shape)}/{t.dtype}, "
                             f"expected {tuple(sp.shape)}/{sp.dtype}")
        self._copy(s, i, t.contiguous())

    def commit(self) -> None:
        s = self._begin()
        self._mark_ready(s)
        self.sent += 1
        self._open_slot = None
        self.counters.set(self.index, self.COMMITTED, self.sent)

    def send(self, tensors: Sequence[torch.Tensor]) -> None:
        for i, t in enumerate(tensors):
            self.put(i, t)
        self.commit()

    # ---------------------------------------------------------------- receiver
    def recv(self) -> List[torch.Tensor]:
        """Views of the next message's slot; the current stream is ordered after its copy."""
        if self._cur is not None:
            raise ChannelError(f"channel {self.spec.name}: previous message not released")
        k = self.received
        self.counters.wait_at_least(self.index, self.COMMITTED, k + 1, f"channel {self.spec.name}: message {k}")
        s = k % self.spec.depth
        self._wait_ready(s)
        self._cur = s
        return self._views(s)

    def release(self) -> None:
        """The work reading the current message has been enqueued: its slot may be refilled."""
        s = self._cur
        if s is None:
            raise ChannelError(f"channel {self.spec.name}: nothing to release")
        self._mark_free(s)
        self._cur = None
        self.received += 1
        self.counters.set(self.index, self.RELEASED, self.received)

    # ---------------------------------------------------------------- backend hooks
    def _copy(self, slot: int, i: int, t: torch.Tensor) -> None:
        raise NotImplementedError

    def _views(self, slot: int) -> List[torch.Tensor]:
        raise NotImplementedError

    def _on_slot_free(self, slot: int, k: int) -> None:
        pass

    def _mark_ready(self, slot: int) -> None:
        pass

    def _wait_ready(self, slot: int) -> None:
        pass

    def _mark_free(self, slot: int) -> None:
        pass

    def close(self) -> None:
        pass


def _views_of(buf: torch.Tensor, spec: ChannelSpec, offs: List[int], slot_bytes: int, slot: int):
    out = []
    base = slot * slot_bytes
    for s, o in zip(spec.specs, offs):
        n = int(np.prod(s.shape))
        esz = torch.tensor([], dtype=s.dtype).element_size()
        out.append(buf[base + o: base + o + n * esz].view(s.dtype).view(s.shape))
    return out


class HostChannel(_ChannelBase):
    """CPU channel: slots in a shared file mapped by sender and receiver."""

    def __init__(self, spec, index, counters, rank, path: str):
        super().__init__(spec, index, counters, rank)
        nbytes = spec.depth * self.slot_bytes
        self.buf = torch.from_file(path, shared=True, size=nbytes, dtype=torch.uint8)

    def _copy(self, slot, i, t):
        _views_of(self.buf, self.spec, self.offs, self.slot_bytes, slot)[i].copy_(t)

    def _views(self, slot):
        return _views_of(self.buf, self.spec, self.offs, self.slot_bytes, slot)


class CudaIpcChannel(_ChannelBase):
    """GPU channel: receive slots in the receiver's memory, written by the sender's copy
    engine through a CUDA IPC mapping; interprocess events order the two devices."""

    def __init__(self, spec, index, counters, rank, device, C):
        super().__init__(spec, index, counters, rank)
        self.device = device
        self.C = C
        self.buf = None
        self.peer_base = None
        self.ready: List[torch.cuda.Event] = []
        self.free: List[torch.cuda.Event] = []
        self.stream = None
        if self.is_receiver:
            self.buf = torch.empty(spec.depth * self.slot_bytes, dtype=torch.uint8, device=device)
            self.free = [torch.cuda.Event(interprocess=True) for _ in range(spec.depth)]
        if self.is_sender:
            self.ready = [torch.cuda.Event(interprocess=True) for _ in range(spec.depth)]
            self.stream = torch.cuda.Stream(device=device, priority=-1)
        self._keep: Dict[int, List[torch.Tensor]] = {}

    # exchange of handles (collective: called on every rank with every channel's export)
    def export(self):
        if self.is_receiver:
            return {"buf": self.C.ipc_export(self.buf), "free": [e.ipc_handle() for e in self.free]}
        if self.is_sender:
            return {"ready": [e.ipc_handle() for e in self.ready]}
        return None

    def attach(self, recv_exp, send_exp, opener) -> None:
        if self.is_sender:
            handle, off = recv_exp["buf"]
            self.peer_base = opener(handle) + int(off)
            self.free = [torch.cuda.Event.from_ipc_handle(self.device, h) for h in recv_exp["free"]]
        if self.is_receiver:
            self.ready = [torch.cuda.Event.from_ipc_handle(self.device, h) for h in send_exp["ready"]]

    def _on_slot_free(self, slot, k):
        if k >= self.spec.depth:  # the slot held message k - depth: wait until it was read
            self.stream.wait_event(self.free[slot])
        self.stream.wait_stream(torch.cuda.current_stream(self.device))

    def _copy(self, slot, i, t):
        dst = self.peer_base + slot * self.slot_bytes + self.offs[i]
        # the copy stream already waits on the current stream as of the slot claim; a later
        # put (a tensor produced since) needs the current stream's newer work too
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            self.C.copy_to_ptr(dst, t)
        t.record_stream(self.stream)

    def _mark_ready(self, slot):
        self.ready[slot].record(self.stream)

    def _wait_ready(self, slot):
        torch.cuda.current_stream(self.device).wait_event(self.ready[slot])

    def _mark_free(self, slot):
        self.free[slot].record(torch.cuda.current_stream(self.device))

    def _views(self, slot):
        return _views_of(self.buf, self.spec, self.offs, self.slot_bytes, slot)

    def close(self):
        if self.stream is not None:
            self.stream.synchronize()


class ChannelSet:
    """Every channel of the job, built collectively (all ranks, same list, same order).
    Each rank keeps the channels it sends or receives on."""

    def __init__(self, specs: Sequence[ChannelSpec], device: torch.device):
        self.rank = dist.get_rank()
        self.device = device
        self.specs = list(specs)
        self.counters = SharedCounters(len(self.specs))
        self.mine: Dict[str, _ChannelBase] = {}
        self._opened: Dict[bytes, int] = {}
        if device.type == "cuda":
            from revpp.ops import ext

            self.C = ext()
            chans = [CudaIpcChannel(s, i, self.counters, self.rank, device, self.C) for i, s in enumerate(self.specs)]
            exports = [c.export() for c in chans]
            allx = [None] * dist.get_world_size()
            dist.all_gather_object(allx, exports)
            with torch.cuda.device(device):
                for i, c in enumerate(chans):
                    if c.is_sender or c.is_receiver:
                        c.attach(allx[c.spec.dst][i], allx[c.spec.src][i], self._open)
            for c in chans:
                if c.is_sender or c.is_receiver:
                    self.mine[c.spec.name] = c
        else:
            paths = None
            if self.rank == 0:
                tag = uuid.uuid4().hex
                paths = [f"/dev/shm/revpp-slots-{tag}-{i}" for i in range(len(self.specs))]
                for p, s in zip(paths, self.specs):
                    _, sb = _layout(s.specs)
                    with open(p, "wb") as fh:
                        fh.truncate(sb * s.depth)
            obj = [paths]
            dist.broadcast_object_list(obj, src=0)
            paths = obj[0]
            for i, s in enumerate(self.specs):
                if self.rank in (s.src, s.dst):
                    self.mine[s.name] = HostChannel(s, i, self.counters, self.rank, paths[i])
            dist.barrier()
            if self.rank == 0:
                for p in paths:
                    os.unlink(p)
        dist.barrier()

    def _open(self, handle: bytes) -> int:
        if handle not in self._opened:
            self._opened[handle] = self.C.ipc_open(handle)
        return self._opened[handle]

    def get(self, name: str) -> Optional[_ChannelBase]:
        return self.mine.get(name)

    def abort(self) -> None:
        self.counters.abort()

    def close(self) -> None:
        for c in self.mine.values():
            c.close()
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
            for base in self._opened.values():
                self.C.ipc_close(base)
            self._opened.clear()


__all__ = ["ChannelSpec", "ChannelSet", "ChannelError", "SharedCounters", "HostChannel", "CudaIpcChannel"]
