"""Point-to-point mailboxes between two GPU processes over NVLink.

A :class:`Mailbox` is a device allocation owned by the *receiving* GPU::

    [ flag: int64 (own 256-byte line) | slot 0 | slot 1 ]

Its CUDA IPC handle is sent to the peer process, which maps it
(:class:`PeerMailbox`) and writes into it with its own kernels: the payload
with plain stores through the peer pointer, then the sequence number with a
system-scope release store (``handoff_put``).  The receiver's
``handoff_wait`` kernel spins with acquire loads on the flag -- bounded by a
2 s limit, after which it sets an error status instead of hanging -- and
copies the payload out.  Message ``seq`` uses slot ``seq & 1``; the
request/reply protocol of the users keeps at most one message in flight per
direction, so a slot is never overwritten while it is read.

Only plain peer loads and stores are used (no multicast object, no NVLS), so
a peer that dies leaves the survivor with a timed-out wait, not a fault.
The reference moves the same messages through a ``multiprocessing`` Pipe
between host processes (``single/eval_async_packed.py:56-346``).
"""
from __future__ import annotations

import time
from typing import Optional

import torch
import torch.distributed as dist

from .. import ops

FLAG_BYTES = 256


class Mailbox:
    """Receive side, on this process's GPU."""

    def __init__(self, slot_bytes: int, device: torch.device):
        if slot_bytes % 256:
            slot_bytes += 256 - slot_bytes % 256
        self.slot_bytes = slot_bytes
        self.device = torch.device(device)
        self.nbytes = FLAG_BYTES + 2 * slot_bytes
        self.ext = ops.ext()
        self.ptr = self.ext.mailbox_alloc(self.nbytes, self.device.index)
        self.mem = self.ext.mailbox_view(self.ptr, self.nbytes, self.device.index)
        self.flag = self.mem[:8].view(torch.int64)
        # written by the wait kernel through the unified address space
        self.status = torch.zeros(1, dtype=torch.int32, pin_memory=True)

    def slot(self, seq: int) -> torch.Tensor:
        off = FLAG_BYTES + (seq & 1) * self.slot_bytes
        return self.mem[off:off + self.slot_bytes]

    def handle(self) -> bytes:
        return self.ext.ipc_handle(self.ptr, self.device.index)

    def wait(self, seq: int, dst: Optional[torch.Tensor], stream: torch.cuda.Stream,
             deadline_s: float = 60.0, poll=None) -> None:
        """Copy message ``seq`` into ``dst`` once it has arrived.  ``dst`` is a
        contiguous tensor of at most one slot, on this GPU or in pinned host
        memory (then the kernel writes it directly and no copy follows).  The
        in-kernel wait is bounded; the host re-arms it until ``deadline_s``,
        and ``poll()`` (if given) may raise to abort."""
        t_end = time.monotonic() + deadline_s
        src = self.slot(seq) if dst is not None else None
        dstb = dst.view(-1).view(torch.uint8) if dst is not None else None
        while True:
            self.status[0] = -1
            with torch.cuda.stream(stream):
                self.ext.handoff_wait(self.flag, seq, src, dstb, self.status)
            stream.synchronize()
            if int(self.status[0]) == 0:
                return
            if poll is not None:
                poll()
            if time.monotonic() > t_end:
                raise TimeoutError(f"no message {seq} from the peer within {deadline_s:.0f} s")

    def close(self) -> None:
        if self.ptr:
            torch.cuda.synchronize(self.device)
            self.ext.mailbox_free(self.ptr, self.device.index)
            self.ptr = 0


class PeerMailbox:
    """Send side: the peer's :class:`Mailbox` mapped into this process."""

    def __init__(self, handle: bytes, slot_bytes: int, device: torch.device):
        self.device = torch.device(device)
        self.slot_bytes = slot_bytes
        self.ext = ops.ext()
        self.base = self.ext.ipc_open(handle, self.device.index)
        self.flag_ptr = self.base
        self.ticket = torch.zeros(1, dtype=torch.int32, device=self.device)

    def slot_ptr(self, seq: int) -> int:
        return self.base + FLAG_BYTES + (seq & 1) * self.slot_bytes

    def put(self, src: torch.Tensor, seq: int, stream: torch.cuda.Stream) -> None:
        """Stream-ordered: copy ``src`` (device, contiguous) into slot ``seq & 1``
        of the peer's mailbox, then publish ``seq``."""
        nb = src.numel() * src.element_size()
        if nb > self.slot_bytes:
            raise ValueError(f"message of {nb} bytes exceeds the {self.slot_bytes}-byte slot")
        with torch.cuda.stream(stream):
            self.ext.handoff_put(src, self.slot_ptr(seq), self.flag_ptr, seq, self.ticket)

    def close(self) -> None:
        if self.base:
            torch.cuda.synchronize(self.device)
            self.ext.ipc_close(self.base, self.device.index)
            self.base = 0


class Link:
    """A bidirectional channel between this rank and ``peer``: an inbox here
    and the peer's inbox mapped for sending.  Both ranks construct it
    (collectively over ``group``) with the same ``slot_bytes``."""

    supports_device_put = True

    def __init__(self, peer: int, slot_bytes: int, device: torch.device, group=None):
        self.peer = peer
        self.device = torch.device(device)
        self.inbox = Mailbox(slot_bytes, self.device)
        world = dist.get_world_size(group)
        handles = [None] * world
        dist.all_gather_object(handles, (dist.get_rank(group), self.inbox.handle()), group=group)
        mine = None
        for r, h in handles:
            if r == peer:
                mine = h
        if mine is None:
            raise RuntimeError(f"rank {peer} did not publish a mailbox")
        self.outbox = PeerMailbox(mine, self.inbox.slot_bytes, self.device)
        self.send_seq = 0
        self.recv_seq = 0

    @property
    def slot_bytes(self) -> int:
        return self.inbox.slot_bytes

    def send(self, src: torch.Tensor, stream: torch.cuda.Stream) -> int:
        self.send_seq += 1
        self.outbox.put(src, self.send_seq, stream)
        return self.send_seq

    def recv(self, dst: Optional[torch.Tensor], stream: torch.cuda.Stream, deadline_s: float = 60.0,
             poll=None) -> int:
        """Wait for the next message and copy its first ``dst.nbytes`` bytes."""
        self.recv_seq += 1
        self.inbox.wait(self.recv_seq, dst, stream, deadline_s, poll)
        return self.recv_seq

    def fetch(self, dst: torch.Tensor, offset: int, stream: torch.cuda.Stream) -> None:
        """Copy more of the last received message (bytes ``offset ..``) into
        ``dst``; valid until the peer's next-but-one message."""
        src = self.inbox.slot(self.recv_seq)
        d = dst.reshape(-1).view(torch.uint8)
        with torch.cuda.stream(stream):
            d.copy_(src[offset:offset + d.numel()], non_blocking=True)
        stream.synchronize()

    def close(self, group=None) -> None:
        """Unmap the peer's inbox, wait until the peer has unmapped ours
        (barrier over ``group``), then free it."""
        self.outbox.close()
        if dist.is_initialized():
            dist.barrier(group=group)
        self.inbox.close()


class HostLink:
    """The :class:`Link` interface over ``torch.distributed`` point-to-point
    messages (``gloo`` between CPU processes): every message is one slot of
    ``slot_bytes``.  Used where there is no GPU pair (tests, CPU runs)."""

    supports_device_put = False

    def __init__(self, peer: int, slot_bytes: int, group=None):
        self.peer = peer
        self.group = group
        self.slot_bytes = (slot_bytes + 255) // 256 * 256
        self.buf_out = torch.zeros(self.slot_bytes, dtype=torch.uint8)
        self.buf_in = torch.zeros(self.slot_bytes, dtype=torch.uint8)
        self.send_seq = 0
        self.recv_seq = 0

    def send(self, src: torch.Tensor, stream=None) -> int:
        b = src.reshape(-1).view(torch.uint8)
        if b.numel() > self.slot_bytes:
            raise ValueError(f"message of {b.numel()} bytes exceeds the {self.slot_bytes}-byte slot")
        self.buf_out[: b.numel()] = b.cpu()
        dist.send(self.buf_out, self.peer, group=self.group)
        self.send_seq += 1
        return self.send_seq

    def recv(self, dst: Optional[torch.Tensor], stream=None, deadline_s: float = 60.0, poll=None) -> int:
        dist.recv(self.buf_in, self.peer, group=self.group)
        if dst is not None:
            d = dst.reshape(-1).view(torch.uint8)
            d.copy_(self.buf_in[: d.numel()])
        self.recv_seq += 1
        return self.recv_seq

    def fetch(self, dst: torch.Tensor, offset: int, stream=None) -> None:
        d = dst.reshape(-1).view(torch.uint8)
        d.copy_(self.buf_in[offset:offset + d.numel()])

    def close(self, group=None) -> None:
        pass
