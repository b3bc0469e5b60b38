"""Target service in another process (another GPU, or another CPU process).

The reference runs its target in a spawned process and ships Python lists
through a ``multiprocessing`` Pipe (``serving/target_process.py:9-139``,
``single/eval_async_packed.py:56-346``).  Here the two sides are ranks of a
``torch.distributed`` process group (``gloo`` between CPU processes, or
between the host sides of two GPU processes) and exchange fixed-layout int64
/ float32 tensors:

=========  =====================================  ===================================
command    request                                reply
=========  =====================================  ===================================
PREFILL    meta [n, 2] (seq id, length), tokens   anchors [n], hidden [n, H]
VERIFY     meta [B, 2] (seq id, prefix), blocks   [B, 2+K] (commit, corr, posterior),
           [B, K]                                 hidden [B, H]
RELEASE    seq id                                 (none)
CLOSE      —                                      (none)
=========  =====================================  ===================================

Every message starts with an 8-int64 header.  A server-side exception is
returned as an ERROR header followed by the UTF-8 traceback, and re-raised by
the client (``serving/target_process.py:59-66``).  Liveness relies on the
process group's timeout: a peer that died or never joined ends the next
collective with an error instead of hanging.

The verify request is sent non-blocking, so the drafter runs its packed
all-outcome forward while the target verifies — the asynchronous overlap of
the reference, across processes.
"""
from __future__ import annotations

import traceback
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from ..engine.backends import SeqState, TargetBackend, VerifyResult

CMD_CLOSE, CMD_PREFILL, CMD_VERIFY, CMD_RELEASE, CMD_ERROR = 0, 1, 2, 3, -1
HDR = 8


def _hdr(*vals) -> torch.Tensor:
    h = torch.zeros(HDR, dtype=torch.int64)
    h[: len(vals)] = torch.tensor(vals, dtype=torch.int64)
    return h


class TargetServer:
    """Serves a :class:`TargetBackend` to one client rank."""

    def __init__(self, backend: TargetBackend, client_rank: int, group=None):
        self.be = backend
        self.peer = client_rank
        self.group = group
        self.seqs: Dict[int, SeqState] = {}

    def _send_error(self, exc: BaseException) -> None:
        msg = ("".join(traceback.format_exception(exc))).encode()[:65536]
        dist.send(_hdr(CMD_ERROR, len(msg)), self.peer, group=self.group)
        dist.send(torch.frombuffer(bytearray(msg), dtype=torch.uint8), self.peer, group=self.group)

    def serve(self) -> None:
        H = int(self.be.hidden_size)
        while True:
            h = torch.empty(HDR, dtype=torch.int64)
            dist.recv(h, self.peer, group=self.group)
            cmd = int(h[0])
            if cmd == CMD_CLOSE:
                return
            try:
                if cmd == CMD_RELEASE:
                    s = self.seqs.pop(int(h[1]), None)
                    if s is not None:
                        self.be.release(s)
                    continue
                if cmd == CMD_PREFILL:
                    n, total = int(h[1]), int(h[2])
                    meta = torch.empty(n, 2, dtype=torch.int64)
                    toks = torch.empty(total, dtype=torch.int64)
                    dist.recv(meta, self.peer, group=self.group)
                    dist.recv(toks, self.peer, group=self.group)
                    group, off = [], 0
                    for sid, ln in meta.tolist():
                        s = SeqState(index=sid, prompt=toks[off:off + ln].tolist(), prefix=ln)
                        off += ln
                        self.seqs[sid] = s
                        group.append(s)
                    anchors, hidden = self.be.prefill(group)
                    hid = (hidden.float().cpu() if hidden is not None else torch.zeros(n, H))
                    dist.send(_hdr(CMD_PREFILL, n, H), self.peer, group=self.group)
                    dist.send(anchors.to(torch.int64).cpu().contiguous(), self.peer, group=self.group)
                    dist.send(hid.contiguous(), self.peer, group=self.group)
                    continue
                if cmd == CMD_VERIFY:
                    B, K = int(h[1]), int(h[2])
                    meta = torch.empty(B, 2, dtype=torch.int64)
                    blocks = torch.empty(B, K, dtype=torch.int64)
                    dist.recv(meta, self.peer, group=self.group)
                    dist.recv(blocks, self.peer, group=self.group)
                    group = []
                    for sid, prefix in meta.tolist():
                        s = self.seqs[sid]
                        s.prefix = prefix
                        group.append(s)
                    r = self.be.verify(group, blocks)
                    out = torch.cat([r.commit.view(B, 1).to(torch.int64).cpu(),
                                     r.correction.view(B, 1).to(torch.int64).cpu(),
                                     r.posterior.to(torch.int64).cpu().view(B, K)], 1).contiguous()
                    hid = r.hidden.float().cpu().contiguous() if r.hidden is not None else torch.zeros(B, H)
                    dist.send(_hdr(CMD_VERIFY, B, K, H), self.peer, group=self.group)
                    dist.send(out, self.peer, group=self.group)
                    dist.send(hid, self.peer, group=self.group)
                    continue
                raise ValueError(f"unknown target command {cmd}")
            except Exception as exc:  # reported to the client, server keeps serving
                self._send_error(exc)


class RemoteTarget(TargetBackend):
    """Client side: a :class:`TargetBackend` whose target lives on ``server_rank``."""

    def __init__(self, server_rank: int, hidden_size: int, group=None):
        self.peer = server_rank
        self.group = group
        self.hidden_size = hidden_size
        self._pending: Optional[tuple] = None
        self._reqs: List = []
        self.closed = False

    def _recv_header(self, expect: int) -> torch.Tensor:
        h = torch.empty(HDR, dtype=torch.int64)
        dist.recv(h, self.peer, group=self.group)
        if int(h[0]) == CMD_ERROR:
            msg = torch.empty(int(h[1]), dtype=torch.uint8)
            dist.recv(msg, self.peer, group=self.group)
            raise RuntimeError("target service failed:\n" + bytes(msg.tolist()).decode(errors="replace"))
        if int(h[0]) != expect:
            raise RuntimeError(f"target protocol error: expected {expect}, got {int(h[0])}")
        return h

    def prefill(self, seqs: List[SeqState]):
        meta = torch.tensor([[s.index, len(s.prompt)] for s in seqs], dtype=torch.int64)
        toks = torch.tensor([t for s in seqs for t in s.prompt], dtype=torch.int64)
        dist.send(_hdr(CMD_PREFILL, len(seqs), toks.numel()), self.peer, group=self.group)
        dist.send(meta, self.peer, group=self.group)
        dist.send(toks, self.peer, group=self.group)
        h = self._recv_header(CMD_PREFILL)
        n, H = int(h[1]), int(h[2])
        anchors = torch.empty(n, dtype=torch.int64)
        hid = torch.empty(n, H, dtype=torch.float32)
        dist.recv(anchors, self.peer, group=self.group)
        dist.recv(hid, self.peer, group=self.group)
        return anchors, hid

    def submit_verify(self, seqs, blocks, q=None):
        if q is not None:
            raise NotImplementedError("the remote target verifies greedily (temperature 0)")
        if self._pending is not None:
            raise RuntimeError("target already has an outstanding verify")
        B, K = blocks.shape
        meta = torch.tensor([[s.index, s.prefix] for s in seqs], dtype=torch.int64)
        blk = blocks.to(torch.int64).cpu().contiguous()
        self._reqs = [dist.isend(_hdr(CMD_VERIFY, B, K), self.peer, group=self.group),
                      dist.isend(meta, self.peer, group=self.group),
                      dist.isend(blk, self.peer, group=self.group)]
        self._pending = (B, K, meta, blk)   # keep the send buffers alive

    def receive(self) -> VerifyResult:
        if self._pending is None:
            raise RuntimeError("no outstanding target request")
        B, K, _, _ = self._pending
        try:
            for r in self._reqs:
                r.wait()
            h = self._recv_header(CMD_VERIFY)
            H = int(h[3])
            out = torch.empty(B, 2 + K, dtype=torch.int64)
            hid = torch.empty(B, H, dtype=torch.float32)
            dist.recv(out, self.peer, group=self.group)
            dist.recv(hid, self.peer, group=self.group)
        finally:
            self._pending = None
            self._reqs = []
        return VerifyResult(out[:, 0], out[:, 1], out[:, 2:], hid)

    def release(self, seq: SeqState) -> None:
        dist.send(_hdr(CMD_RELEASE, seq.index), self.peer, group=self.group)

    def close(self) -> None:
        if not self.closed:
            self.closed = True
            dist.send(_hdr(CMD_CLOSE), self.peer, group=self.group)
