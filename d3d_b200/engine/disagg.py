"""Disaggregated decode: the target on one GPU, the drafter on another.

This is the reference's two-GPU arrangement (verifier process on its own
device, drafter and coordinator in the main process,
``single/eval_async_packed.py:56-346,796-1297``), built on the NVLink
mailboxes of :mod:`d3d_b200.parallel.p2p` instead of a host Pipe:

* the coordinator (:class:`~d3d_b200.engine.spec.SpecDecoder`) runs on the
  drafter's rank with a :class:`P2PTarget` as its target backend;
* :class:`P2PTargetServer` runs on the target's rank around a
  :class:`~d3d_b200.engine.fast.FastTarget`.

Every message is a run of int64 words in one mailbox slot, starting with an
8-word header (the same messages travel over ``torch.distributed`` between
CPU processes through :class:`~d3d_b200.parallel.p2p.HostLink`,
:mod:`d3d_b200.serving.remote`):

=========  ==========================================  ==========================================
command    request (drafter -> target)                 reply (target -> drafter)
=========  ==========================================  ==========================================
PREFILL    [1, n, total] meta[n, 2] tokens[total]      [1, n, H] anchors[n] | hidden bf16 [n, H]
VERIFY     [2, B, K] meta[B, 2] blocks[B, K]           [2, B, K, H] res[B, 2+K] | hidden bf16 [B, H]
RELEASE    [3, seq id]                                 [3]
CLOSE      [0]                                         (none)
ERROR      --                                          [-1, nbytes] utf-8 traceback
=========  ==========================================  ==========================================

``meta`` rows are (sequence id, prefix length); ``res`` rows are (commit,
correction, posterior[K]).  The bf16 hidden block starts at byte
:func:`hidden_offset`.  The VERIFY reply is written by the ``accept_send``
kernel straight from the verify graph's buffers into the drafter GPU's
mailbox (acceptance, correction, hidden-state pick and the NVLink transfer in
one launch); the drafter's ``handoff_wait`` kernel writes it into pinned host
memory, so the coordinator reads it after one stream synchronize.
"""
from __future__ import annotations

import os
import traceback
from typing import Dict, List, Optional

import numpy as np
import torch

from .. import ops
from .backends import SeqState, TargetBackend, VerifyResult

CMD_CLOSE, CMD_PREFILL, CMD_VERIFY, CMD_RELEASE, CMD_ERROR = 0, 1, 2, 3, -1
HDR = 8
HEAD_WORDS = 512          # first 4 KB of a message; the rest is fetched on demand
DEFAULT_SLOT_BYTES = 1 << 20


def hidden_offset(n_words: int) -> int:
    """Byte offset of the bf16 hidden block after ``n_words`` int64 words."""
    return (8 * n_words + 255) // 256 * 256


def _prefill_words(n: int) -> int:
    return HDR + n


def _verify_words(B: int, K: int) -> int:
    return HDR + B * (2 + K)


class P2PTargetServer:
    """Serves a :class:`~d3d_b200.engine.fast.FastTarget` to the drafter rank
    at the other end of ``link``."""

    def __init__(self, backend, link, deadline_s: float = 600.0, replies: str = "all"):
        """``replies="ack"`` is for the ranks of a tensor-parallel target other
        than rank 0: they run every command but answer only RELEASE (an
        acknowledgement), since rank 0's replies carry the results."""
        self.be = backend
        self.link = link
        self.deadline_s = deadline_s
        if replies not in ("all", "ack"):
            raise ValueError("replies must be 'all' or 'ack'")
        self.replies = replies
        self.seqs: Dict[int, SeqState] = {}
        self.H = int(backend.hidden_size)
        # fused path: the verify graph's accept kernel writes the reply into the
        # drafter GPU's mailbox (a FastTarget on one end of an NVLink Link)
        self.fused = bool(getattr(link, "supports_device_put", False)) and hasattr(backend, "runner")
        pin = bool(getattr(link, "supports_device_put", False))
        self.req = torch.empty(link.slot_bytes // 8, dtype=torch.int64, pin_memory=pin)
        self.rep_host = torch.zeros(link.slot_bytes // 8, dtype=torch.int64, pin_memory=pin)
        self.stream = getattr(backend, "stream", None)
        self.served = 0

    # ------------------------------------------------------------ replies
    def _reply_host(self, n_words: int) -> None:
        """Send the first ``n_words`` of ``rep_host`` (rounded to 16 bytes)."""
        n = (n_words + 1) // 2 * 2
        self.link.send(self.rep_host[:n], self.stream)
        if self.stream is not None:
            self.stream.synchronize()   # rep_host is reused by the next reply

    def _send_error(self, exc: BaseException) -> None:
        msg = ("".join(traceback.format_exception(exc))).encode()
        cap = self.link.slot_bytes - 8 * HDR
        msg = msg[:cap]
        self.rep_host[:HDR] = 0
        self.rep_host[0] = CMD_ERROR
        self.rep_host[1] = len(msg)
        body = self.rep_host[HDR:].view(torch.uint8)
        body[: len(msg)] = torch.frombuffer(bytearray(msg), dtype=torch.uint8)
        self._reply_host(HDR + (len(msg) + 7) // 8)

    # ---------------------------------------------------------- commands
    def _prefill(self, h) -> None:
        n, total = int(h[1]), int(h[2])
        meta = self.req[HDR:HDR + 2 * n].view(n, 2).tolist()
        toks = self.req[HDR + 2 * n:HDR + 2 * n + total].tolist()
        group, off = [], 0
        for sid, ln in meta:
            s = SeqState(index=sid, prompt=toks[off:off + ln], prefix=ln)
            off += ln
            self.seqs[sid] = s
            group.append(s)
        anchors, hidden = self.be.prefill(group)
        if self.replies != "all":
            return
        words = _prefill_words(n)
        ho = hidden_offset(words)
        self.rep_host[:HDR] = 0
        self.rep_host[0], self.rep_host[1], self.rep_host[2] = CMD_PREFILL, n, self.H
        self.rep_host[HDR:HDR + n] = anchors.to(torch.int64).cpu()
        hb = self.rep_host.view(torch.uint8)[ho:ho + 2 * n * self.H].view(torch.bfloat16)
        hb.copy_(hidden.to(torch.bfloat16).reshape(-1).cpu())
        self._reply_host((ho + 2 * n * self.H + 7) // 8)

    def _verify(self, h) -> list:
        """Run one VERIFY; returns its sequences (in request order)."""
        B, K, S = int(h[1]), int(h[2]), int(h[3])
        meta = self.req[HDR:HDR + 2 * B].view(B, 2).tolist()
        end = HDR + 2 * B + B * K
        blocks = self.req[HDR + 2 * B:end].view(B, K).clone()
        q = None
        if S:       # sampled verify: the drafts' sparse proposal follows the blocks
            n = B * (K - 1) * S
            q = (self.req[end:end + n].view(B, K - 1, S).clone(),
                 self.req[end + n:end + 2 * n].clone().view(torch.float64).view(B, K - 1, S).float())
        group = []
        for sid, prefix in meta:
            s = self.seqs[sid]
            s.prefix = prefix
            group.append(s)
        if self.replies != "all":
            if self.fused and q is None:
                self.be.submit_verify(group, blocks, sink=lambda ids, post, xn: None)
            else:
                self.be.verify(group, blocks, q)
            return group
        if not self.fused or q is not None:
            r = self.be.verify(group, blocks, q)
            words = _verify_words(B, K)
            ho = hidden_offset(words)
            self.rep_host[:HDR] = 0
            self.rep_host[0], self.rep_host[1], self.rep_host[2], self.rep_host[3] = CMD_VERIFY, B, K, self.H
            res = torch.cat([r.commit.view(B, 1).to(torch.int64).cpu(), r.correction.view(B, 1).to(torch.int64).cpu(),
                             r.posterior.to(torch.int64).cpu().view(B, K)], 1)
            self.rep_host[HDR:words] = res.reshape(-1)
            hb = self.rep_host.view(torch.uint8)[ho:ho + 2 * B * self.H].view(torch.bfloat16)
            if r.hidden is not None:
                hb.copy_(r.hidden.to(torch.bfloat16).reshape(-1).cpu())
            self._reply_host((ho + 2 * B * self.H + 7) // 8)
            return group
        seq = self.link.send_seq + 1
        self.link.send_seq = seq
        out_ptr = self.link.outbox.slot_ptr(seq)
        hid_ptr = out_ptr + hidden_offset(_verify_words(B, K))
        flag_ptr = self.link.outbox.flag_ptr
        E = ops.ext()

        def sink(ids, post, xn):
            E.accept_send(ids, post, xn, out_ptr, hid_ptr, flag_ptr, seq)

        self.be.submit_verify(group, blocks, sink=sink)
        return group

    # ------------------------------------------------------ armed verifies
    def _can_arm(self) -> bool:
        return (self.fused and getattr(self.be, "supports_arm", False)
                and os.environ.get("D3D_ARMED_VERIFY", "1") != "0")

    def _arm(self, group: list, K: int):
        """Enqueue the verify of ``group``'s next block before its request
        exists (``FastTarget.arm_verify``): the request is read from the inbox
        on the device, and the reply goes out from the device as before."""
        lk = self.link
        seq_in, seq_out = lk.recv_seq + 1, lk.send_seq + 1
        B = len(group)
        src = torch.tensor([[lk.inbox.flag.data_ptr()], [lk.inbox.slot(seq_in).data_ptr()],
                            [self.req.data_ptr()], [seq_in]], dtype=torch.int64)
        rows_of = torch.tensor([[0], [B]], dtype=torch.int64)
        out_ptr = lk.outbox.slot_ptr(seq_out)
        hid_ptr = out_ptr + hidden_offset(_verify_words(B, K))
        flag_ptr = lk.outbox.flag_ptr
        E = ops.ext()

        def sink(ids, post, xn, gate):
            if self.replies == "all":     # other tensor-parallel ranks run the verify, rank 0 answers
                E.accept_send(ids, post, xn, out_ptr, hid_ptr, flag_ptr, seq_out, gate)

        arm = self.be.arm_verify(group, K, [s.index for s in group], src, rows_of, sink, HEAD_WORDS)
        return arm, group, seq_in, seq_out

    def _armed_outcome(self, armed) -> str:
        """``"verified"`` (the armed verify ran on the request and replied),
        ``"message"`` (another message arrived: its head is in ``req``) or
        ``"none"`` (nothing arrived within the kernel's bounded wait)."""
        arm, group, seq_in, seq_out = armed
        arm["ev"].synchronize()
        st0, overall = int(arm["status"][0]), int(arm["status"][1])
        if overall == 3:
            raise RuntimeError("armed verify: no decision from tensor-parallel rank 0, or messages unlike it")
        if overall == 0:
            self.link.recv_seq = seq_in
            if self.replies == "all":
                self.link.send_seq = seq_out
            B = len(group)
            for (sid, prefix), s in zip(self.req[HDR:HDR + 2 * B].view(B, 2).tolist(), group):
                s.prefix = prefix
            return "verified"
        if st0 == 1:
            self.link.recv_seq = seq_in
            return "message"
        return "none"

    def serve(self, poll=None) -> None:
        """Answer requests until CLOSE.  ``poll()`` is called whenever a
        bounded wait for the next request ran out (it may raise to stop).
        On a GPU link with a greedy single-GPU target, every VERIFY is
        followed at once by an armed verify of the same sequences, so the
        next request starts verifying the moment it lands."""
        armed = None
        while True:
            have = False
            if armed is not None:
                kind = self._armed_outcome(armed)
                group = armed[1]
                armed = None
                if kind == "verified":
                    self.served += 1
                    armed = self._arm(group, int(self.req[2]))
                    continue
                have = kind == "message"
            if not have:
                self.link.recv(self.req[:HEAD_WORDS], self.stream, deadline_s=self.deadline_s, poll=poll)
            h = self.req[:HDR].tolist()
            cmd = h[0]
            chk = getattr(self.be, "check_tp", None)
            if chk is not None:
                chk()   # a failed tensor-parallel exchange ends serving loudly
            words = 0
            if cmd == CMD_PREFILL:
                words = HDR + 2 * h[1] + h[2]
            elif cmd == CMD_VERIFY:
                words = HDR + 2 * h[1] + h[1] * h[2] + 2 * h[1] * (h[2] - 1) * h[3]
            if words > HEAD_WORDS:
                self.link.fetch(self.req[HEAD_WORDS:words], 8 * HEAD_WORDS, self.stream)
            if cmd == CMD_CLOSE:
                return
            try:
                if cmd == CMD_VERIFY:
                    group = self._verify(h)
                    if self._can_arm():
                        armed = self._arm(group, int(h[2]))
                elif cmd == CMD_PREFILL:
                    self._prefill(h)
                elif cmd == CMD_RELEASE:
                    s = self.seqs.pop(int(h[1]), None)
                    if s is not None:
                        self.be.release(s)
                    self.rep_host[:HDR] = 0
                    self.rep_host[0] = CMD_RELEASE
                    self._reply_host(HDR)
                else:
                    raise ValueError(f"unknown target command {cmd}")
                self.served += 1
            except Exception as exc:  # reported to the drafter; the server keeps serving
                if self.replies != "all":
                    raise   # rank 0 of the group reports the failure (its exchange waits time out)
                self._send_error(exc)


class P2PTarget(TargetBackend):
    """Drafter-side target backend whose target is served over ``link``."""

    def __init__(self, link, hidden_size: int, device=None, deadline_s: float = 600.0,
                 want_hidden: bool = True, draft_stream=None):
        """``link`` may be a list: the links to every rank of a tensor-parallel
        target (rank 0 first).  Requests go to all of them; results come from
        rank 0, and RELEASE waits for every rank's acknowledgement.
        ``draft_stream``: the drafter's stream; with it (and GPU links) the
        coordinator may submit a verify whose drafts are still being computed
        -- the request is assembled on the device behind the drafter's
        in-flight forward and sent from there (``gather``)."""
        self.links = list(link) if isinstance(link, (list, tuple)) else [link]
        link = self.links[0]
        self.link = link
        self.want_hidden = want_hidden
        self.hidden_size = int(hidden_size)
        gpu = bool(getattr(link, "supports_device_put", False))
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.deadline_s = deadline_s
        self.stream = torch.cuda.Stream(device=self.device, priority=-1) if gpu else None
        words = link.slot_bytes // 8
        self.req = torch.zeros(words, dtype=torch.int64, pin_memory=gpu)
        self.rep = torch.zeros(words, dtype=torch.int64, pin_memory=gpu)
        self._pending: Optional[tuple] = None
        self.closed = False
        self.draft_stream = draft_stream
        self.supports_gather = gpu and draft_stream is not None
        self.dev_req = torch.zeros(words, dtype=torch.int64, device=self.device) if self.supports_gather \
            else None
        # device branch select (``arm_select``): pinned status, table buffers
        self._armed: Optional[tuple] = None
        self._sent = False
        if self.supports_gather:
            self.sel_status = torch.zeros(2, dtype=torch.int32, pin_memory=True)
            self.sel_ev = torch.cuda.Event()
            self._tab_h = torch.zeros(4096, dtype=torch.int64, pin_memory=True)
            self._tab_d = torch.zeros(4096, dtype=torch.int64, device=self.device)

    def _send(self, n_words: int) -> None:
        n = (n_words + 1) // 2 * 2
        # the put kernels read the pinned request directly
        for lk in self.links:
            lk.send(self.req[:n], self.stream)

    def _recv(self, expect: int, head_words: int = HEAD_WORDS):
        head_words = min(max(head_words, HDR), self.rep.numel())
        head_words += head_words % 2
        self.link.recv(self.rep[:head_words], self.stream, deadline_s=self.deadline_s)
        cmd = int(self.rep[0])
        if cmd == CMD_ERROR:
            nb = int(self.rep[1])
            if HDR + (nb + 7) // 8 > head_words:
                self.link.fetch(self.rep[head_words:HDR + (nb + 7) // 8 + 1], 8 * head_words, self.stream)
            msg = bytes(self.rep[HDR:].view(torch.uint8)[:nb].tolist()).decode(errors="replace")
            raise RuntimeError("target service failed:\n" + msg)
        if cmd != expect:
            raise RuntimeError(f"target protocol error: expected {expect}, got {cmd}")
        return self.rep

    def _bf16_block(self, words: int, rows: int, have_words: int) -> torch.Tensor:
        """The hidden block of the last reply, fetched if it was not in the head."""
        ho = hidden_offset(words)
        nb = 2 * rows * self.hidden_size
        end = (ho + nb + 15) // 16 * 16
        if end > 8 * have_words:
            lo = 8 * have_words
            self.link.fetch(self.rep.view(torch.uint8)[lo:end], lo, self.stream)
        return self.rep.view(torch.uint8)[ho:ho + nb].view(torch.bfloat16).view(rows, self.hidden_size)

    def prefill(self, seqs: List[SeqState]):
        n = len(seqs)
        toks = [t for s in seqs for t in s.prompt]
        need = HDR + 2 * n + len(toks)
        if 8 * need > self.link.slot_bytes:
            raise ValueError("prompts exceed the mailbox slot; raise slot_bytes")
        self.req[:HDR] = 0
        self.req[0], self.req[1], self.req[2] = CMD_PREFILL, n, len(toks)
        self.req[HDR:HDR + 2 * n] = torch.tensor([[s.index, len(s.prompt)] for s in seqs]).view(-1)
        self.req[HDR + 2 * n:need] = torch.tensor(toks, dtype=torch.int64)
        self._send(need)
        r = self._recv(CMD_PREFILL)
        anchors = r[HDR:HDR + n].clone()
        hid = self._bf16_block(_prefill_words(n), n, HEAD_WORDS).clone()
        return anchors, hid

    def submit_verify(self, seqs, blocks, q=None, gather=None):
        """Send a verify request.  ``gather`` (see ``FastTarget.submit_verify``):
        the request is ordered after the drafter's work enqueued so far, its
        listed block entries are taken on the device from the drafter's
        output, and the put kernels send it from device memory."""
        if self._pending is not None:
            raise RuntimeError("target already has an outstanding verify")
        B, K = blocks.shape
        need = HDR + 2 * B + B * K
        S = 0 if q is None else int(q[0].shape[-1])
        if S and gather is not None:
            raise RuntimeError("sampled verifies are sent from the host (no device-assembled request)")
        total = need + 2 * B * (K - 1) * S
        if 8 * total > self.link.slot_bytes:
            raise ValueError(f"verify request of {8 * total} bytes exceeds the {self.link.slot_bytes}-byte slot "
                             "(raise slot_bytes, or sample drafts from a proposal top-k)")
        self.req[:HDR] = 0
        self.req[0], self.req[1], self.req[2], self.req[3] = CMD_VERIFY, B, K, S
        meta = np.array([[s.index, s.prefix] for s in seqs], dtype=np.int64).reshape(-1)
        rn = self.req.numpy()
        rn[HDR:HDR + 2 * B] = meta
        rn[HDR + 2 * B:need] = blocks.numpy().reshape(-1)
        if S:
            # sparse proposal of drafts 1..K-1: support ids, then probabilities as float64 bit patterns
            n = B * (K - 1) * S
            rn[need:need + n] = q[0].to(torch.int64).cpu().numpy().reshape(-1)
            rn[need + n:need + 2 * n] = q[1].to(torch.float64).cpu().numpy().reshape(-1).view(np.int64)
            need = total
        if gather is None:
            self._send(need)
        else:
            if not self.supports_gather or need > self.dev_req.numel():
                raise RuntimeError("device-assembled requests need GPU links and a drafter stream")
            n = (need + 1) // 2 * 2
            with torch.cuda.stream(self.stream):
                # ordered after the drafter's in-flight forward: a request never
                # leaves before the drafts it carries exist
                self.stream.wait_stream(self.draft_stream)
                dev = self.dev_req[:n]
                dev.copy_(self.req[:n], non_blocking=True)
                body = self.dev_req[HDR + 2 * B:]
                for src, dst, rws in gather:
                    d = torch.as_tensor(dst, dtype=torch.int64).to(self.device, non_blocking=True)
                    r = torch.as_tensor(rws, dtype=torch.int64).to(self.device, non_blocking=True)
                    body.index_copy_(0, d, src[:, 0].index_select(0, r))
            for lk in self.links:
                lk.send(self.dev_req[:n], self.stream)
        self._pending = (B, K)

    @property
    def supports_select(self) -> bool:
        return self.supports_gather and os.environ.get("D3D_DEVICE_SELECT", "1") != "0"

    def arm_select(self, B: int, K: int, nk: int, a0: bool, n_eos: int, ctrl: bool, top, tab: List[int]) -> bool:
        """Enqueue the ``select_send`` kernel for the outstanding verify: behind
        the drafter's forward (whose ``top`` ids it reads), it waits for the
        reply and, when every row continues on a drafted branch, sends the
        next VERIFY to the target itself.  ``tab`` is the kernel's table
        (sequence ids, prefixes, finishing limits, branch keys and rows, stop
        tokens, controlled drafts).  ``receive`` then reads the reply the
        kernel copied; ``select_sent`` says whether the request went out."""
        if self._pending is None or self._armed is not None or not self.supports_select:
            return False
        n = len(tab)
        if n > self._tab_h.numel():
            self._tab_h = torch.zeros(2 * n, dtype=torch.int64, pin_memory=True)
            self._tab_d = torch.zeros(2 * n, dtype=torch.int64, device=self.device)
        self._tab_h[:n] = torch.tensor(tab, dtype=torch.int64)
        lk = self.link
        rseq = lk.recv_seq + 1
        words = _verify_words(B, K)
        hw = words + words % 2
        outs = torch.tensor([[l.outbox.slot_ptr(l.send_seq + 1) for l in self.links],
                             [l.outbox.flag_ptr for l in self.links],
                             [l.send_seq + 1 for l in self.links]], dtype=torch.int64)
        self.sel_status.fill_(-1)
        E = ops.ext()
        with torch.cuda.stream(self.stream):
            self.stream.wait_stream(self.draft_stream)
            self._tab_d[:n].copy_(self._tab_h[:n], non_blocking=True)
            E.select_send(lk.inbox.flag, lk.inbox.slot(rseq).view(torch.int64), rseq, self.rep[:hw], B, K, nk, a0,
                          n_eos, ctrl, top, self._tab_d, outs, self.sel_status)
            self.sel_ev.record(self.stream)
        self._armed = (rseq, B, K)
        return True

    def select_sent(self) -> bool:
        """Whether the device sent the next VERIFY (valid after ``receive``)."""
        return self._sent

    def adopt_sent(self, B: int, K: int) -> None:
        """Record the request the device sent as the outstanding verify."""
        if self._pending is not None:
            raise RuntimeError("target already has an outstanding verify")
        self._sent = False
        self._pending = (B, K)

    def receive(self) -> VerifyResult:
        if self._pending is None:
            raise RuntimeError("no outstanding target request")
        B, K = self._pending
        self._pending = None
        words = _verify_words(B, K)
        armed, self._armed = self._armed, None
        self._sent = False
        if armed is not None:
            rseq = armed[0]
            self.sel_ev.synchronize()
            if int(self.sel_status[0]) == 0:
                # the reply is in; its head is in ``rep`` already
                self.link.recv_seq = rseq
                if int(self.rep[0]) == CMD_ERROR:
                    self.link.recv_seq -= 1     # re-read it through the error path below
                    r = self._recv(CMD_VERIFY, words)
                if int(self.rep[0]) != CMD_VERIFY:
                    raise RuntimeError(f"target protocol error: expected {CMD_VERIFY}, got {int(self.rep[0])}")
                r = self.rep
                if int(self.sel_status[1]) == 1:
                    self._sent = True
                    for lk in self.links:
                        lk.send_seq += 1
            else:
                r = self._recv(CMD_VERIFY, words)
        else:
            r = self._recv(CMD_VERIFY, words)
        res = r[HDR:words].view(B, 2 + K).clone()
        hid = self._bf16_block(words, B, words + words % 2).clone() if self.want_hidden else None
        return VerifyResult(res[:, 0], res[:, 1], res[:, 2:], hid)

    def verify(self, seqs, blocks, q=None):
        self.submit_verify(seqs, blocks, q)
        return self.receive()

    def release(self, seq: SeqState) -> None:
        self.req[:HDR] = 0
        self.req[0], self.req[1] = CMD_RELEASE, seq.index
        self._send(HDR)
        self._recv(CMD_RELEASE, HDR)
        for lk in self.links[1:]:
            lk.recv(self.rep[:HDR], self.stream, deadline_s=self.deadline_s)
            if int(self.rep[0]) != CMD_RELEASE:
                raise RuntimeError("tensor-parallel target rank did not acknowledge RELEASE")

    def close(self) -> None:
        """Ends the server's current ``serve()`` call (it may be called again)."""
        self.closed = True
        self.req[:HDR] = 0
        self.req[0] = CMD_CLOSE
        self._send(HDR)
        if self.stream is not None:
            self.stream.synchronize()


class BatchedTargetServer:
    """One target serving several drafter ranks, each at the end of its own
    link (the multi-GPU layout: target on T GPUs, tensor-parallel, drafters
    on the other GPUs, one request stream each).

    Every drafter keeps exactly one request outstanding (the coordinator
    sends a verify, then waits for its reply), so the server works in rounds:
    it takes one message from each drafter still open, runs all PREFILLs of
    the round as one batched prefill and all VERIFYs as one batched verify
    (one forward over every drafter's blocks), and answers each drafter in
    its own mailbox -- on GPU links by one fused accept+send launch per
    drafter on its rows of the verify output.  Sequence ids are made unique
    per drafter before they reach the backend.  The ranks of a
    tensor-parallel target all run the same rounds (every drafter sends to
    every rank), so their forwards and exchanges stay in step; only rank 0
    answers (``replies="ack"`` elsewhere, which still acknowledges RELEASE).
    ``serve()`` returns when every drafter has sent CLOSE."""

    ID_STRIDE = 1 << 32

    def __init__(self, backend, links, deadline_s: float = 600.0, replies: str = "all"):
        self.be = backend
        self.subs = [P2PTargetServer(backend, lk, deadline_s=deadline_s, replies=replies) for lk in links]
        self.replies = replies
        self.deadline_s = deadline_s
        self.seqs: Dict[int, SeqState] = {}
        self.H = int(backend.hidden_size)
        self.served = 0
        self.rounds = 0

    def _gid(self, d: int, sid: int) -> int:
        return d * self.ID_STRIDE + int(sid)

    def _recv(self, d: int, poll=None) -> list:
        sub = self.subs[d]
        sub.link.recv(sub.req[:HEAD_WORDS], sub.stream, deadline_s=self.deadline_s, poll=poll)
        h = sub.req[:HDR].tolist()
        if h[0] == CMD_PREFILL:
            words = HDR + 2 * h[1] + h[2]
            if words > HEAD_WORDS:
                sub.link.fetch(sub.req[HEAD_WORDS:words], 8 * HEAD_WORDS, sub.stream)
        return h

    # ---------------------------------------------------------- commands
    def _prefill(self, items) -> None:
        group, spans = [], []
        for d, h in items:
            sub = self.subs[d]
            n, total = int(h[1]), int(h[2])
            meta = sub.req[HDR:HDR + 2 * n].view(n, 2).tolist()
            toks = sub.req[HDR + 2 * n:HDR + 2 * n + total].tolist()
            off = 0
            for sid, ln in meta:
                s = SeqState(index=self._gid(d, sid), prompt=toks[off:off + ln], prefix=ln)
                off += ln
                self.seqs[s.index] = s
                group.append(s)
            spans.append((d, len(group) - n, n))
        anchors, hidden = self.be.prefill(group)
        if self.replies != "all":
            return
        anchors = anchors.to(torch.int64).cpu()
        hidden = hidden.to(torch.bfloat16).cpu()
        for d, r0, n in spans:
            sub = self.subs[d]
            words = _prefill_words(n)
            ho = hidden_offset(words)
            sub.rep_host[:HDR] = 0
            sub.rep_host[0], sub.rep_host[1], sub.rep_host[2] = CMD_PREFILL, n, self.H
            sub.rep_host[HDR:HDR + n] = anchors[r0:r0 + n]
            hb = sub.rep_host.view(torch.uint8)[ho:ho + 2 * n * self.H].view(torch.bfloat16)
            hb.copy_(hidden[r0:r0 + n].reshape(-1))
            sub._reply_host((ho + 2 * n * self.H + 7) // 8)

    def _verify(self, items) -> None:
        group, blocks, spans, K = [], [], [], None
        for d, h in items:
            sub = self.subs[d]
            B, k = int(h[1]), int(h[2])
            if int(h[3]):
                raise NotImplementedError("the batched target verifies greedily (no proposal in the request)")
            if K is not None and k != K:
                raise ValueError("drafters verify blocks of different sizes in one round")
            K = k
            meta = sub.req[HDR:HDR + 2 * B].view(B, 2).tolist()   # (sequence id, prefix)
            blocks.append(sub.req[HDR + 2 * B:HDR + 2 * B + B * K].view(B, K).clone())
            for sid, prefix in meta:
                s = self.seqs[self._gid(d, sid)]
                s.prefix = prefix
                group.append(s)
            spans.append((d, len(group) - B, B))
        blocks = torch.cat(blocks)
        fused = self.subs[0].fused
        self._last_verify = (group, K)
        if self.replies != "all":
            if fused:
                self.be.submit_verify(group, blocks, sink=lambda ids, post, xn: None)
            else:
                self.be.verify(group, blocks)
            return
        if not fused:
            r = self.be.verify(group, blocks)
            for d, r0, B in spans:
                sub = self.subs[d]
                words = _verify_words(B, K)
                ho = hidden_offset(words)
                sub.rep_host[:HDR] = 0
                sub.rep_host[0], sub.rep_host[1], sub.rep_host[2], sub.rep_host[3] = CMD_VERIFY, B, K, self.H
                res = torch.cat([r.commit[r0:r0 + B].view(B, 1).to(torch.int64).cpu(),
                                 r.correction[r0:r0 + B].view(B, 1).to(torch.int64).cpu(),
                                 r.posterior[r0:r0 + B].to(torch.int64).cpu().view(B, K)], 1)
                sub.rep_host[HDR:words] = res.reshape(-1)
                if r.hidden is not None:
                    hb = sub.rep_host.view(torch.uint8)[ho:ho + 2 * B * self.H].view(torch.bfloat16)
                    hb.copy_(r.hidden[r0:r0 + B].to(torch.bfloat16).reshape(-1).cpu())
                sub._reply_host((ho + 2 * B * self.H + 7) // 8)
            return
        outs = []
        for d, r0, B in spans:
            lk = self.subs[d].link
            seq = lk.send_seq + 1
            lk.send_seq = seq
            out_ptr = lk.outbox.slot_ptr(seq)
            outs.append((r0, B, out_ptr, out_ptr + hidden_offset(_verify_words(B, K)), lk.outbox.flag_ptr, seq))
        E = ops.ext()

        def sink(ids, post, xn):
            for r0, B, out_ptr, hid_ptr, flag_ptr, seq in outs:
                E.accept_send(ids[r0:r0 + B], post[r0:r0 + B], xn[r0 * K:(r0 + B) * K], out_ptr, hid_ptr,
                              flag_ptr, seq)

        self.be.submit_verify(group, blocks, sink=sink)

    # ------------------------------------------------------ armed rounds
    def _arm_round(self, ds: List[int], group: list, K: int):
        """Enqueue the next round's merged verify before its requests exist
        (``FastTarget.arm_verify`` over every drafter's inbox, rows in the
        order of the round just enqueued); each drafter's reply goes out from
        the device behind it, gated on all requests matching."""
        src = [[], [], [], []]
        rows_of = [[], []]
        exp, outs, r0 = [], [], 0
        for d in ds:
            sub = self.subs[d]
            lk = sub.link
            B = sum(1 for s in group if s.index // self.ID_STRIDE == d)
            seq_in, seq_out = lk.recv_seq + 1, lk.send_seq + 1
            for col, v in zip(src, (lk.inbox.flag.data_ptr(), lk.inbox.slot(seq_in).data_ptr(),
                                   sub.req.data_ptr(), seq_in)):
                col.append(v)
            rows_of[0].append(r0)
            rows_of[1].append(B)
            exp += [s.index % self.ID_STRIDE for s in group[r0:r0 + B]]
            out_ptr = lk.outbox.slot_ptr(seq_out)
            outs.append((d, r0, B, out_ptr, out_ptr + hidden_offset(_verify_words(B, K)), lk.outbox.flag_ptr,
                         seq_out, seq_in))
            r0 += B
        if r0 != len(group):
            return None
        E = ops.ext()

        def sink(ids, post, xn, gate):
            if self.replies != "all":    # other tensor-parallel ranks run the verify, rank 0 answers
                return
            for d, q0, B, out_ptr, hid_ptr, flag_ptr, seq_out, _ in outs:
                E.accept_send(ids[q0:q0 + B], post[q0:q0 + B], xn[q0 * K:(q0 + B) * K], out_ptr, hid_ptr,
                              flag_ptr, seq_out, gate)

        arm = self.be.arm_verify(group, K, exp, torch.tensor(src, dtype=torch.int64),
                                 torch.tensor(rows_of, dtype=torch.int64), sink, HEAD_WORDS)
        return arm, ds, group, K, outs

    def _armed_round(self, armed):
        """Outcome of an armed round: ``(True, {})`` when its verify ran on
        every drafter's request, else ``(False, heads)`` with the headers of
        the messages that did arrive (the others are still to be received)."""
        arm, ds, group, K, outs = armed
        arm["ev"].synchronize()
        st = arm["status"]
        if int(st[len(ds)]) == 3:
            raise RuntimeError("armed verify: no decision from tensor-parallel rank 0, or messages unlike it")
        if int(st[len(ds)]) == 0:
            for d, q0, B, _, _, _, seq_out, seq_in in outs:
                sub = self.subs[d]
                sub.link.recv_seq = seq_in
                if self.replies == "all":
                    sub.link.send_seq = seq_out
                for (sid, prefix), s in zip(sub.req[HDR:HDR + 2 * B].view(B, 2).tolist(), group[q0:q0 + B]):
                    s.prefix = prefix
            return True, {}
        heads = {}
        for i, (d, _, _, _, _, _, _, seq_in) in enumerate(outs):
            if int(st[i]) == 1:
                sub = self.subs[d]
                sub.link.recv_seq = seq_in
                h = sub.req[:HDR].tolist()
                if h[0] == CMD_PREFILL:
                    words = HDR + 2 * h[1] + h[2]
                    if words > HEAD_WORDS:
                        sub.link.fetch(sub.req[HEAD_WORDS:words], 8 * HEAD_WORDS, sub.stream)
                heads[d] = h
        return False, heads

    def _release(self, d: int, sid: int) -> None:
        s = self.seqs.pop(self._gid(d, sid), None)
        if s is not None:
            self.be.release(s)
        sub = self.subs[d]
        sub.rep_host[:HDR] = 0
        sub.rep_host[0] = CMD_RELEASE
        sub._reply_host(HDR)

    def serve(self, poll=None) -> None:
        active = list(range(len(self.subs)))
        can_arm = (self.subs[0].fused and getattr(self.be, "supports_arm", False)
                   and os.environ.get("D3D_ARMED_VERIFY", "1") != "0")
        armed = None
        while active:
            heads = {}
            if armed is not None:
                done, heads = self._armed_round(armed)
                prev, armed = armed, None
                if done:
                    self.rounds += 1
                    self.served += len(prev[1])
                    armed = self._arm_round(prev[1], prev[2], prev[3])
                    continue
            msgs = [(d, heads[d] if d in heads else self._recv(d, poll)) for d in active]
            chk = getattr(self.be, "check_tp", None)
            if chk is not None:
                chk()   # a failed tensor-parallel exchange ends serving loudly
            self.rounds += 1
            by = {}
            for d, h in msgs:
                by.setdefault(h[0], []).append((d, h))
            batches = [(self._prefill, by.pop(CMD_PREFILL, []))]
            by_k = {}
            for d, h in by.pop(CMD_VERIFY, []):     # one batched verify per block size
                by_k.setdefault(int(h[2]), []).append((d, h))
            batches += [(self._verify, by_k[k]) for k in sorted(by_k)]
            # a round of nothing but one verify from every open drafter arms the next
            arm_next = (can_arm and len(by_k) == 1 and not batches[0][1] and len(by) == 0
                        and len(next(iter(by_k.values()))) == len(active))
            for run, items in batches:
                if not items:
                    continue
                try:
                    run(items)
                    self.served += len(items)
                except Exception as exc:  # every drafter of the batch hears about it
                    if self.replies != "all":
                        raise
                    arm_next = False
                    for d, _ in items:
                        self.subs[d]._send_error(exc)
            for d, h in by.pop(CMD_RELEASE, []):
                self._release(d, int(h[1]))
                self.served += 1
            closed = {d for d, _ in by.pop(CMD_CLOSE, [])}
            for kind, items in by.items():
                for d, _ in items:
                    if self.replies == "all":
                        self.subs[d]._send_error(ValueError(f"unknown target command {kind}"))
            active = [d for d in active if d not in closed]
            if arm_next and active:
                group, K = self._last_verify
                armed = self._arm_round([d for d, _ in next(iter(by_k.values()))], group, K)
