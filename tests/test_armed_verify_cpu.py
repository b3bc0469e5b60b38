"""Host-side state machine of the target servers' armed verifies
(``P2PTargetServer.serve``, ``BatchedTargetServer.serve``), with the device parts replaced by fakes that
behave as the ``verify_arm`` kernel does: it takes the next message if one
arrives, and the armed verify is valid only for a VERIFY of the armed shape
and sequences.  Checks the order of backend calls and that the mailbox
sequence numbers stay in step with the messages and replies exchanged --
for valid arms, a RELEASE or CLOSE meeting an arm, a request that arrives
only after the arm's wait ran out, a change of batch shape, and rounds of
several drafters where one is late, releases or closes."""
import torch

from d3d_b200.engine import disagg


def _verify(sids_prefixes, K):
    B = len(sids_prefixes)
    words = [2, B, K, 0, 0, 0, 0, 0]
    for sid, p in sids_prefixes:
        words += [sid, p]
    for b in range(B):
        words += [100 + 10 * b + i for i in range(K)]
    return words


def _prefill(sid, toks):
    return [1, 1, len(toks), 0, 0, 0, 0, 0, sid, len(toks)] + list(toks)


def _release(sid):
    return [3, sid, 0, 0, 0, 0, 0, 0]


CLOSE = [0] * 8


class _Mailbox:
    def __init__(self):
        self.flag = torch.zeros(1, dtype=torch.int64)
        self.slots = [torch.zeros(1024, dtype=torch.uint8), torch.zeros(1024, dtype=torch.uint8)]

    def slot(self, seq):
        return self.slots[seq & 1]


class _Outbox:
    flag_ptr = 4096

    def slot_ptr(self, seq):
        return 8192 + 1024 * (seq & 1)


class _Link:
    supports_device_put = False     # no pinned buffers on CPU; the test turns the fused path on
    slot_bytes = 1 << 14

    def __init__(self, msgs):
        self.queue = list(msgs)
        self.recv_seq = self.send_seq = 0
        self.inbox, self.outbox = _Mailbox(), _Outbox()
        self.host_replies = []

    def recv(self, dst, stream, deadline_s=60.0, poll=None):
        m = self.queue.pop(0)
        self.recv_seq += 1
        d = dst.view(-1)
        d.zero_()
        d[:len(m)] = torch.tensor(m, dtype=torch.int64)
        return self.recv_seq

    def send(self, src, stream):
        self.send_seq += 1
        self.host_replies.append(int(src[0]))
        return self.send_seq

    def fetch(self, dst, offset, stream):
        pass


class _Ev:
    def synchronize(self):
        pass


class _Backend:
    """Target backend fake: records calls; ``arm_verify`` acts like the kernel."""
    hidden_size = 8
    runner = None
    stream = None
    supports_arm = True

    def __init__(self, link, reserved=1000):
        self.link, self.reserved = link, reserved
        self.log = []
        self.server = None
        self.late = set()          # arm calls (by count) whose request arrives after the wait
        self.arms = 0

    def prefill(self, group):
        self.log.append(("prefill", [s.index for s in group]))
        return torch.zeros(len(group), dtype=torch.long), torch.zeros(len(group), 8)

    def submit_verify(self, group, blocks, sink=None):
        self.log.append(("verify", [s.prefix for s in group]))

    def release(self, s):
        self.log.append(("release", s.index))

    def arm_verify(self, group, K, sids, src, rows_of, sink, head_words):
        self.arms += 1
        st = torch.full((9,), -1, dtype=torch.int32)
        lk = self.link
        assert int(src[3, 0]) == lk.recv_seq + 1          # waits for the next message
        if self.arms in self.late or not lk.queue:
            st[0], st[1] = 2, 1                            # nothing arrived in time
            self.log.append(("arm-timeout",))
        else:
            m = lk.queue.pop(0)
            req = self.server.req
            req.zero_()
            req[:len(m)] = torch.tensor(m, dtype=torch.int64)
            B = len(group)
            ok = m[0] == 2 and m[1] == B and m[2] == K and all(
                m[8 + 2 * b] == sids[b] and 0 <= m[9 + 2 * b] and m[9 + 2 * b] + K <= self.reserved
                for b in range(B))
            st[0] = 0 if ok else 1
            st[1] = 0 if ok else 1
            self.log.append(("armed", [m[9 + 2 * b] for b in range(B)]) if ok else ("arm-placeholder", m[0]))
        return {"ev": _Ev(), "status": st}


class _Ext:
    def accept_send(self, *a, **k):
        pass


class _Ops:
    @staticmethod
    def ext():
        return _Ext()


def _serve(monkeypatch, msgs, late=()):
    monkeypatch.setattr(disagg, "ops", _Ops)
    link = _Link(msgs)
    be = _Backend(link)
    be.late = set(late)
    srv = disagg.P2PTargetServer(be, link)
    srv.fused = True
    be.server = srv
    srv.serve()
    return srv, be, link


def test_armed_verifies_follow_the_request_stream(monkeypatch):
    msgs = [_prefill(7, [5, 6, 7]), _verify([(7, 3)], 4), _verify([(7, 5)], 4), _verify([(7, 9)], 4),
            _release(7), CLOSE]
    srv, be, link = _serve(monkeypatch, msgs)
    assert be.log == [("prefill", [7]), ("verify", [3]), ("armed", [5]), ("armed", [9]),
                      ("arm-placeholder", 3), ("release", 7)]
    assert link.recv_seq == 6 and not link.queue
    # replies: prefill and release from the host; one per verify from the device
    assert link.host_replies == [1, 3]
    assert link.send_seq == 5
    assert srv.served == 5


def test_request_after_the_arms_wait_and_a_shape_change(monkeypatch):
    msgs = [_prefill(7, [5, 6, 7]), _prefill(8, [1, 2]), _verify([(7, 3)], 4),
            _verify([(7, 5)], 4),                       # lands after the first arm gave up
            _verify([(7, 8), (8, 2)], 4),               # two sequences: not the armed shape
            _verify([(7, 12), (8, 6)], 4), _release(7), _release(8), CLOSE]
    srv, be, link = _serve(monkeypatch, msgs, late={1})
    assert be.log == [("prefill", [7]), ("prefill", [8]), ("verify", [3]), ("arm-timeout",), ("verify", [5]),
                      ("arm-placeholder", 2), ("verify", [8, 2]), ("armed", [12, 6]),
                      ("arm-placeholder", 3), ("release", 7), ("release", 8)]
    assert link.recv_seq == len(msgs) and not link.queue
    assert link.send_seq == 2 + 4 + 2        # two prefills, four verifies, two releases
    assert srv.seqs == {}


def test_armed_prefix_updates_reach_the_sequences(monkeypatch):
    msgs = [_prefill(7, [5, 6, 7]), _verify([(7, 3)], 4), _verify([(7, 6)], 4), CLOSE]
    srv, be, link = _serve(monkeypatch, msgs)
    assert srv.seqs[7].prefix == 6
    assert be.log[-1] == ("arm-placeholder", 0)


class _BatchedBackend(_Backend):
    """``arm_verify`` over several drafters' inboxes, as the kernel does it:
    valid only when every source sent a VERIFY of the armed shape."""

    def __init__(self, links):
        super().__init__(links[0])
        self.links = links
        self.subs = None

    def arm_verify(self, group, K, sids, src, rows_of, sink, head_words):
        self.arms += 1
        n = src.shape[1]
        st = torch.full((9,), -1, dtype=torch.int32)
        msgs = []
        for d in range(n):
            sub = next(s for s in self.subs if s.req.data_ptr() == int(src[2, d]))
            lk = sub.link
            assert int(src[3, d]) == lk.recv_seq + 1
            if (self.arms, d) in self.late or not lk.queue:
                msgs.append(None)
                continue
            m = lk.queue.pop(0)
            sub.req.zero_()
            sub.req[:len(m)] = torch.tensor(m, dtype=torch.int64)
            msgs.append(m)
        ok = all(m is not None for m in msgs)
        r = 0
        for d, m in enumerate(msgs):
            B = int(rows_of[1, d])
            if ok:
                ok = m[0] == 2 and m[1] == B and m[2] == K and all(m[8 + 2 * b] == sids[r + b] for b in range(B))
            r += B
        for d, m in enumerate(msgs):
            st[d] = 2 if m is None else (0 if ok else 1)
        st[n] = 0 if ok else 1
        self.log.append(("armed", [[m[9 + 2 * b] for b in range(m[1])] for m in msgs]) if ok else
                        ("arm-placeholder", [None if m is None else m[0] for m in msgs]))
        return {"ev": _Ev(), "status": st}


def _serve_batched(monkeypatch, streams, late=()):
    monkeypatch.setattr(disagg, "ops", _Ops)
    links = [_Link(s) for s in streams]
    be = _BatchedBackend(links)
    be.late = set(late)
    srv = disagg.BatchedTargetServer(be, links)
    for sub in srv.subs:
        sub.fused = True
    be.subs = srv.subs
    srv.serve()
    return srv, be, links


def test_batched_armed_rounds(monkeypatch):
    d0 = [_prefill(1, [5, 6]), _verify([(1, 2)], 4), _verify([(1, 5)], 4), _verify([(1, 9)], 4),
          _verify([(1, 12)], 4), _verify([(1, 15)], 4), _release(1), CLOSE]
    d1 = [_prefill(1, [7, 8, 9]), _verify([(1, 3)], 4), _verify([(1, 6)], 4), _verify([(1, 8)], 4),
          _release(1), CLOSE]
    srv, be, links = _serve_batched(monkeypatch, [d0, d1], late={(2, 1)})
    g0, g1 = 0 * srv.ID_STRIDE + 1, 1 * srv.ID_STRIDE + 1
    assert be.log == [
        ("prefill", [g0, g1]),
        ("verify", [2, 3]),                # the second serving round runs on the host; the next is armed
        ("armed", [[5], [6]]),             # the third on the device
        ("arm-placeholder", [2, None]),    # drafter 1's request lands after the wait ...
        ("verify", [9, 8]),                # ... so the fourth runs on the host
        ("arm-placeholder", [2, 3]),       # drafter 1 releases: the fifth runs on the host
        ("verify", [12]), ("release", g1),
        ("verify", [15]),                  # drafter 1 closes in this round: nothing armed
        ("release", g0),
    ]
    assert all(lk.recv_seq == n for lk, n in zip(links, (len(d0), len(d1))))
    assert [lk.send_seq for lk in links] == [1 + 5 + 1, 1 + 3 + 1]
    assert srv.seqs == {}
