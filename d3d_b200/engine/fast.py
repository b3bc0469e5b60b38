"""Target and draft backends on the sm_100a kernels (one GPU, two streams).

The target verifies on its own CUDA stream while the drafter's packed
all-outcome forward runs on a second stream of the same GPU (the 1-GPU
configuration: target and drafter co-located; the reference needs two GPUs
and a process boundary, ``single/eval_async_packed.py:216-346``).

Every decode-shaped forward (verify ``B x K``, AR ``B x 1``, recovery
``B x K``, packed ``B x (K + branches*K)``) is captured once in a CUDA graph
and replayed; only the small integer inputs (token ids, RoPE positions, KV
slots, row descriptors) are copied in per step, from pinned host memory.
Greedy acceptance runs on the device inside the target's graph
(``greedy_accept`` kernel) and copies the hidden state that produced the
correction token for the conditioned drafter.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from .. import ops
from ..config import ModelConfig
from ..utils import launches
from ..utils.timing import NULL as _NULL_PROF
from ..models.fast import FastRunner, FastWeights, PagedKV, StepBuffers
from .backends import DraftBackend, SeqState, TargetBackend, VerifyResult
from .layout import causal_rows, prefix_rows
from .sampling import is_greedy, pq_accept_sparse


def K_of(blocks) -> int:
    """Block width (tokens per sequence) of a verify request."""
    return int(blocks.shape[1])


class _GraphCache:
    def __init__(self, runner: FastRunner, stream: torch.cuda.Stream, use_graphs: bool = True):
        self.r = runner
        self.stream = stream
        self.use_graphs = use_graphs
        self.graphs: Dict[tuple, torch.cuda.CUDAGraph] = {}
        self.counts: Dict[tuple, int] = {}
        self.pool = None

    def run(self, key, b: StepBuffers, fn):
        """Run ``fn(b)`` on the stream, through a CUDA graph captured on first use."""
        if not self.use_graphs:
            with torch.cuda.stream(self.stream):
                launches.add(fn(b) or 0)
            return
        g = self.graphs.get(key)
        if g is None:
            with torch.cuda.stream(self.stream):
                fn(b)      # warm-up (module attributes, TMA descriptor caches)
            self.stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream, pool=self.pool):
                self.counts[key] = fn(b) or 0
            if self.pool is None:
                self.pool = g.pool()
            self.graphs[key] = g
        with torch.cuda.stream(self.stream):
            g.replay()
        launches.add(self.counts[key])


class _Pinned:
    """Reusable pinned staging buffers keyed by name."""

    def __init__(self):
        self.bufs: Dict[str, torch.Tensor] = {}

    def get(self, name, n, dtype):
        t = self.bufs.get(name)
        if t is None or t.numel() < n or t.dtype != dtype:
            t = torch.empty(max(n, 64), dtype=dtype, pin_memory=True)
            self.bufs[name] = t
        return t[:n]


def _stage(pin: _Pinned, name: str, arr: np.ndarray, dst: torch.Tensor, stream) -> None:
    h = pin.get(name, arr.size, dst.dtype)
    h.numpy()[...] = arr.reshape(-1)
    with torch.cuda.stream(stream):
        dst.view(-1)[: arr.size].copy_(h, non_blocking=True)


class _FastModelBackend:
    def __init__(self, weights: FastWeights, *, pages: int, page_size: int, max_seqs: int,
                 max_context: int, extra_slots: int, batch_invariant: bool, use_graphs: bool,
                 device="cuda", stream: Optional[torch.cuda.Stream] = None, tp=None):
        self.w = weights
        self.cfg: ModelConfig = weights.cfg
        self.device = torch.device(device)
        max_pages_seq = math.ceil((max_context + extra_slots) / page_size)
        self.kv = PagedKV(self.cfg, pages, page_size, max_seqs, max_pages_seq, device)
        self.runner = FastRunner(weights, self.kv, max_context=max_context + extra_slots,
                                 batch_invariant=batch_invariant, device=device, tp=tp)
        self.stream = stream or torch.cuda.Stream(device=self.device)
        self.graphs = _GraphCache(self.runner, self.stream, use_graphs)
        self.pin = _Pinned()
        self.prof = _NULL_PROF
        self.rows_of: Dict[int, int] = {}           # seq index -> block-table row
        self.free_rows: List[int] = list(range(max_seqs - 1, -1, -1))
        self.extra_slots = extra_slots
        self.max_context = max_context

    def _row(self, s: SeqState) -> int:
        r = self.rows_of.get(s.index)
        if r is None:
            if not self.free_rows:
                raise RuntimeError("too many concurrent sequences for this backend")
            r = self.rows_of[s.index] = self.free_rows.pop()
        return r

    def leak_check(self) -> None:
        """Raise if a sequence still holds pages or the allocator lost some
        (called when a decode run has finished every request)."""
        if self.kv.tables or self.kv.leaked:
            raise RuntimeError(f"KV pages leaked: {len(self.kv.tables)} sequences still allocated, "
                               f"{self.kv.leaked} pages unaccounted for")

    def _release(self, s: SeqState) -> None:
        r = self.rows_of.pop(s.index, None)
        if r is not None:
            self.free_rows.append(r)
        self.kv.release(s.index)

    def _fill(self, b: StepBuffers, seqs: List[SeqState], ids: np.ndarray, pos: np.ndarray,
              rows: np.ndarray, kv_end: np.ndarray, tag: str, cond_rows=None) -> None:
        """Write one forward's integer inputs into the pinned twin of ``b.inbuf``
        and copy them to the device with a single transfer."""
        q = b.Q
        for i, s in enumerate(seqs):
            b.h_slots[i * q:(i + 1) * q] = self.kv.slots(s.index, s.prefix, q)
        b.h_ids[:] = ids.reshape(-1)
        b.h_pos[:] = pos.reshape(-1)
        b.h_rows[:] = rows.reshape(-1, 3)
        b.h_kv_end[:] = kv_end.reshape(-1)
        b.h_seq_rows[:] = [self._row(s) for s in seqs]
        if cond_rows is not None:
            b.h_cond_rows[:] = cond_rows.reshape(-1)
        with torch.cuda.stream(self.stream):
            b.inbuf.copy_(b.inbuf_host, non_blocking=True)

    @torch.inference_mode()
    def hidden_states(self, ids: torch.Tensor) -> torch.Tensor:
        """Final-norm hidden states ``[B, L, H]`` of one causal forward over
        ``ids`` ``[B, L]`` (every row of every sequence; no LM head, no KV
        kept afterwards).  Used for the frozen teacher of distillation."""
        B, L = ids.shape
        seqs = [SeqState(index=-(i + 1), prompt=[], prefix=0) for i in range(B)]
        try:
            for s in seqs:
                self.kv.reserve(s.index, self._row(s), L)
            b = self.runner.buffers(B, L, 0, prefill=True)
            rows = np.broadcast_to(causal_rows(0, L).numpy()[None], (B, L, 3))
            pos = np.broadcast_to(np.arange(L, dtype=np.int64)[None], (B, L))
            self._fill(b, seqs, ids.cpu().numpy(), pos, rows, np.full(B, L, dtype=np.int64), "hs")
            with torch.cuda.stream(self.stream):
                launches.add(self.runner.forward(b))
                out = b.xn.view(B, L, -1).clone()
            torch.cuda.current_stream(self.device).wait_stream(self.stream)
            out.record_stream(torch.cuda.current_stream(self.device))
            return out
        finally:
            for s in seqs:
                self._release(s)

    def _prefill_one(self, s: SeqState, rows: np.ndarray, topk: int, reserve: int):
        n = len(s.prompt)
        self.kv.reserve(s.index, self._row(s), reserve)
        b = StepBuffers(self.cfg, 1, n, topk, 1, self.runner.splits(n), self.device,
                        fused_norm=self.runner.fused_norm)
        b.bt_view = torch.zeros(1, self.kv.max_pages_per_seq, dtype=torch.int32, device=self.device)
        b.chunk = self.runner.chunk_for(prefill=True)
        saved = s.prefix
        s.prefix = 0
        self._fill(b, [s], np.array(s.prompt), np.arange(n), rows, np.array([n]), "pf")
        s.prefix = saved
        with torch.cuda.stream(self.stream):
            launches.add(self.runner.forward(b))
        # the pinned staging buffers are reused by the next call
        self.stream.synchronize()
        return b


class FastTarget(_FastModelBackend, TargetBackend):
    """Greedy target verification on the kernels."""

    def __init__(self, weights: FastWeights, *, pages: int = 4096, page_size: int = 16,
                 max_seqs: int = 16, max_context: int = 4096, use_graphs: bool = True,
                 device="cuda", stream=None, tp=None, temperature: float = 0.0, top_k: int = 0,
                 top_p: float = 1.0, seed: int = 0):
        """``tp``: a :class:`~d3d_b200.parallel.tp.TPGroup` when ``weights`` is one
        shard of a tensor-parallel target (every rank of the group then runs
        the same calls in the same order).

        ``temperature > 0`` turns on lossless speculative sampling against the
        target's distribution.  With ``top_k`` in 1..4 the fused top-k
        epilogue of the LM head gives exactly the logits of the truncated
        distribution (no logits are materialised); with ``top_k = 0`` (the
        full vocabulary, the reference's default) or ``top_k > 4`` the LM-head
        GEMM writes the fp32 logits of the verified rows (B*K rows, about 10
        MB for a 16-token block) and the distribution is formed on the device
        (temperature, top-k, then ``top_p``)."""
        super().__init__(weights, pages=pages, page_size=page_size, max_seqs=max_seqs,
                         max_context=max_context, extra_slots=64, batch_invariant=True,
                         use_graphs=use_graphs, device=device, stream=stream, tp=tp)
        self.hidden_size = self.cfg.hidden_size
        self.tp = tp
        self._pending = None
        self._arm_bufs: Dict[int, dict] = {}
        self._arm_epoch = 0       # armed verifies so far: the same count on every tensor-parallel rank
        self.scratch = self.kv.scratch_slot()
        self._accept_bufs: Dict[tuple, dict] = {}
        self.verify_events: List[Tuple[torch.cuda.Event, torch.cuda.Event]] = []
        self.time_verify = False
        self.temperature, self.top_k, self.top_p = float(temperature), int(top_k), float(top_p)
        self.sampled = not is_greedy(self.temperature)
        self.full_vocab = self.sampled and not 1 <= self.top_k <= 4
        # LM-head mode of sampled forwards: fused top-k (1..4) or full logits (-1)
        self.lm_k = -1 if self.full_vocab else self.top_k
        if self.sampled:
            if self.top_k < 0:
                raise ValueError("target top_k must be >= 0")
            if tp is not None:
                raise NotImplementedError("sampled verification with a tensor-parallel target")
            self.gen = torch.Generator(device=self.device)
            self.gen.manual_seed(int(seed))
        if tp is not None:
            # every rank is ready before the first exchange, so no rank's
            # bounded flag wait runs out while a peer still initialises
            import torch.distributed as dist
            torch.cuda.synchronize(self.device)
            if dist.is_initialized():
                dist.barrier(group=tp.group)

    def check_tp(self) -> None:
        """Raise if a tensor-parallel exchange of this rank ran out of its
        bounded wait (results since then are not valid)."""
        if self.tp is not None and int(self.tp.status.item()) != 0:
            raise RuntimeError(f"tensor-parallel exchange failed on rank {self.tp.rank} "
                               f"(status {int(self.tp.status.item())})")

    @torch.inference_mode()
    def prefill(self, seqs):
        anchors, hid = [], []
        for s in seqs:
            n = len(s.prompt)
            rows = causal_rows(0, n).numpy()
            b = self._prefill_one(s, rows, topk=self.lm_k if self.sampled else 1,
                                  reserve=self.max_context + 64)
            with torch.cuda.stream(self.stream):
                if self.full_vocab:
                    pr = self._probs_full(b.logits[n - 1:n])
                    a = torch.multinomial(pr, 1, generator=self.gen)[0, 0]
                elif self.sampled:
                    pr = self._probs(b.top_v[n - 1:n])
                    a = b.top_i[n - 1].gather(0, torch.multinomial(pr, 1, generator=self.gen)[0])[0]
                else:
                    a = b.top_i[n - 1, 0].clone()
                h = b.xn[n - 1].clone()
            anchors.append(a)
            hid.append(h)
        self.stream.synchronize()
        return torch.stack(anchors).cpu(), torch.stack(hid)

    def _abufs(self, B, K):
        key = (B, K)
        a = self._accept_bufs.get(key)
        if a is None:
            dev = self.device
            a = dict(commit=torch.zeros(B, dtype=torch.int64, device=dev),
                     corr=torch.zeros(B, dtype=torch.int64, device=dev),
                     hid=torch.zeros(B, self.cfg.hidden_size, dtype=torch.bfloat16, device=dev),
                     h_commit=torch.zeros(B, dtype=torch.int64, pin_memory=True),
                     h_corr=torch.zeros(B, dtype=torch.int64, pin_memory=True),
                     h_post=torch.zeros(B * K, dtype=torch.int64, pin_memory=True),
                     ev=torch.cuda.Event())
            self._accept_bufs[key] = a
        return a

    def _probs(self, top_v: torch.Tensor) -> torch.Tensor:
        """Sampling distribution over the top-k logits (temperature, then top-p)."""
        sl = top_v.float() / self.temperature
        if self.top_p < 1.0:
            pr = torch.softmax(sl, -1)
            remove = pr.cumsum(-1) > self.top_p
            remove[..., 1:] = remove[..., :-1].clone()
            remove[..., 0] = False
            sl = sl.masked_fill(remove, float("-inf"))
        return torch.softmax(sl, -1)

    def _probs_full(self, logits: torch.Tensor) -> torch.Tensor:
        """Sampling distribution over the whole vocabulary from fp32 logits
        ``[..., V]``: temperature, then top-k (when > 0), then top-p."""
        sl = logits.float() / self.temperature
        if self.top_k > 0:
            kth = sl.topk(self.top_k, dim=-1).values[..., -1:]
            sl = sl.masked_fill(sl < kth, float("-inf"))
        if self.top_p < 1.0:
            srt, idx = sl.sort(dim=-1, descending=True)
            pr = torch.softmax(srt, -1)
            remove = pr.cumsum(-1) > self.top_p
            remove[..., 1:] = remove[..., :-1].clone()
            remove[..., 0] = False
            sl = sl.scatter(-1, idx, srt.masked_fill(remove, float("-inf")))
        return torch.softmax(sl, -1)

    def _sampled_accept(self, b: StepBuffers, a: dict, q) -> None:
        """Lossless acceptance of ``b``'s block against the verify forward's
        distribution (top-k truncated, or the full vocabulary from the
        logits) on the device (``sampling.pq_accept_sparse``)."""
        B, K = b.B, b.Q
        if self.full_vocab:
            dense = self._probs_full(b.logits.view(B, K, -1))
            b.top_i[:, 0].copy_(b.logits.argmax(-1))     # the posterior (argmax) the result reports
        else:
            vals = b.top_v.view(B, K, -1)[..., :self.top_k]
            ids = b.top_i.view(B, K, -1)[..., :self.top_k]
            dense = torch.zeros(B, K, self.cfg.vocab_size, device=self.device)
            dense.scatter_(-1, ids, self._probs(vals))
        qi = q[0].to(self.device, non_blocking=True)
        qp = q[1].to(self.device, non_blocking=True)
        u = torch.rand(B, K - 1, generator=self.gen, device=self.device)
        cu = torch.rand(B, generator=self.gen, device=self.device)
        commit, corr = pq_accept_sparse(b.ids.view(B, K), dense, qi, qp, u, cu)
        a["commit"].copy_(commit)
        a["corr"].copy_(corr)
        rows = torch.arange(B, device=self.device) * K + commit - 1
        a["hid"].copy_(b.xn.index_select(0, rows))

    def _verify_fn(self, a):
        E = ops.ext()

        def fn(b: StepBuffers):
            n = self.runner.forward(b)
            post = b.top_i[:, 0]
            E.greedy_accept(b.ids.view(b.B, b.Q), post.view(b.B, b.Q), a["commit"], a["corr"],
                            b.xn, a["hid"])
            return n + 1
        return fn

    supports_gather = True

    @property
    def supports_arm(self) -> bool:
        """Greedy verification can be armed ahead of its request (on a
        tensor-parallel target every rank arms, rank 0 decides)."""
        return not self.sampled and getattr(self.tp, "local_only", False) is False

    @torch.inference_mode()
    def arm_verify(self, seqs, K: int, exp_sids, sources, rows_of, sink, head_words: int) -> dict:
        """Enqueue the next greedy verify of ``seqs`` (in the order of the
        last verify of this shape) before its request has arrived: the
        ``verify_arm`` kernel waits for the request messages, writes the
        graph's inputs from them (or placeholders and a cleared gate when a
        message does not match), then the captured verify graph and
        ``sink(ids, posterior, hidden, gate)`` run.  ``exp_sids``: the
        sequence ids the messages must carry, per row; ``sources`` int64
        [4, n_src] (inbox flag, message slot, pinned head copy, sequence
        number) and ``rows_of`` [2, n_src] (first row, rows) as the kernel
        takes them; ``head_words`` of each message are copied to its pinned
        head buffer.  Returns the arm's buffers: ``status`` (pinned; [n_src]
        is 0 when the armed verify is valid) is final once ``ev`` has
        completed."""
        B = len(seqs)
        if not self.supports_arm:
            raise RuntimeError("only greedy verification can be armed")
        b = self.runner.buffers(B, K, 1)
        a = self._abufs(B, K)
        arm = self._arm_bufs.get(B)
        if arm is None:
            arm = dict(tab=torch.zeros(2 * B, dtype=torch.int64, device=self.device),
                       tab_h=torch.zeros(2 * B, dtype=torch.int64, pin_memory=True),
                       gate=torch.zeros(1, dtype=torch.int32, device=self.device),
                       status=torch.zeros(9, dtype=torch.int32, pin_memory=True),
                       ev=torch.cuda.Event())
            self._arm_bufs[B] = arm
        th = arm["tab_h"]
        th[:B] = torch.tensor([int(x) for x in exp_sids], dtype=torch.int64)
        th[B:] = torch.tensor([len(self.kv.tables.get(s.index, ())) * self.kv.page_size for s in seqs],
                              dtype=torch.int64)
        arm["status"].fill_(-1)
        E = ops.ext()
        with torch.cuda.stream(self.stream):
            arm["tab"].copy_(th, non_blocking=True)
            self._arm_epoch += 1
            role, dec = 0, None
            if self.tp is not None and self.tp.size > 1:
                role, dec = (1 if self.tp.rank == 0 else 2), self.tp.decision_records()
            E.verify_arm(sources, rows_of, K, head_words, self.kv.page_size, arm["tab"], self.kv.block_table,
                         b.seq_rows, self.scratch, b.ids, b.pos, b.slots, b.rows.view(-1), b.kv_end, arm["gate"],
                         arm["status"], role, dec, self._arm_epoch)
            arm["ev"].record(self.stream)
            ev0 = ev1 = None
            if self.time_verify:     # the verify proper: from its request's arrival to its reply
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                ev0.record(self.stream)
        launches.add(2)
        tok = self.prof.dev_begin(f"verify_B{B}_K{K}", self.stream)
        self.graphs.run(("verify", B, K), b, self._verify_fn(a))
        self.prof.dev_end(tok)
        with torch.cuda.stream(self.stream):
            sink(b.ids.view(B, K), b.top_i[:, 0].view(B, K), b.xn, arm["gate"])
            if ev1 is not None:
                ev1.record(self.stream)
                self.verify_events.append((ev0, ev1))
        launches.add(1)
        return arm

    @torch.inference_mode()
    def submit_verify(self, seqs, blocks, q=None, sink=None, gather=None):
        """Enqueue one verify of ``blocks`` [B, K].  With ``sink`` given, it is
        called on the target stream right after the verify graph as
        ``sink(ids [B, K], posterior [B, K], hidden [B*K, H])`` (device views
        of the graph's buffers) and nothing is copied back to this host.
        ``gather``: ``[(src [R, k] device ids, dst positions in the flattened
        [B*K] block, src rows)]`` -- block entries taken on the device from a
        drafter forward still in flight (column 0 of ``src``), so the verify
        can be enqueued before the host has the draft."""
        if (q is not None) != self.sampled and K_of(blocks) > 1:
            raise ValueError("draft proposals (q) are required exactly when verification samples")
        B, K = blocks.shape
        sampled = self.sampled
        if sampled and q is None:     # single-token verify (AR): only the next token is sampled
            q = (torch.zeros(B, 0, 1, dtype=torch.long), torch.ones(B, 0, 1))
        b = self.runner.buffers(B, K, self.lm_k if sampled else 1)
        a = self._abufs(B, K)
        pref = np.fromiter((s.prefix for s in seqs), dtype=np.int64, count=B)
        pos = pref[:, None] + np.arange(K, dtype=np.int64)
        rows = np.zeros((B, K, 3), dtype=np.int32)
        rows[..., 0] = pos + 1                      # causal: row i sees slots [0, prefix + i]
        kv_end = pref + K
        self._fill(b, seqs, blocks.numpy(), pos, rows, kv_end, f"v{B}_{K}")
        if gather:
            with torch.cuda.stream(self.stream):
                flat = b.ids.view(-1)
                for src, dst, rws in gather:
                    d = torch.as_tensor(dst, dtype=torch.int64).to(self.device, non_blocking=True)
                    r = torch.as_tensor(rws, dtype=torch.int64).to(self.device, non_blocking=True)
                    flat.index_copy_(0, d, src[:, 0].index_select(0, r))
            launches.add(2 * len(gather))
        ev0 = ev1 = None
        if self.time_verify:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(self.stream)
        tok = self.prof.dev_begin(f"verify_B{B}_K{K}", self.stream)
        if sampled:
            self.graphs.run(("verify_s", B, K, self.lm_k), b, lambda bb: self.runner.forward(bb))
            with torch.cuda.stream(self.stream):
                self._sampled_accept(b, a, q)
        else:
            self.graphs.run(("verify", B, K), b, self._verify_fn(a))
        self.prof.dev_end(tok)
        if sink is not None:
            with torch.cuda.stream(self.stream):
                sink(b.ids.view(B, K), b.top_i[:, 0].view(B, K), b.xn)
            launches.add(1)
        if ev1 is not None:
            ev1.record(self.stream)
            self.verify_events.append((ev0, ev1))
        if sink is not None:
            return
        with torch.cuda.stream(self.stream):
            a["h_commit"].copy_(a["commit"], non_blocking=True)
            a["h_corr"].copy_(a["corr"], non_blocking=True)
            a["h_post"].copy_(b.top_i[:, 0], non_blocking=True)
            # the conditioning rows leave the graph's static buffer before the next replay
            hid = a["hid"].clone()
            a["ev"].record(self.stream)
        self._pending = (B, K, a, hid)

    @torch.inference_mode()
    def receive(self) -> VerifyResult:
        B, K, a, hid = self._pending
        self._pending = None
        a["ev"].synchronize()
        return VerifyResult(a["h_commit"].clone(), a["h_corr"].clone(),
                            a["h_post"].clone().view(B, K), hid)

    def release(self, seq):
        self._release(seq)


class FastDraft(_FastModelBackend, DraftBackend):
    """Drafter forwards (prefill, recovery, packed outcomes) on the kernels."""

    def __init__(self, weights: FastWeights, *, pages: int = 8192, page_size: int = 16,
                 max_seqs: int = 16, max_context: int = 4096, packed_q: int = 1024,
                 use_graphs: bool = True, device="cuda", stream=None):
        super().__init__(weights, pages=pages, page_size=page_size, max_seqs=max_seqs,
                         max_context=max_context, extra_slots=packed_q, batch_invariant=False,
                         use_graphs=use_graphs, device=device, stream=stream)
        self.vocab_size = self.cfg.vocab_size
        self.mask_id = int(self.cfg.mask_token_id)
        self._host: Dict[tuple, dict] = {}

    supports_async = True

    @torch.inference_mode()
    def prefill(self, seqs, mode, block_size):
        for s in seqs:
            n = len(s.prompt)
            rows = prefix_rows(0, n, mode, block_size).numpy()
            self._prefill_one(s, rows, topk=0, reserve=self.max_context + self.extra_slots)
        self.stream.synchronize()

    def _hbufs(self, B, Q, k):
        key = (B, Q, k)
        h = self._host.get(key)
        if h is None:
            h = dict(top=torch.zeros(B * Q, max(k, 1), dtype=torch.int64, pin_memory=True),
                     ev=torch.cuda.Event())
            self._host[key] = h
        return h

    @torch.inference_mode()
    def forward(self, seqs, ids, positions, rows, *, store, topk, cond_rows=None, sample=None,
                wait: bool = True):
        """One drafter forward.  With ``wait=False`` it returns a handle right
        after enqueueing; ``handle.result()`` waits and gives the usual dict.
        Either way the dict also carries ``"dev_top"``: the device top-k ids
        [B*Q, k], valid until the next forward of the same shape is enqueued
        (stream order makes device reads enqueued before that safe)."""
        B, Q = ids.shape
        k = max(1, topk)
        if sample is not None:
            # proposals from the drafter's top-k (fused LM-head epilogue, k <= 4)
            sk = int(sample.get("top_k") or 0)
            if not 1 <= sk <= 4:
                raise ValueError("sampled drafting on the kernels needs proposal top_k in 1..4")
            k = max(k, sk)
        b = self.runner.buffers(B, Q, k)
        kv_end = torch.maximum(rows[:, :, 0].amax(1), rows[:, :, 2].amax(1)).numpy()
        use_cond = cond_rows is not None and self.w.cond_proj is not None and seqs[0].cond is not None
        self._fill(b, seqs, ids.numpy(), positions.numpy(), rows.numpy(), kv_end, f"d{B}_{Q}",
                   cond_rows.numpy().astype(np.uint8) if use_cond else None)
        if use_cond:
            with torch.cuda.stream(self.stream):
                for i, s in enumerate(seqs):
                    b.cond[i].copy_(s.cond.to(self.device, torch.bfloat16), non_blocking=True)
        tok = self.prof.dev_begin(f"draft_B{B}_Q{Q}", self.stream)
        self.graphs.run(("draft", B, Q, k, use_cond), b, lambda bb: self.runner.forward(bb, use_cond))
        self.prof.dev_end(tok)
        h = self._hbufs(B, Q, k)
        with torch.cuda.stream(self.stream):
            h["top"].copy_(b.top_i, non_blocking=True)
            if sample is not None:
                sp, tok = self._propose(b.top_v[:, :sk], b.top_i[:, :sk], sample)
                h["sp"] = sp.to("cpu")       # small; the sampled path is not pipelined
                h["tok"] = tok.to("cpu")
                h["sk"] = sk
            else:
                h["sk"] = 0
            h["ev"].record(self.stream)
        handle = _PendingDraft(h, B, Q, k, topk, b.top_i)
        return handle.result() if wait else handle

    def _propose(self, vals, ids, sample):
        """Sample one proposal per row from softmax(top-k logits / T) after
        top-p; returns the proposal probabilities on the top-k support and
        the sampled tokens (``sampling.sparse_proposal`` on the top-k)."""
        if not hasattr(self, "gen"):
            self.gen = torch.Generator(device=self.device)
            self.gen.manual_seed(int(sample.get("seed", 0)))
        sl = vals.float() / float(sample["temperature"])
        tp = float(sample.get("top_p", 1.0))
        if tp < 1.0:
            pr = torch.softmax(sl, -1)
            remove = pr.cumsum(-1) > tp
            remove[..., 1:] = remove[..., :-1].clone()
            remove[..., 0] = False
            sl = sl.masked_fill(remove, float("-inf"))
        sp = torch.softmax(sl, -1)
        local = torch.multinomial(sp, 1, generator=self.gen)
        return sp, ids.gather(1, local)[:, 0]

    def release(self, seq):
        self._release(seq)


class _PendingDraft:
    """A drafter forward in flight (``FastDraft.forward(..., wait=False)``)."""

    def __init__(self, h, B, Q, k, topk, dev_top):
        self.h, self.B, self.Q, self.k, self.topk, self.dev_top = h, B, Q, k, topk, dev_top
        self._out = None

    def result(self) -> dict:
        if self._out is None:
            self.h["ev"].synchronize()
            top = self.h["top"].view(self.B, self.Q, self.k).clone()
            out = {"greedy": top[:, :, 0], "dev_top": self.dev_top}
            if self.topk:
                out["top"] = top[:, :, :self.topk]
            sk = self.h.get("sk", 0)
            if sk:
                out["tokens"] = self.h["tok"].view(self.B, self.Q).clone()
                out["q_ids"] = top[:, :, :sk]
                out["q_probs"] = self.h["sp"].view(self.B, self.Q, sk).clone()
            self._out = out
        return self._out
