"""Asynchronous speculative decoding coordinator (single request and batched).

This restates the reference's two decode loops in one batched loop:

* single request, ``single/eval_async_packed.py:796-1297``
  (``run_d3d_generate_async``): submit the current block to the target, run
  the packed all-outcome draft while the target verifies, commit
  ``accepted + 1`` tokens, reuse the branch keyed
  ``(commit_len, correction)`` or redraft from the anchor on a miss;
* concurrent serving, ``serving/engine.py:148-227``: the same step over every
  running request, strict admission up to ``concurrency``, prefill in groups,
  draft micro-batches, and leak checks at the end.

Decode accounting follows the reference: ``accept_length`` is the number of
tokens committed per verify, anchor included
(``single/eval_async_packed.py:1097,1150``); single-request throughput is
decode-only (prefill and the first token excluded); concurrent throughput is
end to end.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch

from ..utils.timing import StepProfiler
from .backends import DraftBackend, SeqState, TargetBackend
from .layout import branch_specs, full_rows, packed_layout
from .sampling import is_greedy

EOS_DEFAULT = (151643, 151645)


@dataclass
class DecodeConfig:
    block_size: int = 16
    anchor_num: int = 1
    attention_mask_mode: str = "causal"
    max_new_tokens: int = 512
    temperature: float = 0.0
    top_k: int = 0            # proposal top-k (sampling; 0 = full vocabulary, kernel drafter 1..4)
    top_p: float = 1.0
    target_top_k: int = 0     # target sampling truncation (0 = full vocabulary)
    target_top_p: float = 1.0
    draft_microbatch: int = 4
    prefill_group: int = 4
    ignore_eos: bool = False
    eos: Tuple[int, ...] = EOS_DEFAULT
    packed_accepted_counts: Optional[Tuple[int, ...]] = None
    use_cond: bool = True     # feed target hidden to a conditioned drafter
    backup: str = "neural"    # on a branch miss: "neural" redraft; "fast" / "fast_legacy" random block (greedy only)
    backup_seed: int = 42
    fast_miss_anchors: int = 0  # fast backup: anchors of a fast-seeded block's drafts (0 = anchor_num)

    def validate(self):
        if self.block_size <= 1:
            raise ValueError("--block-size must be > 1")
        if self.anchor_num < 0:
            raise ValueError("--anchor-num must be non-negative")
        if self.top_k < 0:
            raise ValueError("--proposal-top-k must be >= 0 (0 = the drafter's full distribution)")
        if self.backup not in ("neural", "fast", "fast_legacy"):
            raise ValueError("--backup must be neural, fast or fast_legacy")
        if self.fast_miss_anchors < 0:
            raise ValueError("--fast-miss-anchors must be non-negative")
        if self.backup != "neural" and not is_greedy(self.temperature):
            raise ValueError("the fast backup (random block on a miss) is greedy only")
        return self


@dataclass
class RequestOutput:
    index: int
    tokens: List[int]
    accepts: List[int]
    sources: List[str]
    hits: int
    recoveries: int
    latency_s: float            # admission to completion
    decode_s: float = 0.0       # after the request's prefill to completion (the single-request metric)


class _Outcomes:
    """The branches of one packed forward for one sequence, sliced on demand
    (only the branch that matches the verification outcome is materialised).
    ``out`` may be a drafter forward still in flight (a handle with
    ``result()``); it is resolved the first time a branch is read."""

    def __init__(self, lay, out, i: int, q_len: int = 0):
        self.lay, self._out, self.i, self.q_len = lay, out, i, q_len
        self.index = {key: j for j, key in enumerate(lay.keys)}

    @property
    def out(self) -> Dict[str, torch.Tensor]:
        if not isinstance(self._out, dict):
            self._out = self._out.result()
        return self._out

    def has(self, key) -> bool:
        return key in self.index

    def device_rows(self, key):
        """(device top-k ids of the forward, rows holding drafts 1..K-1 of
        branch ``key``): what the target's verify input gathers on the device."""
        sl = self.lay.segment(self.index[key])
        src = self._out.dev_top if not isinstance(self._out, dict) else self._out["dev_top"]
        base = self.i * self.q_len + sl.start
        return src, list(range(base + 1, base + (sl.stop - sl.start)))

    def get(self, key):
        j = self.index.get(key)
        if j is None:
            return None
        sl = self.lay.segment(j)
        out, i = self.out, self.i
        toks = out["tokens"] if "tokens" in out else out["greedy"]
        blk = toks[i, sl].clone()
        if key[1] is not None:
            blk[0] = key[1]
        top = out["top"][i, sl].clone() if "top" in out else None
        qq = (out["q_ids"][i, sl], out["q_probs"][i, sl]) if "q_ids" in out else None
        return blk, top, qq


class SpecDecoder:
    """Drives a target backend and a draft backend through the async loop."""

    def __init__(self, target: TargetBackend, draft: DraftBackend, cfg: DecodeConfig,
                 overlap: bool = True):
        self.t, self.d, self.cfg = target, draft, cfg.validate()
        self.overlap = overlap
        self.stats: Dict[str, float] = {}
        self.prof = StepProfiler(False)
        for be in (target, draft):
            if hasattr(be, "prof"):
                be.prof = self.prof

    # ------------------------------------------------------------ helpers
    def _controlled(self, s: SeqState, block: torch.Tensor, top, anchor_pos: int):
        if s.controlled is not None:
            s.controlled.override(block, top, anchor_pos)

    def _sample_cfg(self):
        c = self.cfg
        if is_greedy(c.temperature):
            return None
        return dict(temperature=c.temperature, top_k=c.top_k, top_p=c.top_p)

    def _cond_rows(self, b: int, q: int, starts: Sequence[int]):
        if not self.cfg.use_cond:
            return None
        cr = torch.zeros(b, q, dtype=torch.bool)
        for st in starts:
            cr[:, st] = True
        return cr

    # ----------------------------------------------------------- recovery
    def recover(self, seqs: List[SeqState]) -> None:
        """Draft ``[anchor, MASK x K-1]`` from each anchor in one forward
        (``single/eval_async_packed.py:950-984``; ``serving/engine.py:54-62``)."""
        k, a = self.cfg.block_size, self.cfg.anchor_num
        for off in range(0, len(seqs), self.cfg.draft_microbatch):
            group = seqs[off:off + self.cfg.draft_microbatch]
            b = len(group)
            ids = torch.full((b, k), self.d.mask_id, dtype=torch.long)
            ids[:, 0] = torch.tensor([s.anchor for s in group])
            pos = torch.stack([torch.arange(s.prefix, s.prefix + k) for s in group])
            rows = torch.stack([full_rows(s.prefix + k, k) for s in group])
            out = self.d.forward(group, ids, pos, rows, store=False, topk=a + 1 if a else 0,
                                 cond_rows=self._cond_rows(b, k, [0]),
                                 sample=self._sample_cfg())
            toks = out["tokens"] if "tokens" in out else out["greedy"]
            for i, s in enumerate(group):
                blk = toks[i].clone().cpu()
                blk[0] = s.anchor
                top = out["top"][i].clone().cpu() if "top" in out else None
                self._controlled(s, blk, top, s.prefix)
                s.current, s.top = blk, top
                if "q_ids" in out:
                    s.q_ids, s.q_probs = out["q_ids"][i].cpu(), out["q_probs"][i].cpu()
                s.recoveries += 1
                s.source = "redraft"

    def fast_backup(self, seqs: List[SeqState]) -> None:
        """On a miss, verify ``[anchor, random x K-1]`` at once instead of
        redrafting on the critical path: greedy verification needs token ids
        only, and commits at least the anchor.  The drafter's view of the
        anchor (its top tokens, for the next step's branches) is computed in
        the next :meth:`predict`, off the critical path
        (``serving/engine.py:64-92``, ``backup="fast"``)."""
        k = self.cfg.block_size
        if not hasattr(self, "_backup_gen"):
            self._backup_gen = torch.Generator().manual_seed(int(self.cfg.backup_seed))
        for s in seqs:
            blk = torch.randint(int(self.d.vocab_size), (k,), generator=self._backup_gen)
            blk[0] = s.anchor
            s.current, s.top = blk, None
            s.extra["needs_seed"] = True
            s.extra["fast_backups"] = s.extra.get("fast_backups", 0) + 1
            s.source = "fast_backup"

    def _seed_tops(self, seqs: List[SeqState]) -> None:
        """The drafter's top tokens after each fast-backup anchor (``[anchor,
        MASK x K-1]`` rows, KV not stored), without touching the random block
        being verified."""
        k, a = self.cfg.block_size, self.cfg.anchor_num
        for off in range(0, len(seqs), self.cfg.draft_microbatch):
            group = seqs[off:off + self.cfg.draft_microbatch]
            b = len(group)
            ids = torch.full((b, k), self.d.mask_id, dtype=torch.long)
            ids[:, 0] = torch.tensor([s.anchor for s in group])
            pos = torch.stack([torch.arange(s.prefix, s.prefix + k) for s in group])
            rows = torch.stack([full_rows(s.prefix + k, k) for s in group])
            wide = max(a, self.cfg.fast_miss_anchors) if a and self.cfg.backup == "fast" else a
            out = self.d.forward(group, ids, pos, rows, store=False, topk=wide + 1 if a else 0,
                                 cond_rows=self._cond_rows(b, k, [0]))
            for i, s in enumerate(group):
                top = out["top"][i].clone().cpu() if "top" in out else None
                if top is not None and s.controlled is not None:
                    seed = out["greedy"][i].clone().cpu()
                    seed[0] = s.anchor
                    self._controlled(s, seed, top, s.prefix)
                s.top = top
                s.extra["needs_seed"] = False

    # ------------------------------------------------------ packed outcomes
    def _pipelined(self) -> bool:
        """Whether the next verify may be enqueued behind a drafter forward still
        in flight, its draft tokens gathered on the device (kernel backends of
        one GPU, greedy)."""
        return (is_greedy(self.cfg.temperature) and getattr(self.t, "supports_gather", False)
                and getattr(self.d, "supports_async", False)
                and getattr(self.d, "stream", None) is not None
                and (getattr(self.t, "stream", None) is self.d.stream
                     or getattr(self.t, "draft_stream", None) is self.d.stream))

    def predict(self, seqs: List[SeqState], wait: bool = True) -> Dict[int, "_Outcomes"]:
        """One packed forward per micro-batch: commit the pending block into the
        draft KV and draft one continuation per (commit length, anchor).  With
        ``wait=False`` (asynchronous drafter backends) the forwards are only
        enqueued; each outcome resolves when first read."""
        k, a = self.cfg.block_size, self.cfg.anchor_num
        seeds = [s for s in seqs if s.extra.get("needs_seed")]
        if seeds:
            self._seed_tops(seeds)
        # A sequence whose block was a random fast-backup block almost surely
        # commits only its anchor: its packed forward drafts only the commit
        # length 1 outcomes, with ``fast_miss_anchors`` anchors (default: the
        # anchor count), in micro-batches of its own (``serving/engine.py:88-104``).
        # ``fast_legacy`` drafts every outcome of such a block at full depth.
        shallow_ids = {s.index for s in seeds} if self.cfg.backup == "fast" else set()
        parts = [([s for s in seqs if s.index not in shallow_ids], False),
                 ([s for s in seqs if s.index in shallow_ids], True)]
        fanout = self.cfg.fast_miss_anchors or a
        groups = [(part[off:off + self.cfg.draft_microbatch], shallow) for part, shallow in parts
                  for off in range(0, len(part), self.cfg.draft_microbatch)]
        results: Dict[int, _Outcomes] = {}
        for group, shallow in groups:
            layouts = []
            for s in group:
                top = None if s.top is None else s.top.tolist()
                if shallow:
                    specs = branch_specs(s.current.tolist(), top, fanout if a else 0, (1,))
                else:
                    specs = branch_specs(s.current.tolist(), top, a, self.cfg.packed_accepted_counts)
                layouts.append(packed_layout(s.current, specs, s.prefix, k, self.d.mask_id,
                                             self.cfg.attention_mask_mode))
            q = layouts[0].q_len
            if any(l.q_len != q for l in layouts):
                raise RuntimeError("packed layouts in one micro-batch must have equal length")
            ids = torch.stack([l.input_ids for l in layouts])
            pos = torch.stack([l.positions for l in layouts])
            rows = torch.stack([l.rows for l in layouts])
            seg_starts = [0] + [k + j * k for j in range(len(layouts[0].keys))]
            kw = {} if wait else {"wait": False}
            out = self.d.forward(group, ids, pos, rows, store=True, topk=a + 1 if a else 0,
                                 cond_rows=self._cond_rows(len(group), q, seg_starts),
                                 sample=self._sample_cfg(), **kw)
            for i, (s, lay) in enumerate(zip(group, layouts)):
                self.d.trim(s, s.prefix + k)
                results[s.index] = _Outcomes(lay, out, i, q)
        return results

    def _arm_select(self, running: List[SeqState], predictions, block_t: torch.Tensor) -> bool:
        """Hand the choice of verify(t+1)'s blocks to the drafter GPU (the
        target backend's ``arm_select``): per row the sequence id, prefix,
        the commit length at which the row finishes (output budget, or a stop
        token among the block's drafts), the packed forward's branch keys
        with the first row of each branch, the stop tokens, and -- in
        acceptance-controlled mode -- the controlled drafts of the positions
        the next block can cover.  The kernel sends only when every row
        continues on a drafted branch, exactly when the host loop would
        enqueue verify(t+1) ahead; otherwise the host takes the step."""
        cfg, k = self.cfg, self.cfg.block_size
        B = len(running)
        if B == 0 or B > 64:
            return False
        ctrl = running[0].controlled is not None
        if any((s.controlled is not None) != ctrl for s in running):
            return False
        prs = [predictions.get(s.index) for s in running]
        if any(p is None for p in prs):
            return False
        top = None
        for p in prs:
            src = p._out["dev_top"] if isinstance(p._out, dict) else getattr(p._out, "dev_top", None)
            if src is None or (top is not None and src is not top):
                return False
            top = src
        nk = max(len(p.lay.keys) for p in prs)
        eos = [] if cfg.ignore_eos else [int(t) for t in cfg.eos]
        sid, pref, lim, keys, krows, ctl = [], [], [], [], [], []
        for r, (s, p) in enumerate(zip(running, prs)):
            for j, key in enumerate(p.lay.keys):
                sl = p.lay.segment(j)
                if sl.stop - sl.start != k:
                    return False
                keys += [int(key[0]), -1 if key[1] is None else int(key[1])]
                krows.append(p.i * p.q_len + sl.start)
            pad = nk - len(p.lay.keys)
            keys += [-1, -1] * pad
            krows += [0] * pad
            room = s.budget - len(s.generated)
            first_stop = k
            if eos:
                for j, tok in enumerate(block_t[r, :k].tolist()):
                    if tok in cfg.eos:
                        first_stop = j
                        break
            lim.append(min(room, first_stop + 1))
            sid.append(int(s.index))
            pref.append(int(s.prefix))
            if ctrl:
                ctl += [int(s.controlled.draft_at(s.prefix + 1 + m)) for m in range(2 * k)]
        tab = sid + pref + lim + keys + krows + eos + ctl
        return self.t.arm_select(B, k, nk, cfg.anchor_num == 0, len(eos), ctrl, top, tab)

    # ------------------------------------------------------------ main loop
    def generate(self, prompts: Sequence[Sequence[int]], concurrency: int = 1,
                 controlled: Optional[Callable[[int], object]] = None,
                 on_step: Optional[Callable[[int], None]] = None,
                 max_new: Optional[Sequence[int]] = None) -> dict:
        """Decode every prompt (``concurrency`` at a time, closed loop).
        ``max_new``: per-request output budgets (default: the config's)."""
        cfg = self.cfg
        k = cfg.block_size
        if concurrency < 1 or cfg.max_new_tokens < 1:
            raise ValueError("positive concurrency and output length required")
        waiting = iter(enumerate(prompts))
        running: List[SeqState] = []
        outputs: List[RequestOutput] = []
        exhausted = False
        started = time.perf_counter()
        steps = 0
        verify_tokens = 0
        miss_rounds = 0
        batch_sizes: List[int] = []
        preverified: Optional[torch.Tensor] = None   # block of a verify already enqueued
        while running or not exhausted:
            admitted: List[SeqState] = []
            while len(running) + len(admitted) < concurrency and not exhausted:
                try:
                    idx, ids = next(waiting)
                except StopIteration:
                    exhausted = True
                    break
                s = SeqState(index=idx, prompt=[int(t) for t in ids], prefix=len(ids),
                             born=time.perf_counter(),
                             budget=int(max_new[idx]) if max_new is not None else cfg.max_new_tokens)
                s.controlled = controlled(idx) if controlled is not None else None
                admitted.append(s)
            for off in range(0, len(admitted), cfg.prefill_group):
                group = admitted[off:off + cfg.prefill_group]
                anchors, hidden = self.t.prefill(group)
                self.d.prefill(group, cfg.attention_mask_mode, k)
                t_decode = time.perf_counter()
                ready = []
                for i, s in enumerate(group):
                    s.extra["t_decode"] = t_decode
                    s.anchor = int(anchors[i])
                    s.cond = None if hidden is None or not cfg.use_cond else hidden[i]
                    if not cfg.ignore_eos and s.anchor in cfg.eos:
                        s.generated = [s.anchor]
                        self._finish(s, outputs)
                    else:
                        ready.append(s)
                self.recover(ready)
                running.extend(ready)
            if not running:
                continue
            batch_sizes.append(len(running))
            # The reference truncates the last block at the output budget
            # (``eval_async_packed.py:1022-1030``); here the full block is
            # verified (one captured shape) and the commit is clipped instead,
            # which emits the same tokens.
            width = k
            qq = None
            if preverified is not None:
                # verify(t) was enqueued during the previous step, behind draft(t-1)
                block_t, preverified = preverified, None
            else:
                block_t = torch.stack([s.current[:k] for s in running])
                if not is_greedy(cfg.temperature):
                    qq = (torch.stack([s.q_ids[1:width] for s in running]),
                          torch.stack([s.q_probs[1:width] for s in running]))
                with self.prof.phase("submit_verify"):
                    self.t.submit_verify(running, block_t, qq)
            pipe = self._pipelined()
            with self.prof.phase("predict"):
                predictions = self.predict(running, wait=not pipe) if width == k else {}
            armed = (pipe and width == k and (exhausted or len(running) >= concurrency)
                     and getattr(self.t, "supports_select", False)
                     and self._arm_select(running, predictions, block_t))
            with self.prof.phase("receive"):
                res = self.t.receive()
            dev_sent = bool(armed) and self.t.select_sent()
            steps += 1
            verify_tokens += width * len(running)
            remaining, recover = [], []
            t_sel = time.perf_counter()
            cont = []   # (sequence, commit length, correction, branch key)
            for i, s in enumerate(running):
                n = int(res.commit[i])
                corr = int(res.correction[i])
                emitted = block_t[i, :n].tolist()
                room = s.budget - len(s.generated)
                emitted = emitted[:room]
                stop = False
                if not cfg.ignore_eos:
                    for j, tok in enumerate(emitted):
                        if tok in cfg.eos:
                            emitted = emitted[:j + 1]
                            stop = True
                            break
                s.generated.extend(emitted)
                s.accepts.append(n)
                s.sources.append(s.source)
                s.prefix += n
                s.anchor = corr
                if res.hidden is not None and cfg.use_cond:
                    s.cond = res.hidden[i]
                if stop or len(s.generated) >= s.budget:
                    self._finish(s, outputs)
                    continue
                if not cfg.ignore_eos and corr in cfg.eos:
                    s.generated.append(corr)
                    self._finish(s, outputs)
                    continue
                cont.append((s, n, corr, (n, None if (n == k or cfg.anchor_num == 0) else corr)))
            # Every continuing sequence hit a drafted branch and nothing will be
            # admitted: enqueue verify(t+1) now, behind draft(t) on the same
            # stream, so the GPU goes straight on while the host selects.
            nxt = None
            if dev_sent:
                # the drafter GPU already picked every row's branch and sent
                # verify(t+1); the host mirrors that choice for its records
                if len(cont) != len(running) or not all(
                        predictions.get(c[0].index) is not None and predictions[c[0].index].has(c[3])
                        for c in cont):
                    raise RuntimeError("device branch select disagrees with the host's selection")
                nxt = torch.zeros(len(cont), k, dtype=torch.long)
                for r, (s, n, corr, key) in enumerate(cont):
                    nxt[r, 0] = corr
                    if s.controlled is not None:
                        self._controlled(s, nxt[r], None, s.prefix)
                self.t.adopt_sent(len(cont), k)
            elif pipe and cont and (exhausted or len(cont) >= concurrency) and all(
                    predictions.get(c[0].index) is not None and predictions[c[0].index].has(c[3])
                    for c in cont):
                nxt = torch.zeros(len(cont), k, dtype=torch.long)
                gather = []
                for r, (s, n, corr, key) in enumerate(cont):
                    nxt[r, 0] = corr
                    if s.controlled is not None:
                        self._controlled(s, nxt[r], None, s.prefix)
                    else:
                        src, rows = predictions[s.index].device_rows(key)
                        gather.append((src, [r * k + j for j in range(1, k)], rows))
                self.t.submit_verify([c[0] for c in cont], nxt, gather=gather)
            for r, (s, n, corr, key) in enumerate(cont):
                pr = predictions.get(s.index)
                sel = pr.get(key) if pr is not None else None
                self.d.trim(s, s.prefix)
                if sel is None:
                    recover.append(s)
                else:
                    blk, top, q2 = sel
                    blk = blk.clone()
                    blk[0] = corr
                    top = None if top is None else top.clone()
                    self._controlled(s, blk, top, s.prefix)
                    s.current, s.top = blk, top
                    if q2 is not None:
                        s.q_ids, s.q_probs = q2
                    s.hits += 1
                    s.source = "packed_full" if n == k else f"packed_outcome_{n}"
                    if nxt is not None and s.controlled is None:
                        nxt[r] = blk      # the host copy of what the device gathered
                    elif nxt is not None and not torch.equal(nxt[r], blk):
                        raise RuntimeError("pipelined verify input differs from the selected branch")
                remaining.append(s)
            if nxt is not None:
                preverified = nxt
            if self.prof.enabled:
                self.prof.host["select"] += time.perf_counter() - t_sel
            running = remaining
            miss_rounds += bool(recover)
            with self.prof.phase("recover"):
                if cfg.backup != "neural":
                    self.fast_backup(recover)
                else:
                    self.recover(recover)
            if on_step is not None:
                on_step(steps)
        elapsed = time.perf_counter() - started
        for be in (self.t, self.d):      # every request released its pages (reference: serving/engine.py:216-218)
            check = getattr(be, "leak_check", None)
            if check is not None:
                check()
        outputs.sort(key=lambda o: o.index)
        total = sum(len(o.tokens) for o in outputs)
        accepts = [a for o in outputs for a in o.accepts]
        return dict(outputs=outputs, elapsed_s=elapsed, output_tokens=total,
                    tps=total / elapsed if elapsed > 0 else 0.0, steps=steps,
                    verify_tokens=verify_tokens, miss_rounds=miss_rounds,
                    mean_accept_length=(sum(accepts) / len(accepts)) if accepts else 0.0,
                    decode_batch_sizes=batch_sizes)

    def _finish(self, s: SeqState, outputs: List[RequestOutput]) -> None:
        now = time.perf_counter()
        outputs.append(RequestOutput(s.index, list(s.generated), list(s.accepts),
                                     list(s.sources), s.hits, s.recoveries, now - s.born,
                                     now - s.extra.get("t_decode", now)))
        self.t.release(s)
        self.d.release(s)


def ar_generate(target: TargetBackend, prompts: Sequence[Sequence[int]], max_new_tokens: int,
                eos: Tuple[int, ...] = EOS_DEFAULT, ignore_eos: bool = False,
                concurrency: int = 1, max_new: Optional[Sequence[int]] = None, prefill_group: int = 4) -> dict:
    """Target-only autoregressive decoding through the same verify path
    (``single/eval_async_packed.py:1489-1535``; ``serving/baseline_ar.py``,
    ``serving/baseline_concurrency.py``): up to ``concurrency`` requests in
    flight, a finished request's place refilled at once (closed loop, like
    :meth:`SpecDecoder.generate`), admitted requests prefilled in groups of
    ``prefill_group`` as the speculative engine does.  ``max_new``:
    per-request budgets.  Besides the outputs: per-request latency (admission
    to completion) and finish reason, the largest number in flight and every
    decode step's batch size."""
    started = time.perf_counter()
    waiting = iter(enumerate(prompts))
    exhausted = False
    results: Dict[int, List[int]] = {}
    latency: Dict[int, float] = {}
    reason: Dict[int, str] = {}
    live: List[SeqState] = []
    max_active, batches = 0, []

    decode: Dict[int, float] = {}

    def finish(s: SeqState, toks: List[int], why: str) -> None:
        results[s.index] = toks
        now = time.perf_counter()
        latency[s.index] = now - s.born
        decode[s.index] = now - s.extra.get("t_decode", now)
        reason[s.index] = why
        target.release(s)

    def budget(i: int) -> int:
        return int(max_new[i]) if max_new is not None else int(max_new_tokens)

    while live or not exhausted:
        new: List[SeqState] = []
        while len(live) + len(new) < concurrency and not exhausted:
            try:
                i, p = next(waiting)
            except StopIteration:
                exhausted = True
                break
            new.append(SeqState(index=i, prompt=[int(t) for t in p], prefix=len(p), budget=budget(i),
                                born=time.perf_counter()))
        max_active = max(max_active, len(live) + len(new))
        for off in range(0, len(new), max(1, prefill_group)):
            group = new[off:off + max(1, prefill_group)]
            anchors, _ = target.prefill(group)
            t_decode = time.perf_counter()
            for s, a in zip(group, anchors.tolist()):
                s.extra["t_decode"] = t_decode
                s.anchor = int(a)
                s.generated = [s.anchor]
                if not ignore_eos and s.anchor in eos:
                    finish(s, s.generated[:s.budget], "eos")
                elif s.budget <= 1:
                    finish(s, s.generated[:s.budget], "length")
                else:
                    live.append(s)
        if not live:
            continue
        batches.append(len(live))
        blocks = torch.tensor([[s.anchor] for s in live], dtype=torch.long)
        res = target.verify(live, blocks)
        nxt = []
        for i, s in enumerate(live):
            s.prefix += 1
            s.anchor = int(res.correction[i])
            s.generated.append(s.anchor)
            if not ignore_eos and s.anchor in eos:
                finish(s, s.generated, "eos")
            elif len(s.generated) >= s.budget:
                finish(s, s.generated, "length")
            else:
                nxt.append(s)
        live = nxt
    elapsed = time.perf_counter() - started
    outs = [results[i] for i in range(len(prompts))]
    total = sum(len(o) for o in outs)
    lat = sorted(latency.values())
    n = len(outs)
    return dict(outputs=outs, elapsed_s=elapsed, output_tokens=total,
                tps=total / elapsed if elapsed > 0 else 0.0, requests=n, max_active=max_active,
                decode_batch_sizes=batches, latency_s=[latency[i] for i in range(n)],
                decode_s=[decode[i] for i in range(n)],
                finish_reasons=[reason[i] for i in range(n)],
                latency_p50_s=lat[len(lat) // 2] if lat else 0.0,
                latency_p95_s=lat[min(len(lat) - 1, int(0.95 * len(lat)))] if lat else 0.0,
                length_limit_fraction=sum(r == "length" for r in reason.values()) / max(1, n),
                mean_output_tokens=total / max(1, n))


def ar_decode_fixed(target: TargetBackend, prompts: Sequence[Sequence[int]], steps: int,
                    capture: bool = False) -> dict:
    """Fixed-batch decode-only AR throughput (``serving/baseline_ar.py:23-47``):
    every prompt is prefilled, then the whole batch decodes ``steps`` tokens
    with no stop condition.  The prefill and its first token are excluded
    from the time and the token count."""
    seqs = [SeqState(index=i, prompt=[int(t) for t in p], prefix=len(p)) for i, p in enumerate(prompts)]
    anchors, _ = target.prefill(seqs)
    cur = [int(a) for a in anchors.tolist()]
    toks = [[a] for a in cur] if capture else None
    started = time.perf_counter()
    for _ in range(int(steps)):
        res = target.verify(seqs, torch.tensor([[a] for a in cur], dtype=torch.long))
        cur = [int(c) for c in res.correction.tolist()]
        for i, s in enumerate(seqs):
            s.prefix += 1
            if capture:
                toks[i].append(cur[i])
    elapsed = time.perf_counter() - started
    for s in seqs:
        target.release(s)
    n = len(prompts) * int(steps)
    return dict(elapsed_s=elapsed, tokens=n, requests=len(prompts), tps=n / elapsed if elapsed > 0 else 0.0,
                outputs=toks)
