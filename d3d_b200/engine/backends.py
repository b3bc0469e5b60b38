"""Backend interfaces of the decoding engines and their PyTorch implementation.

A *target backend* owns the target model and its KV; a *draft backend* owns
the drafter and its KV.  The coordinator (:mod:`d3d_b200.engine.spec`) holds
the reference's decode logic once and drives either:

* :class:`TorchTarget` / :class:`TorchDraft` — dense per-sequence KV, SDPA
  with the dense masks of :func:`~d3d_b200.engine.layout.rows_to_dense`; runs
  on CPU and is the oracle of the fast path;
* :class:`d3d_b200.engine.fast.FastTarget` / ``FastDraft`` — paged KV and the
  sm_100a kernels, CUDA-graph captured;
* :class:`d3d_b200.serving.remote.RemoteTarget` — a target served by another
  process (``torch.distributed`` point-to-point).

Every backend indexes KV by *slot*: query row ``j`` of a forward for sequence
``s`` is written to slot ``s.prefix + j``.  "Cropping" is only a change of the
valid length the coordinator tracks.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

import torch

from ..models.qwen3 import DenseKVCache, Qwen3LM
from .layout import prefix_rows, rows_to_dense
from .sampling import (greedy_accept, is_greedy, pq_accept_sparse, sample_tokens,
                       sampling_probs, sparse_proposal)


@dataclass
class SeqState:
    """Per-request decode state shared by the engines."""
    index: int
    prompt: List[int]
    prefix: int = 0                       # committed tokens present in both KV caches
    anchor: int = -1                      # target token at slot ``prefix`` (not yet in KV)
    generated: List[int] = field(default_factory=list)
    current: Optional[torch.Tensor] = None        # [K] block to verify (anchor first)
    top: Optional[torch.Tensor] = None            # [K, A+1] draft top tokens of ``current``
    q_ids: Optional[torch.Tensor] = None          # [K, S] sparse proposal support (sampling)
    q_probs: Optional[torch.Tensor] = None
    cond: Optional[torch.Tensor] = None           # target hidden that produced ``anchor``
    accepts: List[int] = field(default_factory=list)
    sources: List[str] = field(default_factory=list)
    source: str = "redraft"
    hits: int = 0
    recoveries: int = 0
    controlled: Any = None
    born: float = 0.0
    slot: int = -1                        # batch slot in fixed-size engines
    budget: int = 0                       # output tokens for this request (0 = the decoder default)
    extra: Dict[str, Any] = field(default_factory=dict)


@dataclass
class VerifyResult:
    commit: torch.Tensor       # [B] committed tokens (anchor + accepted drafts)
    correction: torch.Tensor   # [B] next anchor
    posterior: torch.Tensor    # [B, K] target greedy tokens after each block token
    hidden: Optional[torch.Tensor] = None   # [B, H] hidden that produced ``correction``
    gpu_s: float = 0.0


class TargetBackend:
    hidden_size: int = 0

    def prefill(self, seqs: List[SeqState]) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        raise NotImplementedError

    def submit_verify(self, seqs: List[SeqState], blocks: torch.Tensor, q=None) -> None:
        raise NotImplementedError

    def receive(self) -> VerifyResult:
        raise NotImplementedError

    def verify(self, seqs, blocks, q=None) -> VerifyResult:
        self.submit_verify(seqs, blocks, q)
        return self.receive()

    def release(self, seq: SeqState) -> None:
        pass

    def close(self) -> None:
        pass


class DraftBackend:
    vocab_size: int = 0
    mask_id: int = 0

    def prefill(self, seqs: List[SeqState], mode: str, block_size: int) -> None:
        raise NotImplementedError

    def forward(self, seqs: List[SeqState], ids: torch.Tensor, positions: torch.Tensor,
                rows: torch.Tensor, *, store: bool, topk: int, cond_rows=None,
                sample: Optional[dict] = None) -> Dict[str, torch.Tensor]:
        """Run one drafter forward for ``B`` sequences with equal ``Q``.

        ``rows [B, Q, 3]`` are absolute-slot attention descriptors.  Returns
        ``greedy [B, Q]`` and, when ``topk`` > 0, ``top [B, Q, topk]``; with
        ``sample`` set (temperature > 0) also ``tokens``/``q_ids``/``q_probs``."""
        raise NotImplementedError

    def trim(self, seq: SeqState, length: int) -> None:
        pass

    def release(self, seq: SeqState) -> None:
        pass


# --------------------------------------------------------------------------
# PyTorch implementations (oracle)
# --------------------------------------------------------------------------
class _DenseKVPool:
    def __init__(self, n_layers: int):
        self.n_layers = n_layers
        self.caches: Dict[int, DenseKVCache] = {}

    def get(self, seq: SeqState) -> DenseKVCache:
        c = self.caches.get(seq.index)
        if c is None:
            c = self.caches[seq.index] = DenseKVCache(self.n_layers)
        return c

    def release(self, seq: SeqState) -> None:
        self.caches.pop(seq.index, None)


class TorchTarget(TargetBackend):
    """Target verification in PyTorch (``single/eval_async_packed.py:86-199``)."""

    def __init__(self, model: Qwen3LM, temperature: float = 0.0, top_k: int = 0,
                 top_p: float = 1.0, seed: int = 0):
        self.model = model.eval()
        self.device = next(model.parameters()).device
        self.kv = _DenseKVPool(model.cfg.num_hidden_layers)
        self.hidden_size = model.cfg.hidden_size
        self.temperature, self.top_k, self.top_p = temperature, top_k, top_p
        self.gen = torch.Generator(device="cpu").manual_seed(seed)
        self._pending = None

    @torch.inference_mode()
    def prefill(self, seqs):
        anchors, hiddens = [], []
        for s in seqs:
            ids = torch.tensor([s.prompt], dtype=torch.long, device=self.device)
            cache = self.kv.get(s)
            cache.crop(0)
            h = self.model(ids, cache=cache, store_kv=True)
            logits = self.model.logits(h[:, -1])
            if is_greedy(self.temperature):
                a = logits.argmax(-1)
            else:
                pr = sampling_probs(logits, self.temperature, self.top_k, self.top_p)
                u = torch.rand(1, generator=self.gen).item()
                a = torch.searchsorted(pr.cumsum(-1) / pr.sum(-1, keepdim=True),
                                       torch.tensor([[u]], device=pr.device))[:, 0]
            anchors.append(int(a[0]))
            hiddens.append(h[0, -1].float())
        return torch.tensor(anchors, dtype=torch.long), torch.stack(hiddens)

    @torch.inference_mode()
    def submit_verify(self, seqs, blocks, q=None):
        self._pending = (seqs, blocks, q)

    @torch.inference_mode()
    def receive(self) -> VerifyResult:
        seqs, blocks, q = self._pending
        self._pending = None
        blocks = blocks.to(self.device)
        commits, corrs, posts, hids = [], [], [], []
        for b, s in enumerate(seqs):
            cache = self.kv.get(s)
            cache.crop(s.prefix)
            blk = blocks[b:b + 1]
            k = blk.shape[1]
            h = self.model(blk, cache=cache, store_kv=True)
            logits = self.model.logits(h)[0]            # [K, V]
            post = logits.argmax(-1)
            if is_greedy(self.temperature) or k == 1:
                commit, corr = greedy_accept(blk, post[None])
                if not is_greedy(self.temperature):
                    pr = sampling_probs(logits[-1:], self.temperature, self.top_k, self.top_p)
                    u = torch.rand(1, generator=self.gen)
                    corr = torch.searchsorted(pr.cumsum(-1), u[None].to(pr.device))[:, 0]
            else:
                qi, qp = q[0][b:b + 1].to(self.device), q[1][b:b + 1].to(self.device)
                probs = sampling_probs(logits, self.temperature, self.top_k, self.top_p)[None]
                u = torch.rand(1, k - 1, generator=self.gen).to(self.device)
                cu = torch.rand(1, generator=self.gen).to(self.device)
                commit, corr = pq_accept_sparse(blk, probs, qi, qp, u, cu)
            c = int(commit[0])
            cache.crop(s.prefix + c)
            commits.append(c)
            corrs.append(int(corr[0]))
            posts.append(post)
            hids.append(h[0, c - 1].float())
        return VerifyResult(torch.tensor(commits), torch.tensor(corrs),
                            torch.stack(posts).cpu(), torch.stack(hids))

    def release(self, seq):
        self.kv.release(seq)

    def leak_check(self) -> None:
        """Raise if a sequence still holds a KV cache after a finished run."""
        if self.kv.caches:
            raise RuntimeError(f"KV caches leaked: {len(self.kv.caches)} sequences still allocated")


class TorchDraft(DraftBackend):
    """Drafter forwards in PyTorch with dense masks (``models/d3d/modeling_d3d.py``)."""

    def __init__(self, model: Qwen3LM, seed: int = 0):
        self.model = model.eval()
        self.device = next(model.parameters()).device
        self.kv = _DenseKVPool(model.cfg.num_hidden_layers)
        self.vocab_size = model.cfg.vocab_size
        self.mask_id = int(model.cfg.mask_token_id)
        self.record_logits = False    # also return every row's logits
        self.last: Dict[str, torch.Tensor] = {}
        self.gen = torch.Generator(device="cpu").manual_seed(seed)

    @torch.inference_mode()
    def prefill(self, seqs, mode, block_size):
        for s in seqs:
            ids = torch.tensor([s.prompt], dtype=torch.long, device=self.device)
            n = ids.shape[1]
            rows = prefix_rows(0, n, mode, block_size, self.device)
            cache = self.kv.get(s)
            cache.crop(0)
            self.model(ids, mask=rows_to_dense(rows, n)[None], cache=cache, store_kv=True)

    @torch.inference_mode()
    def forward(self, seqs, ids, positions, rows, *, store, topk, cond_rows=None, sample=None):
        out: Dict[str, List[torch.Tensor]] = {"greedy": [], "top": [], "tokens": [],
                                              "q_ids": [], "q_probs": [], "logits": []}
        for b, s in enumerate(seqs):
            cache = self.kv.get(s)
            cache.crop(s.prefix)
            q = ids.shape[1]
            mask = rows_to_dense(rows[b].to(self.device), s.prefix + q)[None]
            cond = None if s.cond is None else s.cond[None].to(self.device)
            cr = None if cond_rows is None else cond_rows[b:b + 1].to(self.device)
            h = self.model(ids[b:b + 1].to(self.device), positions[b:b + 1].to(self.device),
                           mask=mask, cache=cache, store_kv=store, cond=cond, cond_rows=cr)
            logits = self.model.logits(h)[0].float()
            out["greedy"].append(logits.argmax(-1))
            if self.record_logits:     # every row's logits (near-tie analysis of a validation)
                out["logits"].append(logits)
            if topk:
                out["top"].append(torch.topk(logits, k=topk, dim=-1).indices)
            if sample is not None:
                tok, qi, qp = sparse_proposal(logits, sample["temperature"], sample["top_k"],
                                              sample["top_p"], generator=self.gen)
                out["tokens"].append(tok)
                out["q_ids"].append(qi)
                out["q_probs"].append(qp)
        self.last = {k: torch.stack(v) for k, v in out.items() if v}
        return self.last

    def trim(self, seq, length):
        self.kv.get(seq).crop(length)

    def release(self, seq):
        self.kv.release(seq)
