"""Sampling and lossless acceptance (CPU/PyTorch semantics; the CUDA kernels
in :mod:`d3d_b200.ops` are checked against these functions).

* ``sampling_probs`` / ``sample_tokens``: greedy, temperature, top-k, top-p
  (``single/eval_sync.py:287-338``).
* ``sparse_proposal``: the drafter's sparse top-k proposal that travels to the
  target (``single/eval_sync.py:341-367``).
* ``greedy_accept``: accepted length and correction token of a greedy verify
  (``single/eval_async_packed.py:170-175``; ``serving/engine.py:138-145``).
* ``pq_accept_sparse``: standard p/q rejection sampling against a sparse
  proposal, batched (``single/speculative_sampling.py:79-143``, which is
  batch-1 only).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

GREEDY_EPS = 1e-5


def is_greedy(temperature: Optional[float]) -> bool:
    return temperature is None or float(temperature) <= GREEDY_EPS


def _filter_logits(logits: torch.Tensor, temperature: float, top_k: int, top_p: float) -> torch.Tensor:
    logits = logits.float() / float(temperature)
    if top_k and top_k > 0:
        kth = torch.topk(logits, min(int(top_k), logits.shape[-1]), dim=-1).values[..., -1, None]
        logits = logits.masked_fill(logits < kth, torch.finfo(logits.dtype).min)
    if top_p is not None and top_p < 1.0:
        sl, si = torch.sort(logits, descending=True, dim=-1)
        pr = torch.softmax(sl, dim=-1)
        remove = pr.cumsum(-1) > top_p
        remove[..., 1:] = remove[..., :-1].clone()
        remove[..., 0] = False
        sl = sl.masked_fill(remove, torch.finfo(logits.dtype).min)
        logits = torch.full_like(logits, torch.finfo(logits.dtype).min).scatter(-1, si, sl)
    return logits


def sampling_probs(logits: torch.Tensor, temperature: float = 0.0, top_k: int = 0,
                   top_p: float = 1.0) -> torch.Tensor:
    if is_greedy(temperature):
        probs = torch.zeros_like(logits, dtype=torch.float32)
        return probs.scatter_(-1, logits.argmax(-1, keepdim=True), 1.0)
    return torch.softmax(_filter_logits(logits, temperature, top_k, top_p), dim=-1)


def sample_tokens(logits: torch.Tensor, temperature: float = 0.0, top_k: int = 0,
                  top_p: float = 1.0, generator: Optional[torch.Generator] = None) -> torch.Tensor:
    if is_greedy(temperature):
        return logits.argmax(-1)
    probs = sampling_probs(logits, temperature, top_k, top_p)
    flat = probs.reshape(-1, probs.shape[-1])
    return torch.multinomial(flat, 1, generator=generator).reshape(logits.shape[:-1])


def sparse_proposal(logits: torch.Tensor, temperature: float, top_k: int, top_p: float,
                    generator: Optional[torch.Generator] = None
                    ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Sample from the top-k (then top-p) support; return tokens, support ids
    ``[..., S]`` and the exact proposal probabilities on that support."""
    if is_greedy(temperature):
        tok = logits.argmax(-1)
        return tok, tok[..., None], torch.ones(tok.shape + (1,), dtype=torch.float32,
                                               device=logits.device)
    v = logits.shape[-1]
    s = min(int(top_k), v) if int(top_k) > 0 else v
    scaled = logits.float() / float(temperature)
    sl, sid = torch.topk(scaled, k=s, dim=-1)
    if top_p is not None and top_p < 1.0:
        pr = torch.softmax(sl, -1)
        remove = pr.cumsum(-1) > float(top_p)
        remove[..., 1:] = remove[..., :-1].clone()
        remove[..., 0] = False
        sl = sl.masked_fill(remove, torch.finfo(sl.dtype).min)
    sp = torch.softmax(sl, -1)
    local = torch.multinomial(sp.reshape(-1, s), 1, generator=generator).reshape(logits.shape[:-1])
    tok = sid.gather(-1, local[..., None])[..., 0]
    return tok, sid, sp


def greedy_accept(blocks: torch.Tensor, posterior: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """``blocks [B, K]`` = anchor + K-1 drafts, ``posterior [B, K]`` = target
    argmax after each block token.  Returns ``commit [B]`` (anchor + accepted
    drafts, in 1..K) and ``correction [B]`` = ``posterior[commit-1]``."""
    k = blocks.shape[1]
    if k == 1:
        commit = torch.ones(blocks.shape[0], dtype=torch.long, device=blocks.device)
    else:
        match = (blocks[:, 1:] == posterior[:, :-1]).long()
        commit = match.cumprod(dim=1).sum(dim=1) + 1
    corr = posterior.gather(1, (commit - 1)[:, None])[:, 0]
    return commit, corr


def pq_accept_sparse(blocks: torch.Tensor, target_probs: torch.Tensor, q_ids: torch.Tensor,
                     q_probs: torch.Tensor, uniforms: torch.Tensor, correction_u: torch.Tensor
                     ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Batched lossless speculative sampling against a sparse proposal.

    ``blocks [B, K]``; ``target_probs [B, K, V]`` (row i = p after block token
    i); ``q_ids/q_probs [B, K-1, S]`` proposal support of drafts 1..K-1;
    ``uniforms [B, K-1]`` acceptance draws; ``correction_u [B]`` the draw for
    the correction token (inverse-CDF sampling, so the result is a pure
    function of its inputs).  Returns ``commit [B]`` and ``correction [B]``."""
    b, k = blocks.shape
    p = target_probs.float()
    p = p / p.sum(-1, keepdim=True).clamp_min(1e-12)
    qp = q_probs.float()
    qp = qp / qp.sum(-1, keepdim=True).clamp_min(1e-12)
    drafts = blocks[:, 1:].long()
    if k > 1:
        p_tok = p[:, :-1].gather(-1, drafts[..., None])[..., 0]
        q_tok = (qp * (q_ids.long() == drafts[..., None])).sum(-1)
        ok = uniforms <= torch.minimum(torch.ones_like(p_tok), p_tok / q_tok.clamp_min(1e-12))
        acc = ok.long().cumprod(1).sum(1)
    else:
        acc = torch.zeros(b, dtype=torch.long, device=blocks.device)
    commit = acc + 1
    rows = p.gather(1, acc[:, None, None].expand(b, 1, p.shape[-1]))[:, 0].clone()
    rejected = acc < (k - 1)
    if rejected.any():
        idx = acc.clamp(max=max(k - 2, 0))
        sub_ids = q_ids.long().gather(1, idx[:, None, None].expand(b, 1, q_ids.shape[-1]))[:, 0]
        sub_p = qp.gather(1, idx[:, None, None].expand(b, 1, qp.shape[-1]))[:, 0]
        resid = rows.scatter_add(-1, sub_ids, -sub_p).clamp_min(0.0)
        mass = resid.sum(-1, keepdim=True)
        use_resid = rejected[:, None] & (mass > 1e-12)
        rows = torch.where(use_resid, resid / mass.clamp_min(1e-12), rows)
    cdf = rows.cumsum(-1)
    cdf = cdf / cdf[:, -1:].clamp_min(1e-12)
    corr = torch.searchsorted(cdf, correction_u[:, None].float().clamp(0, 1 - 1e-7))[:, 0]
    corr = corr.clamp(max=p.shape[-1] - 1)
    return commit, corr
