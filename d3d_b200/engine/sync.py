"""Synchronous draft-then-verify decoding with multi-step block denoising.

Restates the reference's synchronous primitives (``single/eval_sync.py``):

* a block ``[anchor, MASK x (K-1)]`` is denoised in ``denoising_steps``
  forwards; each step commits the ``k`` most confident masked positions
  (``low_confidence``) or every position above ``threshold`` (``dynamic``,
  capped at ``k``), with the per-step counts of
  ``_get_num_transfer_tokens`` (``eval_sync.py:440-464``);
* the tokens committed by the previous verify ("pending commit") are written
  into the draft KV by the first denoising forward of the next block
  (``d3d_draft_block_fused_commit``, ``eval_sync.py:595-775``);
* ``sync_generate`` is the KV-cached loop (``eval_sync.py:999-1314``) and
  ``sync_generate_nocache`` recomputes the whole prefix every step
  (``eval_sync.py:778-996``).

These run on the PyTorch module (:class:`~d3d_b200.models.qwen3.Qwen3LM`) —
the oracle path; the asynchronous engine uses single-step denoising, as the
reference's async loop requires (``eval_async_packed.py:820-821``).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import torch

from ..models.qwen3 import DenseKVCache, Qwen3LM
from .layout import fused_commit_rows, full_rows, prefix_rows, rows_to_dense
from .sampling import greedy_accept, is_greedy, sampling_probs, sample_tokens


def num_transfer_tokens(num_masks: int, steps: int) -> List[int]:
    steps = max(1, int(steps))
    base, extra = divmod(int(num_masks), steps)
    return [base + (1 if i < extra else 0) for i in range(steps)]


def select_transfer(block: torch.Tensor, mask_index: torch.Tensor, x0: torch.Tensor, x0_p: torch.Tensor,
                    k: int, remasking: str, threshold: float) -> Optional[torch.Tensor]:
    """Commit up to ``k`` masked positions of ``block [1, L]`` in place."""
    if k <= 0 or not bool(mask_index.any()):
        return None
    scores = x0_p.masked_fill(~mask_index, -1.0)
    k = min(int(k), int(mask_index.sum()))
    if "dynamic" in (remasking or ""):
        confident = (scores >= threshold) & mask_index
        if bool(confident.any()):
            idx = confident.nonzero(as_tuple=True)[1]
            if idx.numel() > k:
                idx = idx[torch.topk(scores[:, idx], k, dim=-1).indices[0]]
        else:
            idx = torch.topk(scores, k, dim=-1).indices[0]
    else:
        idx = torch.topk(scores, k, dim=-1).indices[0]
    block[:, idx] = x0[:, idx]
    return idx


@dataclass
class DraftResult:
    block: torch.Tensor                      # [1, L]
    proposal_probs: Optional[torch.Tensor]   # [1, L, V] (sampling)
    top_tokens: Optional[torch.Tensor]       # [1, L, k] from the last step


def _logits(model: Qwen3LM, ids, positions, mask, cache, store, cond=None):
    h = model(ids, positions, mask=mask, cache=cache, store_kv=store, cond=cond)
    return model.logits(h).float()


@torch.inference_mode()
def draft_block(model: Qwen3LM, block: torch.Tensor, *, cache: DenseKVCache, cache_len: int,
                pending: Optional[torch.Tensor], denoising_steps: int, remasking: str = "low_confidence",
                threshold: float = 0.9, temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0,
                mask_id: int, mode: str = "block_causal", return_topk: int = 0,
                cond: Optional[torch.Tensor] = None,
                generator: Optional[torch.Generator] = None) -> DraftResult:
    """Denoise ``block`` against the draft KV; the first forward also commits
    ``pending`` (tokens verified since the KV was last written)."""
    dev = block.device
    cur = block.clone()
    p = 0 if pending is None else int(pending.shape[1])
    L = int(cur.shape[1])
    num_masks = int((cur == mask_id).sum())
    probs_out = None
    if num_masks == 0:
        if p:
            ids = torch.cat([pending, cur], 1)
            rows = fused_commit_rows(cache_len, p, L, mode, dev)
            cache.crop(cache_len)
            _logits(model, ids, torch.arange(cache_len, cache_len + p + L, device=dev)[None],
                    rows_to_dense(rows, cache_len + p + L)[None], cache, True, cond)
            cache.crop(cache_len + p)
        return DraftResult(cur, None, None)
    schedule = num_transfer_tokens(num_masks, denoising_steps)
    written = False
    last_logits = None
    for step, k in enumerate(schedule):
        mask_index = cur == mask_id
        if not bool(mask_index.any()):
            break
        if p and not written:
            ids = torch.cat([pending, cur], 1)
            rows = fused_commit_rows(cache_len, p, L, mode, dev)
            cache.crop(cache_len)
            logits = _logits(model, ids, torch.arange(cache_len, cache_len + p + L, device=dev)[None],
                             rows_to_dense(rows, cache_len + p + L)[None], cache, True, cond)[:, p:]
            cache.crop(cache_len + p)
            written = True
        else:
            base = cache_len + (p if written else 0)
            rows = full_rows(base + L, L, dev)
            logits = _logits(model, cur, torch.arange(base, base + L, device=dev)[None],
                             rows_to_dense(rows, base + L)[None], cache, False, cond)
        if step == len(schedule) - 1:
            k = int(mask_index.sum())
            last_logits = logits
        if is_greedy(temperature):
            x0 = logits.argmax(-1)
            x0_p = torch.softmax(logits, -1).gather(-1, x0[..., None])[..., 0]
        else:
            pr = sampling_probs(logits, temperature, top_k, top_p)
            x0 = torch.multinomial(pr[0], 1, generator=generator).view(1, -1)
            x0_p = pr.gather(-1, x0[..., None])[..., 0]
            if probs_out is None:
                probs_out = torch.zeros(1, L, logits.shape[-1], device=dev)
        idx = select_transfer(cur, mask_index, x0, x0_p, k, remasking, threshold)
        if probs_out is not None and idx is not None:
            probs_out[:, idx] = sampling_probs(logits, temperature, top_k, top_p)[:, idx]
    top = None
    if return_topk and last_logits is not None:
        top = torch.topk(last_logits, min(return_topk, last_logits.shape[-1]), -1).indices
    return DraftResult(cur, probs_out, top)


def pq_accept_dense(drafts: torch.Tensor, target_probs: torch.Tensor, draft_probs: torch.Tensor,
                    generator: Optional[torch.Generator] = None):
    """Standard p/q rejection sampling against a dense proposal
    (``single/speculative_sampling.py:15-76``); batch 1.  Returns
    ``(accepted_drafts, correction_token)``."""
    p = target_probs.float()[0]
    p = p / p.sum(-1, keepdim=True).clamp_min(1e-12)
    q = draft_probs.float()[0]
    q = q / q.sum(-1, keepdim=True).clamp_min(1e-12)
    k = drafts.shape[1]
    tok = drafts[0].long()
    pos = torch.arange(k, device=tok.device)
    ratio = torch.minimum(torch.ones(k, device=tok.device), p[pos, tok] / q[pos, tok].clamp_min(1e-12))
    u = torch.rand(k, generator=generator, device="cpu").to(tok.device)
    rej = (u > ratio).nonzero(as_tuple=True)[0]
    if rej.numel() == 0:
        n, dist = k, p[k]
    else:
        n = int(rej[0])
        resid = (p[n] - q[n]).clamp_min(0.0)
        dist = p[n] if float(resid.sum()) <= 1e-12 else resid / resid.sum()
    corr = torch.multinomial(dist.cpu(), 1, generator=generator).to(tok.device)
    return n, corr


@dataclass
class SyncStats:
    output_tokens: List[int]
    acceptance_lengths: List[int] = field(default_factory=list)
    decode_elapsed_s: float = 0.0
    num_input_tokens: int = 0


@torch.inference_mode()
def sync_generate(target: Qwen3LM, drafter: Qwen3LM, prompt: Sequence[int], max_new_tokens: int, *,
                  block_size: int = 16, denoising_steps: int = 1, remasking: str = "low_confidence",
                  threshold: float = 0.9, temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0,
                  mode: str = "block_causal", stop_ids: Sequence[int] = (), seed: int = 0) -> SyncStats:
    """KV-cached synchronous speculative decoding (one request)."""
    dev = next(target.parameters()).device
    mask_id = int(drafter.cfg.mask_token_id)
    gen = torch.Generator().manual_seed(seed)
    ids = torch.tensor([list(prompt)], dtype=torch.long, device=dev)
    n_in = ids.shape[1]
    max_len = n_in + int(max_new_tokens)
    tkv, dkv = DenseKVCache(target.cfg.num_hidden_layers), DenseKVCache(drafter.cfg.num_hidden_layers)
    h = target(ids, cache=tkv, store_kv=True)
    last = target.logits(h[:, -1:]).float()
    anchor = sample_tokens(last, temperature, top_k, top_p, gen)[:, 0]
    cond = h[:, -1] if drafter.cfg.cond_hidden_size else None
    drafter(ids, mask=rows_to_dense(prefix_rows(0, n_in, mode, block_size, dev), n_in)[None], cache=dkv,
            store_kv=True)
    kv_len, draft_kv_len = n_in, n_in
    pending = ids.new_empty((1, 0))
    out: List[int] = []
    accepts: List[int] = []
    t0 = time.perf_counter()
    while kv_len < max_len:
        L = min(block_size, max_len - kv_len)
        block = torch.full((1, L), mask_id, dtype=torch.long, device=dev)
        block[:, 0] = anchor
        probs = None
        if L > 1:
            r = draft_block(drafter, block, cache=dkv, cache_len=draft_kv_len,
                            pending=pending if pending.shape[1] else None, denoising_steps=denoising_steps,
                            remasking=remasking, threshold=threshold, temperature=temperature, top_k=top_k,
                            top_p=top_p, mask_id=mask_id, mode=mode, cond=cond, generator=gen)
            block, probs = r.block, r.proposal_probs
            if pending.shape[1]:
                draft_kv_len = kv_len
                pending = ids.new_empty((1, 0))
        tkv.crop(kv_len)
        th = target(block, torch.arange(kv_len, kv_len + L, device=dev)[None], cache=tkv, store_kv=True)
        tl = target.logits(th).float()
        if not is_greedy(temperature) and L > 1:
            tp = sampling_probs(tl, temperature, top_k, top_p)
            n, corr = pq_accept_dense(block[:, 1:], tp, probs[:, 1:L], gen)
            commit = n + 1
            corr_tok = int(corr[0])
        else:
            post = sample_tokens(tl, temperature, top_k, top_p, gen)
            c, cr = greedy_accept(block, post)
            commit, corr_tok = int(c[0]), int(cr[0])
        toks = block[0, :commit].tolist()
        tkv.crop(kv_len + commit)
        if drafter.cfg.cond_hidden_size:
            cond = th[:, commit - 1]
        pending = block[:, :commit]
        kv_len += commit
        accepts.append(commit)
        out.extend(toks)
        anchor = torch.tensor([corr_tok], device=dev)
        if any(t in stop_ids for t in toks):
            break
        if kv_len < max_len and corr_tok in stop_ids:
            out.append(corr_tok)
            break
    out = out[:max_new_tokens]
    for i, t in enumerate(out):
        if t in stop_ids:
            out = out[: i + 1]
            break
    return SyncStats(out, accepts, time.perf_counter() - t0, n_in)


@torch.inference_mode()
def sync_generate_nocache(target: Qwen3LM, drafter: Qwen3LM, prompt: Sequence[int], max_new_tokens: int, *,
                          block_size: int = 16, denoising_steps: int = 1, remasking: str = "low_confidence",
                          threshold: float = 0.9, mode: str = "block_causal",
                          stop_ids: Sequence[int] = ()) -> SyncStats:
    """Greedy synchronous decoding that recomputes the full prefix every step
    (no KV cache on either model)."""
    dev = next(target.parameters()).device
    mask_id = int(drafter.cfg.mask_token_id)
    seq = list(prompt)
    n_in = len(seq)
    max_len = n_in + int(max_new_tokens)
    anchor = int(target.logits(target(torch.tensor([seq], device=dev))[:, -1]).argmax(-1))
    out: List[int] = []
    accepts: List[int] = []
    t0 = time.perf_counter()
    while len(seq) < max_len:
        L = min(block_size, max_len - len(seq))
        block = torch.full((1, L), mask_id, dtype=torch.long, device=dev)
        block[:, 0] = anchor
        if L > 1:
            schedule = num_transfer_tokens(int((block == mask_id).sum()), denoising_steps)
            for step, k in enumerate(schedule):
                mask_index = block == mask_id
                if not bool(mask_index.any()):
                    break
                if step == len(schedule) - 1:
                    k = int(mask_index.sum())
                n = len(seq)
                ids = torch.cat([torch.tensor([seq], device=dev), block], 1)
                rows = torch.cat([prefix_rows(0, n, mode, block_size, dev), full_rows(n + L, L, dev)], 0)
                logits = drafter.logits(drafter(ids, mask=rows_to_dense(rows, n + L)[None]))[:, n:].float()
                x0 = logits.argmax(-1)
                x0_p = torch.softmax(logits, -1).gather(-1, x0[..., None])[..., 0]
                select_transfer(block, mask_index, x0, x0_p, k, remasking, threshold)
        full = torch.tensor([seq + block[0].tolist()], device=dev)
        post = target.logits(target(full))[:, len(seq):].argmax(-1)
        c, cr = greedy_accept(block, post)
        commit = int(c[0])
        toks = block[0, :commit].tolist()
        seq.extend(toks)
        out.extend(toks)
        accepts.append(commit)
        anchor = int(cr[0])
        if any(t in stop_ids for t in toks) or (len(seq) < max_len and anchor in stop_ids):
            if anchor in stop_ids and not any(t in stop_ids for t in toks):
                out.append(anchor)
            break
    out = out[:max_new_tokens]
    return SyncStats(out, accepts, time.perf_counter() - t0, n_in)
