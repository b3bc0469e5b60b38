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
from typing import Any, Dict, List, Optional, Sequence

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




def _logits(model: Qwen3LM, ids, positions, mask, cache, store, cond=None, anchors: Sequence[int] = (0,)):
    """Logits of ``ids``; a conditioned drafter adds ``cond`` at the block
    anchor rows ``anchors`` (as the engine's packed forwards do)."""
    rows = None
    if cond is not None:
        rows = torch.zeros(ids.shape, dtype=torch.bool, device=ids.device)
        rows[:, list(anchors)] = True
    h = model(ids, positions, mask=mask, cache=cache, store_kv=store, cond=cond, cond_rows=rows)
    return model.logits(h).float()


def _denoise(cur: torch.Tensor, mask_id: int, denoising_steps: int, logits_at, *, remasking: str,
             threshold: float, temperature: float, top_k: int, top_p: float,
             generator: Optional[torch.Generator]):
    """The denoising schedule over ``cur [1, L]`` (in place).  ``logits_at(step,
    cur)`` returns the drafter's ``[1, L, V]`` logits for the current block; the
    last step commits every position still masked.  Returns the proposal
    distribution of each committed position (sampling only) and the last
    step's logits."""
    probs_out, last = None, None
    schedule = num_transfer_tokens(int((cur == mask_id).sum()), denoising_steps)
    for step, k in enumerate(schedule):
        mask_index = cur == mask_id
        if not bool(mask_index.any()):
            break
        logits = logits_at(step, cur)
        if step == len(schedule) - 1:
            k = int(mask_index.sum())
            last = logits
        if is_greedy(temperature):
            x0 = logits.argmax(-1)
            x0_p = torch.softmax(logits, -1).gather(-1, x0[..., None])[..., 0]
            select_transfer(cur, mask_index, x0, x0_p, k, remasking, threshold)
            continue
        pr = sampling_probs(logits, temperature, top_k, top_p)
        x0 = torch.multinomial(pr[0], 1, generator=generator).view(1, -1)
        x0_p = pr.gather(-1, x0[..., None])[..., 0]
        if probs_out is None:
            probs_out = torch.zeros_like(pr)
        idx = select_transfer(cur, mask_index, x0, x0_p, k, remasking, threshold)
        if idx is not None:
            probs_out[:, idx] = pr[:, idx]
    return probs_out, last


def _top(last: Optional[torch.Tensor], k: int) -> Optional[torch.Tensor]:
    if not k or last is None:
        return None
    return torch.topk(last, min(k, last.shape[-1]), -1).indices


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
    written = False

    def commit_forward():
        ids = torch.cat([pending, cur], 1)
        rows = fused_commit_rows(cache_len, p, L, mode, dev)
        cache.crop(cache_len)
        out = _logits(model, ids, torch.arange(cache_len, cache_len + p + L, device=dev)[None],
                      rows_to_dense(rows, cache_len + p + L)[None], cache, True, cond, (0, p))[:, p:]
        cache.crop(cache_len + p)
        return out

    def logits_at(step, cur_):
        nonlocal written
        if p and not written:
            written = True
            return commit_forward()
        base = cache_len + (p if written else 0)
        return _logits(model, cur_, torch.arange(base, base + L, device=dev)[None],
                       rows_to_dense(full_rows(base + L, L, dev), base + L)[None], cache, False, cond)

    if not bool((cur == mask_id).any()):
        if p:
            commit_forward()
        return DraftResult(cur, None, None)
    probs, last = _denoise(cur, mask_id, denoising_steps, logits_at, remasking=remasking, threshold=threshold,
                           temperature=temperature, top_k=top_k, top_p=top_p, generator=generator)
    return DraftResult(cur, probs, _top(last, return_topk))


@torch.inference_mode()
def draft_block_nocache(model: Qwen3LM, prefix: torch.Tensor, block: torch.Tensor, *, denoising_steps: int,
                        remasking: str = "low_confidence", threshold: float = 0.9, temperature: float = 0.0,
                        top_k: int = 0, top_p: float = 1.0, mask_id: int, mode: str = "block_causal",
                        block_size: int = 16, cond: Optional[torch.Tensor] = None,
                        generator: Optional[torch.Generator] = None) -> DraftResult:
    """Denoise ``block`` by re-reading the whole ``prefix [1, n]`` every step
    (no draft KV; ``d3d_draft_block``, ``single/eval_sync.py:483-593``)."""
    dev = block.device
    cur = block.clone()
    n, L = int(prefix.shape[1]), int(cur.shape[1])
    rows = torch.cat([prefix_rows(0, n, mode, block_size, dev), full_rows(n + L, L, dev)], 0)
    mask = rows_to_dense(rows, n + L)[None]

    def logits_at(step, cur_):
        return _logits(model, torch.cat([prefix, cur_], 1), None, mask, None, False, cond, (n,))[:, n:]

    probs, _ = _denoise(cur, mask_id, denoising_steps, logits_at, remasking=remasking, threshold=threshold,
                        temperature=temperature, top_k=top_k, top_p=top_p, generator=generator)
    return DraftResult(cur, probs, None)


def pq_accept_dense(drafts: torch.Tensor, target_probs: torch.Tensor, draft_probs: torch.Tensor,
                    generator: Optional[torch.Generator] = None):
    """Standard p/q rejection sampling against a dense proposal
    (``single/speculative_sampling.py:15-76``); batch 1.  Returns
    ``(accepted_drafts, correction_token)``.  Draws come from ``generator``
    on its own device (CPU when none is given)."""
    gdev = generator.device if generator is not None else torch.device("cpu")
    p = target_probs.float()[0].to(gdev)
    p = p / p.sum(-1, keepdim=True).clamp_min(1e-12)
    q = draft_probs.float()[0].to(gdev)
    q = q / q.sum(-1, keepdim=True).clamp_min(1e-12)
    k = drafts.shape[1]
    tok = drafts[0].long().to(gdev)
    pos = torch.arange(k, device=gdev)
    ratio = torch.minimum(torch.ones(k, device=gdev), p[pos, tok] / q[pos, tok].clamp_min(1e-12))
    u = torch.rand(k, generator=generator, device=gdev)
    rej = (u > ratio).nonzero(as_tuple=True)[0]
    if rej.numel() == 0:
        n, dist = k, p[k]
    else:
        n = int(rej[0])
        resid = (p[n] - q[n]).clamp_min(0.0)
        dist = p[n] if float(resid.sum()) <= 1e-12 else resid / resid.sum()
    corr = torch.multinomial(dist, 1, generator=generator).to(drafts.device)
    return n, corr


@dataclass
class SyncStats:
    """One request's synchronous decode: the output, one entry per verify in
    each per-step list, and host/device time per stage."""
    output_tokens: List[int]
    acceptance_lengths: List[int] = field(default_factory=list)
    decode_elapsed_s: float = 0.0            # verifier prefill included
    num_input_tokens: int = 0
    draft_blocks: List[List[int]] = field(default_factory=list)    # drafted tokens after the anchor
    target_blocks: List[List[int]] = field(default_factory=list)   # target's token after each block position
    emitted_blocks: List[List[int]] = field(default_factory=list)  # committed tokens
    stopped: List[bool] = field(default_factory=list)
    stage_records: List[Dict[str, Any]] = field(default_factory=list)
    verifier_prefill_s: float = 0.0
    draft_prefill_s: float = 0.0
    draft_s: float = 0.0
    verify_s: float = 0.0
    draft_gpu_s: float = 0.0
    verify_gpu_s: float = 0.0

    @property
    def time_per_output_token(self) -> float:
        return self.decode_elapsed_s / max(len(self.output_tokens), 1)


class _Stage:
    """Wall time of one stage, the device synchronized on both sides, and with
    ``events`` its device time from CUDA events on the current stream."""

    def __init__(self, device, events: bool):
        self.dev = torch.device(device)
        self.cuda = self.dev.type == "cuda"
        self.events = bool(events) and self.cuda
        self.wall = self.gpu = 0.0

    def __enter__(self):
        if self.cuda:
            torch.cuda.synchronize(self.dev)
        if self.events:
            self.e0 = torch.cuda.Event(enable_timing=True)
            self.e1 = torch.cuda.Event(enable_timing=True)
            self.e0.record(torch.cuda.current_stream(self.dev))
        self.t0 = time.perf_counter()
        return self

    def __exit__(self, *exc):
        if self.events:
            self.e1.record(torch.cuda.current_stream(self.dev))
        if self.cuda:
            torch.cuda.synchronize(self.dev)
        self.wall = time.perf_counter() - self.t0
        if self.events:
            self.gpu = self.e0.elapsed_time(self.e1) / 1e3
        return False


@torch.inference_mode()
def _sync_decode(target: Qwen3LM, drafter: Qwen3LM, prompt: Sequence[int], max_new_tokens: int, *, cached: bool,
                 block_size: int, denoising_steps: int, remasking: str, threshold: float, temperature: float,
                 top_k: int, top_p: float, target_top_k: int, target_top_p: float, mode: str,
                 stop_ids: Sequence[int], seed: int, collect_stage_timings: bool) -> SyncStats:
    """Draft a block, verify it, commit, repeat — one request.  The drafter may
    sit on another device than the target (tokens and the conditioning hidden
    state cross over; ``single/eval_sync.py`` ``draft_device``)."""
    tdev = next(target.parameters()).device
    ddev = next(drafter.parameters()).device
    mask_id = int(drafter.cfg.mask_token_id)
    gen_t = torch.Generator(device=tdev).manual_seed(seed)
    gen_d = gen_t if ddev == tdev else torch.Generator(device=ddev).manual_seed(seed + 1)
    stop_ids = set(int(t) for t in stop_ids)
    st = SyncStats([], num_input_tokens=len(prompt))
    if max_new_tokens <= 0:
        return st
    ids = torch.tensor([list(prompt)], dtype=torch.long, device=tdev)
    n_in = ids.shape[1]
    max_len = n_in + int(max_new_tokens)
    sampled = not is_greedy(temperature)
    conditioned = bool(drafter.cfg.cond_hidden_size)
    tkv = DenseKVCache(target.cfg.num_hidden_layers) if cached else None
    dkv = DenseKVCache(drafter.cfg.num_hidden_layers) if cached else None
    draft_kw = dict(denoising_steps=denoising_steps, remasking=remasking, threshold=threshold,
                    temperature=temperature, top_k=top_k, top_p=top_p, mask_id=mask_id, mode=mode,
                    generator=gen_d)
    t_start = time.perf_counter()
    with _Stage(tdev, collect_stage_timings) as sp:
        h = target(ids, cache=tkv, store_kv=cached)
        anchor = sample_tokens(target.logits(h[:, -1:]).float(), temperature, target_top_k, target_top_p,
                               gen_t)[:, 0]
    st.verifier_prefill_s = sp.wall
    cond = h[:, -1].to(ddev) if conditioned else None
    draft_len, pending, seq = n_in, None, ids
    if cached:
        with _Stage(ddev, collect_stage_timings) as sd:
            drafter(ids.to(ddev), mask=rows_to_dense(prefix_rows(0, n_in, mode, block_size, ddev), n_in)[None],
                    cache=dkv, store_kv=True)
        st.draft_prefill_s = sd.wall
    kv_len = n_in
    out: List[int] = []
    while kv_len < max_len:
        L = min(block_size, max_len - kv_len)
        block = torch.full((1, L), mask_id, dtype=torch.long, device=ddev)
        block[:, 0] = anchor.to(ddev)
        probs = None
        sd = _Stage(ddev, collect_stage_timings)
        if L > 1:
            with sd:
                if cached:
                    r = draft_block(drafter, block, cache=dkv, cache_len=draft_len, pending=pending,
                                    cond=cond, **draft_kw)
                    if pending is not None:
                        draft_len, pending = kv_len, None
                else:
                    r = draft_block_nocache(drafter, seq.to(ddev), block, block_size=block_size, cond=cond,
                                            **draft_kw)
            block, probs = r.block, r.proposal_probs
        block = block.to(tdev)
        with _Stage(tdev, collect_stage_timings) as sv:
            if cached:
                tkv.crop(kv_len)
                th = target(block, torch.arange(kv_len, kv_len + L, device=tdev)[None], cache=tkv, store_kv=True)
            else:
                th = target(torch.cat([seq, block], 1))[:, kv_len:]
            tl = target.logits(th).float()
        if sampled and L > 1:
            tp = sampling_probs(tl, temperature, target_top_k, target_top_p)
            n, corr = pq_accept_dense(block[:, 1:], tp, probs[:, 1:L].to(tdev), gen_t)
            commit, corr_tok = n + 1, int(corr[0])
            post = tp.argmax(-1)
        else:
            post = sample_tokens(tl, temperature, target_top_k, target_top_p, gen_t)
            c, cr = greedy_accept(block, post)
            commit, corr_tok = int(c[0]), int(cr[0])
        toks = block[0, :commit].tolist()
        if cached:
            tkv.crop(kv_len + commit)
            pending = block[:, :commit].to(ddev)
        else:
            seq = torch.cat([seq, block[:, :commit]], 1)
        if conditioned:
            cond = th[:, commit - 1].to(ddev)
        before = kv_len
        kv_len += commit
        out.extend(toks)
        anchor = torch.tensor([corr_tok], device=tdev)
        hit = any(t in stop_ids for t in toks)
        stop = hit or (kv_len < max_len and corr_tok in stop_ids)
        st.acceptance_lengths.append(commit)
        st.draft_blocks.append(block[0, 1:].tolist())
        st.target_blocks.append(post[0].tolist())
        st.emitted_blocks.append(toks)
        st.stopped.append(stop)
        st.draft_s += sd.wall
        st.verify_s += sv.wall
        st.draft_gpu_s += sd.gpu
        st.verify_gpu_s += sv.gpu
        if collect_stage_timings:
            st.stage_records.append({
                "step_index": len(st.acceptance_lengths) - 1, "prefix_len_before": before,
                "generated_len_before": before - n_in, "block_size": L, "accepted_draft_tokens": commit - 1,
                "accept_length": commit, "prefix_len_after": kv_len, "generated_len_after": kv_len - n_in,
                "draft_wall_s": sd.wall, "draft_gpu_s": sd.gpu, "verify_wall_s": sv.wall,
                "verify_gpu_s": sv.gpu, "round_wall_s": sd.wall + sv.wall, "round_gpu_s": sd.gpu + sv.gpu})
        if stop:
            if not hit:
                out.append(corr_tok)
            break
    out = out[:max_new_tokens]
    for i, t in enumerate(out):
        if t in stop_ids:
            out = out[: i + 1]
            break
    st.output_tokens = out
    st.decode_elapsed_s = time.perf_counter() - t_start
    return st


def sync_generate(target: Qwen3LM, drafter: Qwen3LM, prompt: Sequence[int], max_new_tokens: int, *,
                  block_size: int = 16, denoising_steps: int = 1, remasking: str = "low_confidence",
                  threshold: float = 0.9, temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0,
                  target_top_k: int = 0, target_top_p: float = 1.0, mode: str = "block_causal",
                  stop_ids: Sequence[int] = (), seed: int = 0, collect_stage_timings: bool = False) -> SyncStats:
    """KV-cached synchronous speculative decoding of one request
    (``run_d3d_generate_cached``, ``single/eval_sync.py:999-1314``)."""
    return _sync_decode(target, drafter, prompt, max_new_tokens, cached=True, block_size=block_size,
                        denoising_steps=denoising_steps, remasking=remasking, threshold=threshold,
                        temperature=temperature, top_k=top_k, top_p=top_p, target_top_k=target_top_k,
                        target_top_p=target_top_p, mode=mode, stop_ids=stop_ids, seed=seed,
                        collect_stage_timings=collect_stage_timings)


def sync_generate_nocache(target: Qwen3LM, drafter: Qwen3LM, prompt: Sequence[int], max_new_tokens: int, *,
                          block_size: int = 16, denoising_steps: int = 1, remasking: str = "low_confidence",
                          threshold: float = 0.9, temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0,
                          target_top_k: int = 0, target_top_p: float = 1.0, mode: str = "block_causal",
                          stop_ids: Sequence[int] = (), seed: int = 0,
                          collect_stage_timings: bool = False) -> SyncStats:
    """Synchronous decoding that recomputes the full prefix every step on both
    models (no KV cache; ``run_d3d_generate``, ``single/eval_sync.py:778-996``)."""
    return _sync_decode(target, drafter, prompt, max_new_tokens, cached=False, block_size=block_size,
                        denoising_steps=denoising_steps, remasking=remasking, threshold=threshold,
                        temperature=temperature, top_k=top_k, top_p=top_p, target_top_k=target_top_k,
                        target_top_p=target_top_p, mode=mode, stop_ids=stop_ids, seed=seed,
                        collect_stage_timings=collect_stage_timings)
