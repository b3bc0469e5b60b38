"""Attention layouts of every drafter/target forward, in structured form.

Every query row of every forward this framework runs sees a key set of the
shape ``{k : k < lim} ∪ {k : lo <= k < hi}`` (key index = KV slot of the
sequence).  The CUDA attention kernels take exactly these three int32 numbers
per row (``rows[..., 3]``) instead of a dense ``[Q, S]`` boolean mask, skip key
tiles that no row of a query tile sees, and never read a mask from memory.
:func:`rows_to_dense` expands the descriptors into the dense mask the CPU oracle
(SDPA) uses, so both paths share one definition.

The layouts restate the reference's mask builders:

* prefix prefill, causal or block-causal (``single/eval_sync.py:194-261``);
* the fused pending-commit draft mask (``single/eval_sync.py:249-275``);
* recovery drafting from an anchor: the block sees the prefix and itself
  (``single/eval_sync.py:519-528``; ``serving/engine.py:37-39``);
* the packed all-outcome forward (``single/eval_async_packed.py:467-661``;
  ``serving/engine.py:34-48``): the pending block first (causal or
  block-causal), then one K-token segment per branch, each seeing the prefix,
  the accepted part of the pending block and its own segment.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch

BranchKey = Tuple[int, Optional[int]]   # (commit length, anchor token or None for all-pass)


def rows_to_dense(rows: torch.Tensor, kv_len: int) -> torch.Tensor:
    """``rows [..., Q, 3]`` (lim, lo, hi) → bool ``[..., Q, kv_len]``."""
    k = torch.arange(kv_len, device=rows.device)
    lim = rows[..., 0:1]
    lo = rows[..., 1:2]
    hi = rows[..., 2:3]
    return (k < lim) | ((k >= lo) & (k < hi))


def causal_rows(start: int, q_len: int, device=None) -> torch.Tensor:
    """Row i (absolute slot start+i) sees slots [0, start+i]."""
    lim = torch.arange(start + 1, start + q_len + 1, dtype=torch.int32, device=device)
    z = torch.zeros_like(lim)
    return torch.stack([lim, z, z], dim=-1)


def block_causal_rows(start: int, q_len: int, block_size: int, device=None) -> torch.Tensor:
    """Block-causal prefix: slot p sees every slot of blocks <= block(p).

    Restates ``single/eval_sync.py:_block_causal_mask`` for a prefix written
    from slot ``start`` (blocks are counted from slot 0)."""
    p = torch.arange(start, start + q_len, dtype=torch.int64, device=device)
    lim = ((p // block_size) + 1) * block_size
    lim = torch.minimum(lim, torch.tensor(start + q_len, device=device))
    lim = lim.to(torch.int32)
    z = torch.zeros_like(lim)
    return torch.stack([lim, z, z], dim=-1)


def prefix_rows(start: int, q_len: int, mode: str, block_size: int, device=None) -> torch.Tensor:
    if mode == "causal":
        return causal_rows(start, q_len, device)
    if mode == "block_causal":
        return block_causal_rows(start, q_len, block_size, device)
    raise ValueError(f"unsupported attention_mask_mode={mode!r}")


def full_rows(kv_end: int, q_len: int, device=None) -> torch.Tensor:
    """Every row sees slots [0, kv_end) — recovery drafting and plain blocks."""
    lim = torch.full((q_len,), kv_end, dtype=torch.int32, device=device)
    z = torch.zeros_like(lim)
    return torch.stack([lim, z, z], dim=-1)


def pending_rows(kv_len: int, pending_len: int, mode: str, device=None) -> torch.Tensor:
    """Rows of a pending block written at slots [kv_len, kv_len+pending_len)."""
    if mode == "causal":
        return causal_rows(kv_len, pending_len, device)
    if mode == "block_causal":
        return full_rows(kv_len + pending_len, pending_len, device)
    raise ValueError(f"unsupported attention_mask_mode={mode!r}")


@dataclass
class PackedLayout:
    """One packed all-outcome forward for one sequence.

    ``input_ids``/``positions``/``rows`` have ``pending_len + n_branches*seg`` entries;
    ``slot_start`` is the KV slot of query row 0 (= draft KV length);
    ``keys[j]`` is branch j's key; its tokens are rows
    ``pending_len + j*seg .. +seg``.
    """
    input_ids: torch.Tensor
    positions: torch.Tensor
    rows: torch.Tensor
    keys: List[BranchKey]
    pending_len: int
    seg: int
    slot_start: int

    @property
    def q_len(self) -> int:
        return int(self.input_ids.shape[0])

    def segment(self, j: int) -> slice:
        s = self.pending_len + j * self.seg
        return slice(s, s + self.seg)


def branch_specs(pending_block: Sequence[int], top_tokens: Optional[Sequence[Sequence[int]]],
                 anchor_num: int, accepted_counts: Optional[Sequence[int]] = None
                 ) -> List[BranchKey]:
    """Branch keys of the packed forward (``single/eval_async_packed.py:497-530``).

    For each commit length ``a`` < K the anchors are the draft's top-(A+1)
    tokens at block position ``a`` other than the token already in the block
    there (had the target agreed with it, more would have been accepted).  The
    all-pass outcome ``a == K`` gets one branch keyed ``None``: its anchor (the
    target's bonus token) is unknown when the branch is drafted, so its slot 0
    stays ``MASK`` and is overwritten after verification."""
    k = len(pending_block)
    counts = range(1, k + 1) if accepted_counts is None else [c for c in accepted_counts if c <= k]
    specs: List[BranchKey] = []
    for a in counts:
        if anchor_num == 0 or a == k:
            specs.append((a, None))
            continue
        if top_tokens is None:
            raise RuntimeError("packed anchor candidates require pending top-token logits")
        cand = [int(t) for t in top_tokens[a][: anchor_num + 1] if int(t) != int(pending_block[a])]
        cand = cand[:anchor_num]
        if len(cand) != anchor_num:
            raise RuntimeError(f"only selected {len(cand)} anchors for anchor_num={anchor_num}")
        specs.extend((a, t) for t in cand)
    return specs


def packed_layout(pending_block, specs: Sequence[BranchKey], kv_len: int,
                  seg: int, mask_id: int, mode: str) -> PackedLayout:
    """Build ids / RoPE positions / row descriptors of the packed forward.

    KV slots run contiguously from ``kv_len`` over all query rows (the
    reference stores the whole packed query and crops back to
    ``kv_len + pending_len`` afterwards); RoPE positions of branch j start at
    ``kv_len + a_j``.  Built with vectorised numpy (this runs on the host on
    every decode step); the returned tensors share the numpy buffers."""
    pend = np.asarray(pending_block.tolist() if isinstance(pending_block, torch.Tensor) else pending_block,
                      dtype=np.int64)
    p = int(pend.shape[0])
    nb = len(specs)
    q = p + nb * seg
    ids = np.full(q, int(mask_id), dtype=np.int64)
    ids[:p] = pend
    pos = np.empty(q, dtype=np.int64)
    pos[:p] = np.arange(kv_len, kv_len + p)
    rows = np.zeros((q, 3), dtype=np.int32)
    if mode == "causal":
        rows[:p, 0] = np.arange(kv_len + 1, kv_len + p + 1)
    elif mode == "block_causal":
        rows[:p, 0] = kv_len + p
    else:
        raise ValueError(f"unsupported attention_mask_mode={mode!r}")
    if nb:
        acc = np.array([a for a, _ in specs], dtype=np.int64)
        starts = p + np.arange(nb, dtype=np.int64) * seg
        off = np.arange(seg, dtype=np.int64)
        pos[p:] = (kv_len + acc[:, None] + off[None, :]).reshape(-1)
        br = rows[p:].reshape(nb, seg, 3)
        br[:, :, 0] = (kv_len + acc)[:, None]
        br[:, :, 1] = (kv_len + starts)[:, None]
        br[:, :, 2] = (kv_len + starts + seg)[:, None]
        anchors = [(j, t) for j, (_, t) in enumerate(specs) if t is not None]
        if anchors:
            js = np.array([j for j, _ in anchors], dtype=np.int64)
            ids[p + js * seg] = np.array([t for _, t in anchors], dtype=np.int64)
    return PackedLayout(torch.from_numpy(ids), torch.from_numpy(pos), torch.from_numpy(rows),
                        list(specs), p, seg, kv_len)


def fused_commit_rows(kv_len: int, pending_len: int, block_len: int, mode: str,
                      device=None) -> torch.Tensor:
    """Pending commit followed by a block drafted in the same forward
    (``single/eval_sync.py:_fused_draft_mask``)."""
    q = pending_len + block_len
    rows = full_rows(kv_len + q, q, device)
    if mode == "causal":
        if pending_len:
            rows[:pending_len] = causal_rows(kv_len, pending_len, device)
    elif mode == "block_causal":
        if pending_len and block_len:
            rows[:pending_len, 0] = kv_len + pending_len
    else:
        raise ValueError(f"unsupported attention_mask_mode={mode!r}")
    return rows


def paged_draft_branch_tokens(block_size: int, anchor_num: int) -> int:
    """Extra KV slots one packed forward needs (``common/runtime.py:46-64``)."""
    return block_size * (2 + (block_size - 1) * anchor_num)
