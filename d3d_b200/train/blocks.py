"""Packed anchor+MASK training blocks (reference: ``train/blocks.py:73-239``).

Each example is ``prompt + response``.  Up to ``max_anchors`` response
offsets are chosen as anchors; block j is ``[response[s_j], MASK x (K-1)]``
at RoPE positions ``anchor_pos_j ..``, and predicts the next ``K-1`` response
tokens.  Query rows see the clean context strictly before their anchor plus
their own block (bidirectionally); rows of empty blocks see only themselves.

Keys of the student forward are ``[clean context (Lc slots) ; draft blocks]``,
so every query row is a ``(lim, lo, hi)`` descriptor of the attention kernels
and of :func:`~d3d_b200.engine.layout.rows_to_dense`.
"""
from __future__ import annotations

import random
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch


@dataclass
class Example:
    prompt_ids: List[int]
    response_ids: List[int]


@dataclass
class PackedTrainBatch:
    clean_ids: torch.Tensor          # [B, Lc] (right-padded with 0)
    clean_lens: torch.Tensor         # [B]
    draft_ids: torch.Tensor          # [B, Q]
    positions: torch.Tensor          # [B, Q]
    rows: torch.Tensor               # [B, Q, 3] over keys [0, Lc + Q)
    active: torch.Tensor             # [B, Q] bool: row has a target
    offsets: torch.Tensor            # [B, Q] offset inside the block (0 = anchor)
    target_ids: torch.Tensor         # [B, Q] next-token targets (0 where inactive)
    teacher_pos: torch.Tensor        # [B, Q] clean position whose AR logits predict the target
    anchor_positions: torch.Tensor   # [B, NB]
    block_keep: torch.Tensor         # [B, NB] bool
    block_size: int

    @property
    def num_active(self) -> int:
        return int(self.active.sum())

    def to(self, device) -> "PackedTrainBatch":
        kw = {k: (v.to(device, non_blocking=True) if isinstance(v, torch.Tensor) else v)
              for k, v in self.__dict__.items()}
        return PackedTrainBatch(**kw)

    def pin(self) -> "PackedTrainBatch":
        """Page-locked host copy (asynchronous host-to-device transfer)."""
        kw = {k: (v.pin_memory() if isinstance(v, torch.Tensor) else v) for k, v in self.__dict__.items()}
        return PackedTrainBatch(**kw)


def select_anchor_starts(response_len: int, max_anchors: int, rng: random.Random,
                         full_block: int = 0) -> List[int]:
    """Response offsets of the anchors: every offset that leaves at least one
    target token (or, with ``full_block=K``, a whole block of K-1 targets),
    ``max_anchors`` of them drawn from ``rng`` when there are more."""
    last = int(response_len) - (full_block - 1 if full_block else 1)
    starts = list(range(0, max(last, 0)))
    if max_anchors > 0 and len(starts) > max_anchors:
        starts = sorted(rng.sample(starts, max_anchors))
    return starts


def build_packed_block_batch(examples: Sequence[Example], *, block_size: int, mask_token_id: int,
                             max_anchors: int, rng: Optional[random.Random] = None, full_blocks: bool = False
                             ) -> Optional[PackedTrainBatch]:
    if max_anchors <= 0:
        raise ValueError("max_anchors must be > 0")
    rng = rng or random.Random(0)
    prepared = []
    for ex in examples:
        starts = select_anchor_starts(len(ex.response_ids), max_anchors, rng, block_size if full_blocks else 0)
        if starts:
            prepared.append((list(ex.prompt_ids), list(ex.response_ids), starts))
    if not prepared:
        return None
    K = int(block_size)
    B = len(prepared)
    Lc = max(len(p) + len(r) for p, r, _ in prepared)
    NB = max(len(s) for _, _, s in prepared)
    Q = NB * K
    clean = torch.zeros(B, Lc, dtype=torch.long)
    clean_lens = torch.zeros(B, dtype=torch.long)
    ids = torch.full((B, Q), int(mask_token_id), dtype=torch.long)
    pos = torch.zeros(B, Q, dtype=torch.long)
    rows = torch.zeros(B, Q, 3, dtype=torch.int32)
    active = torch.zeros(B, Q, dtype=torch.bool)
    offsets = torch.arange(Q).remainder(K).repeat(B, 1)
    tgt = torch.zeros(B, Q, dtype=torch.long)
    tpos = torch.zeros(B, Q, dtype=torch.long)
    anchors = torch.zeros(B, NB, dtype=torch.long)
    keep = torch.zeros(B, NB, dtype=torch.bool)
    for b, (p, r, starts) in enumerate(prepared):
        seq = p + r
        clean[b, : len(seq)] = torch.tensor(seq)
        clean_lens[b] = len(seq)
        # default: every row sees only itself (padding / empty blocks)
        q = torch.arange(Q, dtype=torch.int32)
        rows[b, :, 1] = Lc + q
        rows[b, :, 2] = Lc + q + 1
        for j, s in enumerate(starts):
            a_pos = len(p) + s
            n_act = min(K - 1, len(r) - s - 1)
            if n_act <= 0:
                continue
            q0 = j * K
            anchors[b, j] = a_pos
            keep[b, j] = True
            ids[b, q0] = r[s]
            pos[b, q0:q0 + K] = torch.arange(a_pos, a_pos + K)
            rows[b, q0:q0 + K, 0] = a_pos                 # clean keys strictly before the anchor
            rows[b, q0:q0 + K, 1] = Lc + q0               # own block, bidirectional
            rows[b, q0:q0 + K, 2] = Lc + q0 + K
            for o in range(1, n_act + 1):
                active[b, q0 + o] = True
                tgt[b, q0 + o] = r[s + o]
                tpos[b, q0 + o] = a_pos + o - 1
    if not bool(active.any()):
        return None
    return PackedTrainBatch(clean, clean_lens, ids, pos, rows, active, offsets, tgt, tpos, anchors, keep, K)


def synthetic_examples(n: int, seq_len: int, prompt_frac: float, vocab: int, rng: random.Random) -> List[Example]:
    """Random-token sequences split into a prompt and a response part."""
    out = []
    for _ in range(n):
        toks = [rng.randrange(0, vocab) for _ in range(seq_len)]
        cut = max(1, int(seq_len * prompt_frac))
        out.append(Example(toks[:cut], toks[cut:]))
    return out
