"""Scoring of single-layer deletions by drafted accept length
(reference: ``pruning/modeling.py:58-118``, ``pruning/common.py:122-131``).

An evaluation example is a clean prefix followed by one block
``[anchor, MASK x (K-1)]`` and the K-1 true continuation tokens.  The hard
accept length is ``1 + leading matches`` of the drafted block, the number of
tokens one verify would commit.  One full pass records the input of every
layer; deleting layer j reuses the input of layer j and runs only layers
j+1..L-1, so all L candidates cost about L^2/2 layer evaluations.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple

import torch

from ..engine.layout import block_causal_rows, causal_rows, full_rows, rows_to_dense
from ..models.qwen3 import Qwen3LM, rope_cos_sin


@dataclass
class EvalExample:
    prefix: List[int]
    anchor: int
    continuation: List[int]     # K-1 true next tokens


def hard_accept_length(pred: torch.Tensor, target: torch.Tensor) -> Tuple[int, float]:
    m = pred.eq(target)
    return int(m.long().cumprod(0).sum()) + 1, float(m.float().mean())


def _inputs(model: Qwen3LM, ex: EvalExample, block_size: int, mode: str):
    dev = next(model.parameters()).device
    mask_id = int(model.cfg.mask_token_id)
    n = len(ex.prefix)
    ids = torch.tensor([ex.prefix + [ex.anchor] + [mask_id] * (block_size - 1)], device=dev)
    rows = torch.cat([causal_rows(0, n, dev) if mode == "causal" else block_causal_rows(0, n, block_size, dev),
                      full_rows(n + block_size, block_size, dev)])
    mask = rows_to_dense(rows, n + block_size)[None]
    pos = torch.arange(n + block_size, device=dev)[None]
    return ids, pos, mask


def _mean(rs):
    return (sum(r[0] for r in rs) / len(rs), sum(r[1] for r in rs) / len(rs))


@torch.no_grad()
def evaluate_single_layer_removals(model: Qwen3LM, examples: Sequence[EvalExample], block_size: int,
                                   mode: str = "causal") -> Tuple[Tuple[float, float], Dict[int, Tuple[float, float]]]:
    """Mean (accept length, token accuracy) of the full model and of every
    single-layer deletion."""
    full, cands = score_single_layer_removals(model, examples, block_size, mode)
    return _mean(full), {j: _mean(rs) for j, rs in cands.items()}


@torch.no_grad()
def score_single_layer_removals(model: Qwen3LM, examples: Sequence[EvalExample], block_size: int,
                                mode: str = "causal"):
    """Per-example (accept length, token accuracy) of the full model and of
    every single-layer deletion: ``(full[i], {j: cand_j[i]})`` in example order."""
    L = model.cfg.num_hidden_layers
    full: List[Tuple[int, float]] = []
    cands: Dict[int, List[Tuple[int, float]]] = {j: [] for j in range(L)}
    for ex in examples:
        ids, pos, mask = _inputs(model, ex, block_size, mode)
        target = torch.tensor(ex.continuation, device=ids.device)
        x = model.embed(ids)
        cos, sin = rope_cos_sin(pos, model.cfg.head_dim, model.cfg.rope_theta, x.dtype)
        inputs = []
        for layer in model.model.layers:
            inputs.append(x)
            x = layer(x, cos, sin, mask, None, False)

        def score(h):
            lg = model.logits(model.model.norm(h)[:, -block_size:])[0, 1:]
            return hard_accept_length(lg.argmax(-1), target)

        full.append(score(x))
        for j in range(L):
            h = inputs[j]
            for layer in model.model.layers[j + 1:]:
                h = layer(h, cos, sin, mask, None, False)
            cands[j].append(score(h))
    return full, cands


def examples_from_sequences(seqs: Sequence[Sequence[int]], block_size: int, per_seq: int,
                            rng) -> List[EvalExample]:
    out = []
    for s in seqs:
        s = list(s)
        for _ in range(per_seq):
            if len(s) < block_size + 2:
                break
            a = rng.randrange(1, len(s) - block_size + 1)
            out.append(EvalExample(s[:a], s[a], s[a + 1:a + block_size]))
    return out
