"""Forward helpers of distillation training (reference: ``train/model_utils.py``).

* :func:`clean_prefill` — the student's own causal forward over the clean
  sequence, without gradient, kept as KV (``prefill_clean_kv_cache``,
  ``model_utils.py:186-256``);
* :func:`student_hidden` — the packed block forward against that clean KV,
  with the structured row masks, returning final hidden states;
* :func:`teacher_hidden` — the frozen target's final hidden states at the
  positions whose next-token logits supervise each block row
  (``model_utils.py:274-319``).
"""
from __future__ import annotations

import torch

from ..engine.layout import rows_to_dense
from ..models.qwen3 import DenseKVCache, Qwen3LM
from .blocks import PackedTrainBatch


@torch.no_grad()
def clean_prefill(model: Qwen3LM, batch: PackedTrainBatch) -> DenseKVCache:
    was = model.training
    model.eval()
    cache = DenseKVCache(model.cfg.num_hidden_layers)
    model(batch.clean_ids, cache=cache, store_kv=True)
    model.train(was)
    return cache


def student_hidden(model: Qwen3LM, batch: PackedTrainBatch, cache: DenseKVCache) -> torch.Tensor:
    lc = batch.clean_ids.shape[1]
    q = batch.draft_ids.shape[1]
    mask = rows_to_dense(batch.rows, lc + q)
    return model(batch.draft_ids, batch.positions, mask=mask, cache=cache, store_kv=False)


@torch.no_grad()
def teacher_hidden(target: Qwen3LM, batch: PackedTrainBatch) -> torch.Tensor:
    """[B, Q, Ht] final hidden of the target at ``batch.teacher_pos``."""
    h = target(batch.clean_ids)
    idx = batch.teacher_pos.clamp(max=h.shape[1] - 1)
    return torch.gather(h, 1, idx[..., None].expand(-1, -1, h.shape[-1]))
