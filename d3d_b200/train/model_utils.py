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


class FastTeacher:
    """The frozen teacher's forward on the framework's sm_100a inference
    kernels (tcgen05 GEMMs, tcgen05 attention, fused norms) instead of the
    PyTorch module: one batched causal forward over the clean sequences,
    returning every position's final-norm hidden state.  The module's
    decoder weights are packed once into the kernel layout; the LM-head
    weight stays a plain ``[V, H]`` tensor for the fused LM-head loss.
    Sequence lengths are padded up to a multiple of ``pad`` so a run with
    varying lengths reuses a few buffer shapes."""

    def __init__(self, module: Qwen3LM, max_batch: int, max_len: int, device, pad: int = 256):
        from ..engine.fast import FastTarget
        from ..models.fast import FastWeights
        self.cfg = module.cfg
        self.pad = pad
        self.lm_weight = module.lm_weight.detach()
        self.max_len = (max_len + pad - 1) // pad * pad
        w = FastWeights.from_module(module, device)
        pages = max_batch * (self.max_len + 64 + 16) // 16 + 8
        self.be = FastTarget(w, pages=pages, max_seqs=max_batch, max_context=self.max_len, device=device,
                             use_graphs=False)

    @torch.no_grad()
    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        B, L = ids.shape
        Lp = (L + self.pad - 1) // self.pad * self.pad
        if Lp > self.max_len:
            raise ValueError(f"teacher sequence of {L} tokens exceeds max_len {self.max_len}")
        x = ids
        if Lp != L:
            x = torch.zeros(B, Lp, dtype=ids.dtype, device=ids.device)
            x[:, :L] = ids
        return self.be.hidden_states(x)[:, :L]

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        return torch.nn.functional.linear(h, self.lm_weight)


@torch.no_grad()
def teacher_hidden(target, batch: PackedTrainBatch) -> torch.Tensor:
    """[B, Q, Ht] final hidden of the target (a ``Qwen3LM`` or a
    :class:`FastTeacher`) at ``batch.teacher_pos``."""
    h = target(batch.clean_ids)
    idx = batch.teacher_pos.clamp(max=h.shape[1] - 1)
    return torch.gather(h, 1, idx[..., None].expand(-1, -1, h.shape[-1]))
