"""Recovery training of a pruned drafter (reference: ``pruning/train_recovery.py``).

The frozen parent drafter is the teacher.  Per step, on packed anchor+MASK
blocks (:mod:`d3d_b200.train.blocks`):

``loss = 1.0 * AR + 1.0 * CE + 1.0 * corrected KL + 10.0 * boundary MSE``

(the reference's fixed coefficients, ``train_recovery.py:33-36``): AR is the
student's next-token CE on the clean sequence; CE and corrected KL are on the
block rows against the data tokens and the teacher's block logits; the
boundary term matches the student's hidden state entering the layer that
took the deleted layer's place to the teacher's output of the deleted layer.
Embeddings and the LM head stay frozen, as in the reference.
"""
from __future__ import annotations

import random
from typing import List, Sequence

import torch

from ..engine.layout import rows_to_dense
from ..models.qwen3 import Qwen3LM
from ..train.blocks import Example, build_packed_block_batch
from ..train.model_utils import clean_prefill
from ..train.optim import ShardedAdamW
from .losses import boundary_hidden_mse, corrected_kl, masked_mean, target_ce

LAMBDA_AR, LAMBDA_CE, LAMBDA_KL, LAMBDA_H = 1.0, 1.0, 1.0, 10.0


def _block_forward(model: Qwen3LM, batch, cache, hidden: bool = False):
    lc, q = batch.clean_ids.shape[1], batch.draft_ids.shape[1]
    mask = rows_to_dense(batch.rows, lc + q)
    return model(batch.draft_ids, batch.positions, mask=mask, cache=cache, store_kv=False,
                 output_hidden_states=hidden)


def recovery_step(student: Qwen3LM, teacher: Qwen3LM, removed_original: int, retained_original: Sequence[int],
                  examples: List[Example], opt: ShardedAdamW, *, block_size: int, anchors: int,
                  rng: random.Random, grad_clip: float = 1.0, z3=None) -> dict:
    """One recovery step; ``z3``: the student's sharded decoder layers
    (``parallel.zero3``), stepped with the same clip factor as ``opt``."""
    mask_id = int(student.cfg.mask_token_id)
    batch = build_packed_block_batch(examples, block_size=block_size, mask_token_id=mask_id,
                                     max_anchors=anchors, rng=rng)
    dev = next(student.parameters()).device
    batch = batch.to(dev)
    act = batch.active
    w = act.float()
    with torch.no_grad():
        tcache = clean_prefill(teacher, batch)
        th, ths = _block_forward(teacher, batch, tcache, hidden=True)
        tlog = teacher.logits(th)[act]
    scache = clean_prefill(student, batch)
    sh, shs = _block_forward(student, batch, scache, hidden=True)
    slog = student.logits(sh)[act]
    tgt = batch.target_ids[act]
    ce = masked_mean(target_ce(slog, tgt), w[act], distributed=True)
    kl = masked_mean(corrected_kl(slog, tlog, tgt), w[act], distributed=True)
    # boundary: student input of compact layer b (the one now after the gap)
    # vs teacher output of the deleted original layer
    b = sum(1 for r in retained_original if r < removed_original)
    hb = boundary_hidden_mse(shs[b][act], ths[removed_original + 1][act])
    hmse = masked_mean(hb, w[act], distributed=True)
    # clean AR loss on the prompt+response sequence
    logits_ar = student.logits(student(batch.clean_ids))[:, :-1]
    ar_t = batch.clean_ids[:, 1:]
    ar_w = (torch.arange(batch.clean_ids.shape[1] - 1, device=dev)[None] < (batch.clean_lens[:, None] - 1)).float()
    ar = masked_mean(target_ce(logits_ar.reshape(-1, logits_ar.shape[-1]), ar_t.reshape(-1)), ar_w.reshape(-1),
                     distributed=True)
    loss = LAMBDA_AR * ar + LAMBDA_CE * ce + LAMBDA_KL * kl + LAMBDA_H * hmse
    loss.backward()
    from ..train.trainer import _opt_step
    norm = _opt_step(opt, z3, grad_clip, None)
    opt.zero_grad()
    return {"loss": float(loss.detach()), "ar": float(ar.detach()), "ce": float(ce.detach()),
            "kl": float(kl.detach()), "hidden_mse": float(hmse.detach()),
            "grad_norm": norm}


def make_student(parent: Qwen3LM, removed_compact: int) -> Qwen3LM:
    import copy
    from .prune import drop_layers_inplace
    s = copy.deepcopy(parent)
    drop_layers_inplace(s, [removed_compact])
    for p in s.parameters():
        p.requires_grad_(True)
    s.train()
    s.model.embed_tokens.weight.requires_grad_(False)
    if not s.cfg.tie_word_embeddings:
        s.lm_head.weight.requires_grad_(False)
    return s
