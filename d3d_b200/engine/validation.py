"""Drafter validation: the engine's drafter against the PyTorch module on
the same inputs (reference: ``serving/validation.py:8-55``).

One prompt is prefilled on the engine's target; the engine's drafter and a
:class:`~d3d_b200.engine.backends.TorchDraft` of the oracle module each
prefill it and draft the recovery block from the target's anchor (the
recovery blocks must be equal).  Then both run the packed all-outcome
forward from the SAME pending block and top tokens -- the engine's -- so the
packed forward is compared in isolation: the outcome keys must be equal and
the share of equal drafted tokens is reported.  bf16 kernels may flip near
ties, so the check is an agreement threshold, as in the reference (0.99).
"""
from __future__ import annotations

from typing import Sequence

import torch

from .backends import SeqState, TorchDraft
from .spec import SpecDecoder


@torch.inference_mode()
def validate_draft(decoder: SpecDecoder, oracle, prompt: Sequence[int], *, min_agreement: float = 0.99,
                   index: int = 1 << 30) -> dict:
    """Compare ``decoder``'s drafter with ``oracle`` (a ``Qwen3LM``) on
    ``prompt``; raises ``RuntimeError`` when the recovery blocks differ or the
    packed-token agreement is below ``min_agreement``."""
    cfg = decoder.cfg
    k = cfg.block_size
    ref_draft = TorchDraft(oracle)
    ref = SpecDecoder(decoder.t, ref_draft, cfg)
    ours_s = SeqState(index=index, prompt=list(prompt), prefix=len(prompt))
    ref_s = SeqState(index=index + 1, prompt=list(prompt), prefix=len(prompt))
    anchors, hidden = decoder.t.prefill([ours_s])
    for s in (ours_s, ref_s):
        s.anchor = int(anchors[0])
        s.cond = None if hidden is None or not cfg.use_cond else hidden[0]
    try:
        decoder.d.prefill([ours_s], cfg.attention_mask_mode, k)
        ref_draft.prefill([ref_s], cfg.attention_mask_mode, k)
        decoder.recover([ours_s])
        ref.recover([ref_s])
        recovery_equal = ours_s.current.tolist() == ref_s.current.tolist()
        # same pending block and top tokens on both sides: the packed forward alone
        ref_s.current = ours_s.current.clone()
        ref_s.top = None if ours_s.top is None else ours_s.top.clone()
        ours = decoder.predict([ours_s])[ours_s.index]
        exp = ref.predict([ref_s])[ref_s.index]
        keys_ours, keys_ref = list(ours.lay.keys), list(exp.lay.keys)
        if set(keys_ours) != set(keys_ref):
            raise RuntimeError("packed outcome keys differ between the engine's drafter and the oracle")
        equal = total = 0
        diffs = []
        for key in keys_ref:
            x = ours.get(key)[0].tolist()
            y = exp.get(key)[0].tolist()
            equal += sum(a == b for a, b in zip(x, y))
            total += len(y)
            if x != y:
                diffs.append({"key": [key[0], key[1]], "actual": x, "expected": y})
    finally:
        decoder.t.release(ours_s)
        decoder.d.release(ours_s)
        ref_draft.release(ref_s)
    result = {"recovery_equal": recovery_equal, "candidate_keys": len(keys_ref), "packed_tokens_equal": equal,
              "packed_tokens_total": total, "agreement": equal / total if total else 1.0, "differences": diffs}
    if not recovery_equal or result["agreement"] < min_agreement:
        raise RuntimeError(f"drafter differs materially from the oracle module: recovery_equal={recovery_equal}, "
                           f"agreement={result['agreement']:.4f}")
    return result
