"""Drafter validation: the engine's drafter against the PyTorch module on
the same inputs (reference: ``serving/validation.py:8-55``).

One prompt is prefilled on the engine's target; the engine's drafter and a
:class:`~d3d_b200.engine.backends.TorchDraft` of the oracle module each
prefill it and draft the recovery block from the target's anchor (the
recovery blocks must be equal).  Then both run the packed all-outcome
forward from the SAME pending block and top tokens -- the engine's -- so the
packed forward is compared in isolation: the outcome keys must be equal and
the share of equal drafted tokens is reported.  bf16 kernels may flip near
ties, so the check is an agreement threshold, as in the reference (0.99),
with differences that are the oracle's own near-ties counted as agreeing.
"""
from __future__ import annotations

from typing import Sequence

import torch

from .backends import SeqState, TorchDraft
from .spec import SpecDecoder


def _ties(ours, ref, logits, tol: float):
    """Positions (after the anchor) where ``ours`` differs from the oracle's
    argmax ``ref``, those whose logit regret under the oracle (argmax logit
    minus the logit of our token) is at most ``tol``, and every regret."""
    diff = [j for j in range(1, len(ref)) if ours[j] != ref[j]]
    regret = {j: float(logits[j, ref[j]] - logits[j, ours[j]]) for j in diff}
    return diff, [j for j in diff if regret[j] <= tol], regret


@torch.inference_mode()
def validate_draft(decoder: SpecDecoder, oracle, prompt: Sequence[int], *, min_agreement: float = 0.99,
                   tie_tolerance: float = 0.05, index: int = 1 << 30) -> dict:
    """Compare ``decoder``'s drafter with ``oracle`` (a ``Qwen3LM``) on
    ``prompt``; raises ``RuntimeError`` when the recovery blocks differ or the
    packed-token agreement is below ``min_agreement``.  A differing token
    whose logit under the oracle is within ``tie_tolerance`` of the oracle's
    argmax logit is a near-tie (bf16 rounding can flip it; the reference's AR
    baseline makes the same distinction with a teacher-forced logit regret):
    near-ties are reported and counted as agreement."""
    cfg = decoder.cfg
    k = cfg.block_size
    ref_draft = TorchDraft(oracle)
    ref_draft.record_logits = True
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
        rec = ref_draft.last
        recovery_equal = ours_s.current.tolist() == ref_s.current.tolist()
        rdiff, rties, rregret = _ties(ours_s.current.tolist(), ref_s.current.tolist(), rec["logits"][0],
                                      tie_tolerance)
        # same pending block and top tokens on both sides: the packed forward alone
        ref_s.current = ours_s.current.clone()
        ref_s.top = None if ours_s.top is None else ours_s.top.clone()
        ours = decoder.predict([ours_s])[ours_s.index]
        exp = ref.predict([ref_s])[ref_s.index]
        keys_ours, keys_ref = list(ours.lay.keys), list(exp.lay.keys)
        if set(keys_ours) != set(keys_ref):
            raise RuntimeError("packed outcome keys differ between the engine's drafter and the oracle")
        equal = total = near = 0
        diffs = []
        out = exp.out
        for key in keys_ref:
            x = ours.get(key)[0].tolist()
            y = exp.get(key)[0].tolist()
            equal += sum(a == b for a, b in zip(x, y))
            total += len(y)
            if x != y:
                sl = exp.lay.segment(exp.index[key])
                _, ties, regret = _ties(x, y, out["logits"][exp.i, sl], tie_tolerance)
                near += len(ties)
                diffs.append({"key": [key[0], key[1]], "actual": x, "expected": y, "near_ties": ties,
                              "max_logit_regret": max(regret.values())})
    finally:
        decoder.t.release(ours_s)
        decoder.d.release(ours_s)
        ref_draft.release(ref_s)
    result = {"recovery_equal": recovery_equal, "recovery_near_ties": rties,
              "recovery_max_logit_regret": max(rregret.values()) if rregret else 0.0, "candidate_keys": len(keys_ref),
              "packed_tokens_equal": equal, "packed_tokens_total": total,
              "agreement": equal / total if total else 1.0, "packed_near_ties": near,
              "agreement_up_to_near_ties": (equal + near) / total if total else 1.0, "tie_tolerance": tie_tolerance,
              "differences": diffs}
    recovery_ok = recovery_equal or len(rties) == len(rdiff)
    if not recovery_ok or result["agreement_up_to_near_ties"] < min_agreement:
        raise RuntimeError(f"drafter differs materially from the oracle module: recovery_equal={recovery_equal} "
                           f"({len(rdiff) - len(rties)} non-tie differences, max logit regret "
                           f"{result['recovery_max_logit_regret']:.4f}), agreement={result['agreement']:.4f}, "
                           f"up to near-ties={result['agreement_up_to_near_ties']:.4f}")
    return result
