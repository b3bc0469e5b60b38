"""Prompt formatting and stop-token helpers (reference: ``common/text.py``)."""
from __future__ import annotations

from typing import Any, Iterable, List, Optional, Sequence


def apply_chat_template(tokenizer: Any, messages: List[dict], enable_thinking: bool) -> str:
    try:
        return tokenizer.apply_chat_template(messages, tokenize=False, add_generation_prompt=True,
                                             enable_thinking=enable_thinking)
    except TypeError:
        return tokenizer.apply_chat_template(messages, tokenize=False, add_generation_prompt=True)


def eos_token_ids(tokenizer: Any, explicit: Optional[Sequence[int]] = None) -> List[int]:
    vals: List[int] = []
    eos = getattr(tokenizer, "eos_token_id", None) if tokenizer is not None else None
    if isinstance(eos, int):
        vals.append(eos)
    elif isinstance(eos, (list, tuple)):
        vals.extend(int(x) for x in eos)
    extra = getattr(tokenizer, "eos_token_ids", None) if tokenizer is not None else None
    if isinstance(extra, (list, tuple)):
        vals.extend(int(x) for x in extra)
    if explicit:
        vals.extend(int(x) for x in explicit)
    out: List[int] = []
    for v in vals:
        if v not in out:
            out.append(v)
    return out


def trim_at_stop(tokens: Sequence[int], stop_ids: Optional[Iterable[int]]) -> List[int]:
    """Cut a generated token list after the first stop token (kept)."""
    toks = [int(t) for t in tokens]
    if not stop_ids:
        return toks
    stops = set(int(s) for s in stop_ids)
    for i, t in enumerate(toks):
        if t in stops:
            return toks[: i + 1]
    return toks


def contains_stop(tokens: Sequence[int], stop_ids: Optional[Iterable[int]]) -> bool:
    if not stop_ids:
        return False
    stops = set(int(s) for s in stop_ids)
    return any(int(t) in stops for t in tokens)
