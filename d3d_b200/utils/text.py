"""Tokenizer-facing helpers: chat prompts, stop ids, prompt/response split.

The reference formats prompts with the tokenizer's chat template (thinking
off) and stops on the tokenizer's EOS ids (``common/text.py:9-63``); its
training loader tokenizes a chat sample as prompt + response and supervises
only the response (``train/dataset.py:71-113``).  Those behaviours are
provided here for any Hugging Face tokenizer object.
"""
from __future__ import annotations

import inspect
from typing import Any, Dict, Iterable, List, Optional, Sequence, Tuple


def _template_accepts(tokenizer: Any, name: str) -> bool:
    fn = getattr(tokenizer, "apply_chat_template", None)
    if fn is None:
        return False
    try:
        params = inspect.signature(fn).parameters
    except (TypeError, ValueError):
        return False
    return name in params or any(p.kind is inspect.Parameter.VAR_KEYWORD for p in params.values())


def chat_prompt(tokenizer: Any, user: str, system: Optional[str] = None, thinking: bool = False) -> str:
    """Render one user turn (optionally after a system turn) with the
    generation prompt appended.  Templates that know ``enable_thinking`` get
    it; older ones are rendered without it."""
    msgs: List[Dict[str, str]] = []
    if system:
        msgs.append({"role": "system", "content": system})
    msgs.append({"role": "user", "content": user})
    kw: Dict[str, Any] = {"tokenize": False, "add_generation_prompt": True}
    if _template_accepts(tokenizer, "enable_thinking"):
        kw["enable_thinking"] = thinking
    return tokenizer.apply_chat_template(msgs, **kw)


def split_chat(tokenizer: Any, messages: Sequence[Dict[str, str]]) -> Tuple[List[int], List[int]]:
    """Token ids of a chat sample split at the last assistant turn: the
    prompt (every turn before it, with the generation prompt) and the
    response (what the template appends for that turn).  Training supervises
    the response only."""
    if not messages or messages[-1].get("role") != "assistant":
        raise ValueError("a chat sample must end with an assistant turn")
    kw: Dict[str, Any] = {"tokenize": True}
    if _template_accepts(tokenizer, "enable_thinking"):
        kw["enable_thinking"] = False
    head = list(tokenizer.apply_chat_template(list(messages[:-1]), add_generation_prompt=True, **kw))
    full = list(tokenizer.apply_chat_template(list(messages), add_generation_prompt=False, **kw))
    if full[: len(head)] != head:
        # templates that rewrite earlier turns: fall back to a plain encode of the reply
        return head, list(tokenizer.encode(messages[-1]["content"], add_special_tokens=False))
    return head, full[len(head):]


def stop_ids(tokenizer: Any = None, extra: Iterable[int] = ()) -> List[int]:
    """Ordered, de-duplicated stop ids: the tokenizer's ``eos_token_id``
    (an int or a list), its ``eos_token_ids`` if any, then ``extra``."""
    found: Dict[int, None] = {}
    for attr in ("eos_token_id", "eos_token_ids"):
        v = getattr(tokenizer, attr, None) if tokenizer is not None else None
        for x in ([v] if isinstance(v, int) else list(v or [])):
            found.setdefault(int(x), None)
    for x in extra:
        found.setdefault(int(x), None)
    return list(found)


def cut_at_stop(tokens: Sequence[int], stops: Optional[Iterable[int]]) -> List[int]:
    """``tokens`` up to and including the first stop id."""
    s = set(int(x) for x in (stops or ()))
    out: List[int] = []
    for t in tokens:
        out.append(int(t))
        if out[-1] in s:
            break
    return out
