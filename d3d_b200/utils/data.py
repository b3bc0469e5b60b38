"""Prompt sources.

Prompts come from a local JSONL file (one ``{"prompt": ...}`` or
``{"input_ids": [...]}`` object per line), the synthetic seeded random-token
generator used by every benchmark configuration, or an evaluation set by
name (``utils/benchsets.py``: the reference's seven sets, read from a local
cache, with answer scoring).
"""
from __future__ import annotations

import json
import random
from pathlib import Path
from typing import List, Optional

SPECIAL_START = 151643   # Qwen3 special tokens start here


def synthetic_prompts(n: int, lo: int, hi: int, seed: int, vocab: int = SPECIAL_START) -> List[List[int]]:
    rng = random.Random(seed)
    return [[rng.randrange(0, vocab) for _ in range(rng.randint(lo, hi))] for _ in range(n)]


def load_jsonl_prompts(path: str, tokenizer=None, max_samples: Optional[int] = None) -> List[List[int]]:
    out: List[List[int]] = []
    for line in Path(path).read_text().splitlines():
        if not line.strip():
            continue
        row = json.loads(line)
        if "input_ids" in row:
            out.append([int(t) for t in row["input_ids"]])
        elif tokenizer is not None:
            out.append(tokenizer.encode(row.get("prompt") or row.get("question") or row["text"]))
        else:
            raise ValueError("text prompts need a tokenizer")
        if max_samples and len(out) >= max_samples:
            break
    return out
