"""Shared pieces of the pruning stages: tokenized evaluation examples,
layer provenance, mask-token resolution and the seeded row permutation of
the recovery data window (reference: ``pruning/common.py``,
``pruning/data.py:52-110``).

Evaluation examples are rows with ``prefix_ids`` (clean context) and
``target_ids`` (the block: anchor first, then the true continuation), an
optional ``analysis_id`` and an optional ``split`` column, in Parquet, JSONL
or JSON -- the reference's selection-data format, so one file serves both.
"""
from __future__ import annotations

import json
import math
from pathlib import Path
from typing import List, Optional, Tuple

from ..config import ModelConfig
from ..engine.controlled import splitmix64
from .modeling import EvalExample


def read_examples(path, split: Optional[str] = None, block_size: Optional[int] = None
                  ) -> Tuple[List[str], List[EvalExample]]:
    """``(analysis_ids, examples)`` of a tokenized split.  ``target_ids`` is
    cut to ``block_size`` tokens; a shorter block is an error."""
    import pandas as pd
    path = Path(path)
    if path.suffix == ".parquet":
        frame = pd.read_parquet(path)
    elif path.suffix in (".jsonl", ".json"):
        frame = pd.read_json(path, lines=path.suffix == ".jsonl")
    else:
        raise ValueError("evaluation examples must be .parquet, .jsonl or .json")
    if split is not None and "split" in frame.columns:
        frame = frame[frame["split"].astype(str) == split]
    missing = {"prefix_ids", "target_ids"} - set(frame.columns)
    if missing:
        raise ValueError(f"evaluation examples lack columns {sorted(missing)}")
    ids = ([str(x) for x in frame["analysis_id"]] if "analysis_id" in frame.columns
           else [str(i) for i in range(len(frame))])
    if len(set(ids)) != len(ids):
        raise ValueError("analysis_id must be unique")
    out = []
    for aid, prefix, target in zip(ids, frame["prefix_ids"], frame["target_ids"]):
        target = [int(t) for t in target]
        if block_size is not None:
            if len(target) < block_size:
                raise ValueError(f"example {aid} has an incomplete target block")
            target = target[:block_size]
        out.append(EvalExample([int(t) for t in prefix], target[0], target[1:]))
    return ids, out


def checkpoint_depth(checkpoint) -> int:
    return int(json.loads((Path(checkpoint) / "config.json").read_text())["num_hidden_layers"])


def provenance(checkpoint) -> Tuple[Path, int, List[int]]:
    """``(teacher, original_depth, retained_original_layers)`` of a drafter:
    itself, its depth and every layer when it was never pruned; else what
    its ``layer_prune.json`` records, validated."""
    checkpoint = Path(checkpoint).resolve()
    depth = checkpoint_depth(checkpoint)
    meta_path = checkpoint / "layer_prune.json"
    if not meta_path.is_file():
        return checkpoint, depth, list(range(depth))
    meta = json.loads(meta_path.read_text())
    retained = [int(i) for i in meta["retained_original_layers"]]
    if len(retained) != depth or retained != sorted(set(retained)):
        raise ValueError(f"invalid retained-layer mapping in {meta_path}")
    teacher = Path(meta.get("teacher_checkpoint") or meta["parent_checkpoint"]).resolve()
    original = int(meta.get("original_depth", depth + 1))
    if original < depth:
        raise ValueError(f"invalid teacher provenance in {meta_path}")
    return teacher, original, retained


def resolve_mask_id(checkpoint, requested: Optional[int] = None) -> int:
    """The checkpoint's mask token, checked against ``requested``."""
    cfg = ModelConfig.from_pretrained(checkpoint, mask_token_id=requested)
    if cfg.mask_token_id is None:
        raise ValueError(f"{checkpoint} has no mask token")
    return int(cfg.mask_token_id)


# ------------------------------------------------------------ data window
def window_bounds(cursor: int, steps: int, accumulation: int, world: int, multiplier: float,
                  rows: int) -> dict:
    """The recovery run's slice of the (endless, permuted) row sequence:
    enough candidates for ``steps x accumulation x world`` examples after
    filtering, ``multiplier`` times over."""
    if cursor < 0 or steps <= 0 or rows <= 0 or accumulation <= 0 or world <= 0:
        raise ValueError("invalid data window")
    if multiplier < 1:
        raise ValueError("candidate multiplier must be at least one")
    need = steps * accumulation * world
    cand = max(need, math.ceil(need * multiplier))
    return {"cursor_start": cursor, "cursor_end": cursor + cand, "candidate_rows": cand, "required_examples": need,
            "gradient_accumulation_steps": accumulation, "world_size": world, "candidate_multiplier": float(multiplier),
            "dataset_rows": rows}


def permuted_row(position: int, rows: int, seed: int) -> int:
    """Row read at virtual ``position``: each pass over the data (``cycle``)
    is its own affine permutation ``(a * i + b) mod rows`` with ``a`` coprime
    to ``rows``, so any window is a set of distinct rows without a stored
    permutation."""
    if rows == 1:
        return 0
    cycle, i = divmod(int(position), int(rows))
    a = splitmix64(seed * 1_000_003 + 2 * cycle) % rows or 1
    while math.gcd(a, rows) != 1:
        a = a % rows + 1
    b = splitmix64(seed * 1_000_003 + 2 * cycle + 1) % rows
    return (a * i + b) % rows
