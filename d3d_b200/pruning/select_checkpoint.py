"""Pick the best recovery checkpoint by drafted accept length
(reference: ``pruning/select_checkpoint.py:84-158``): highest mean accept
length, then token accuracy, then the earliest step."""
from __future__ import annotations

import json
import re
from pathlib import Path
from typing import List, Sequence

from ..checkpoint import load_model
from .modeling import EvalExample


def checkpoint_step(path: Path) -> int:
    m = re.search(r"(\d+)$", Path(path).name)
    return int(m.group(1)) if m else 0


def score_checkpoint(path, examples: Sequence[EvalExample], block_size: int, device="cpu") -> dict:
    m = load_model(path, device=device).eval()
    (acc, tok), _ = _score_full(m, examples, block_size)
    return {"checkpoint": str(path), "mean_accept_length": acc, "mean_draft_token_accuracy": tok,
            "step": checkpoint_step(Path(path))}


def _score_full(model, examples, block_size):
    """Mean (accept length, token accuracy) over ``examples``; under
    ``torch.distributed`` each rank scores examples rank::world and the rows
    are gathered in example order (``pruning/select_checkpoint.py:98-120``)."""
    import torch
    import torch.distributed as dist
    from .modeling import _inputs, hard_accept_length
    from .select_layer import gather_in_order
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    rs = []
    with torch.no_grad():
        for ex in list(examples)[rank::world]:
            ids, pos, mask = _inputs(model, ex, block_size, "causal")
            h = model(ids, pos, mask=mask)
            lg = model.logits(h[:, -block_size:])[0, 1:]
            rs.append(hard_accept_length(lg.argmax(-1), torch.tensor(ex.continuation, device=ids.device)))
    rs = gather_in_order(rs, world, rank)
    return (sum(r[0] for r in rs) / len(rs), sum(r[1] for r in rs) / len(rs)), None


def choose(paths: List[str], examples: Sequence[EvalExample], block_size: int, device="cpu") -> dict:
    rows = [score_checkpoint(p, examples, block_size, device) for p in paths]
    rows.sort(key=lambda r: (-r["mean_accept_length"], -r["mean_draft_token_accuracy"], r["step"]))
    return {"best": rows[0], "ranking": rows}
