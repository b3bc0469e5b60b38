"""Choose the layer(s) to delete (reference: ``pruning/select_layer.py``).

Ranks single-layer deletions by mean accept length (then token accuracy,
then the smaller drop), with a bootstrap confidence interval of the mean,
and writes ``selection.json`` with the provenance that :mod:`.prune`
validates.  ``drop > 1`` removes layers greedily one at a time, re-scoring
the pruned model after each removal.  Under ``torch.distributed.run`` the
examples are scored data-parallel, one process per device.
"""
from __future__ import annotations

import json
import random
from pathlib import Path
from typing import Dict, List, Optional, Sequence

from .modeling import EvalExample, _mean, score_single_layer_removals


def gather_in_order(local: list, world: int, rank: int) -> list:
    """Rows scored for examples ``rank::world`` on every rank, gathered and
    put back in example order (rank-major interleave), so a result does not
    depend on how many processes shared the work.  Single process: identity."""
    import torch.distributed as dist
    if world <= 1 or not dist.is_initialized():
        return list(local)
    parts = [None] * world
    dist.all_gather_object(parts, list(local))
    out, n = [], sum(len(p) for p in parts)
    for i in range(n):
        out.append(parts[i % world][i // world])
    return out


def evaluate_removals_parallel(model, examples: Sequence[EvalExample], block_size: int, mode: str = "causal"):
    """Data-parallel scoring of every single-layer deletion (one process per
    device; the reference farms example shards out to a process pool,
    ``pruning/select_layer.py:191-216``): rank r scores examples r::world,
    rows are gathered in example order.  Returns per-example rows
    ``(full, {j: cand_j})`` identical to a single-process run."""
    import torch.distributed as dist
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    full, cands = score_single_layer_removals(model, list(examples)[rank::world], block_size, mode)
    L = model.cfg.num_hidden_layers
    return (gather_in_order(full, world, rank),
            {j: gather_in_order(cands[j], world, rank) for j in range(L)})


def bootstrap_ci(values: Sequence[float], n: int = 200, seed: int = 0, q=(0.025, 0.975)):
    rng = random.Random(seed)
    if not values:
        return (0.0, 0.0)
    means = sorted(sum(rng.choice(values) for _ in values) / len(values) for _ in range(n))
    return means[int(q[0] * (n - 1))], means[int(q[1] * (n - 1))]


def rank_candidates(scores: Dict[int, tuple]) -> List[int]:
    return sorted(scores, key=lambda j: (-scores[j][0], -scores[j][1], j))


def select_layers(model, examples: Sequence[EvalExample], block_size: int, drop: int = 1,
                  mode: str = "causal") -> dict:
    """Greedy progressive selection; returns the original indices removed."""
    from .prune import drop_layers_inplace
    retained = list(range(model.cfg.num_hidden_layers))
    history = []
    for _ in range(drop):
        full_rows, cand_rows = evaluate_removals_parallel(model, examples, block_size, mode)
        base = _mean(full_rows)
        cand = {j: _mean(rs) for j, rs in cand_rows.items()}
        best = rank_candidates(cand)[0]
        ci = bootstrap_ci([r[0] for r in cand_rows[best]])
        history.append({"parent_depth": len(retained), "removed_compact_layer": best,
                        "removed_original_layer": retained[best], "parent_accept_length": base[0],
                        "child_accept_length": cand[best][0], "child_token_accuracy": cand[best][1],
                        "child_accept_length_ci95": list(ci), "samples": len(full_rows),
                        "candidates": {str(k): v for k, v in cand.items()}})
        drop_layers_inplace(model, [best])
        del retained[best]
    return {"retained_original_layers": retained, "history": history}


def write_selection(path: Path, parent_checkpoint: str, parent_depth: int, removed: int,
                    retained_original: Sequence[int], mask_token_id: Optional[int], metrics: dict) -> None:
    data = {"parent_checkpoint": str(parent_checkpoint), "parent_depth": parent_depth,
            "child_depth": parent_depth - 1, "removed_compact_layer": int(removed),
            "child_retained_original_layers": [int(x) for x in retained_original],
            "mask_token_id": mask_token_id, "metrics": metrics}
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + ".tmp")
    tmp.write_text(json.dumps(data, indent=2))
    tmp.replace(path)
