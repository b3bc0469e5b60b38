"""Choose the layer(s) to delete (reference: ``pruning/select_layer.py``).

Ranks single-layer deletions by mean accept length (then token accuracy,
then the smaller drop), with a bootstrap confidence interval of the mean,
and writes ``selection.json`` with the provenance that :mod:`.prune`
validates.  ``drop > 1`` removes layers greedily one at a time, re-scoring
the pruned model after each removal.
"""
from __future__ import annotations

import json
import random
from pathlib import Path
from typing import Dict, List, Optional, Sequence

from .modeling import EvalExample, evaluate_single_layer_removals


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
        base, cand = evaluate_single_layer_removals(model, examples, block_size, mode)
        best = rank_candidates(cand)[0]
        history.append({"parent_depth": len(retained), "removed_compact_layer": best,
                        "removed_original_layer": retained[best], "parent_accept_length": base[0],
                        "child_accept_length": cand[best][0], "child_token_accuracy": cand[best][1],
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
