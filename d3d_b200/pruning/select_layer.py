"""Choose the layer(s) to delete (reference: ``pruning/select_layer.py``).

Ranks single-layer deletions by mean accept length (then token accuracy,
then the lower original layer), with a bootstrap 95% interval of the
relative acceptance damage, and writes ``selection.json`` with the
provenance that :mod:`.prune` validates (:func:`run_select`, the stage).
:func:`select_layers` removes several layers greedily in memory, re-scoring
after each removal.  Examples are scored one process per device, or
data-parallel under ``torch.distributed.run``.
"""
from __future__ import annotations

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


# ------------------------------------------------------------ the stage
def _score_shard(parent: str, examples: list, device: str, dtype: str, block_size: int,
                 mask_token_id: Optional[int]):
    """One device's share of the deletion scoring (a worker process when
    several devices are given)."""
    import torch
    from ..checkpoint import load_model
    from .modeling import score_single_layer_removals
    dt = {"bf16": torch.bfloat16, "fp32": torch.float32}[dtype]
    m = load_model(parent, device=device, dtype=dt, mask_token_id=mask_token_id).eval()
    return score_single_layer_removals(m, examples, block_size, "causal")


def score_on_devices(parent: str, examples: list, devices: Sequence[str], dtype: str, block_size: int,
                     mask_token_id: Optional[int]):
    """Examples ``i::len(devices)`` on device ``i``, one spawned process per
    device when there are several (``pruning/select_layer.py:191-216``);
    under ``torch.distributed`` every rank scores its own share instead.
    Returns per-example rows in example order."""
    import torch.distributed as dist
    if dist.is_initialized() and dist.get_world_size() > 1:
        world, rank = dist.get_world_size(), dist.get_rank()
        full, cands = _score_shard(parent, examples[rank::world], devices[0], dtype, block_size, mask_token_id)
        return gather_in_order(full, world, rank), {j: gather_in_order(c, world, rank) for j, c in cands.items()}
    n = len(devices)
    if n == 1:
        return _score_shard(parent, examples, devices[0], dtype, block_size, mask_token_id)
    import concurrent.futures
    import multiprocessing
    with concurrent.futures.ProcessPoolExecutor(max_workers=n, mp_context=multiprocessing.get_context("spawn")) as ex:
        futs = [ex.submit(_score_shard, parent, examples[i::n], devices[i], dtype, block_size, mask_token_id)
                for i in range(n)]
        parts = [f.result() for f in futs]
    full = [parts[i % n][0][i // n] for i in range(len(examples))]
    cands = {j: [parts[i % n][1][j][i // n] for i in range(len(examples))] for j in parts[0][1]}
    return full, cands


def damage_table(full_rows, cand_rows, retained_original: Sequence[int], bootstrap_samples: int,
                 bootstrap_seed: int) -> List[dict]:
    """Per deletion candidate: mean accept length and token accuracy, the
    relative acceptance damage ``(parent - candidate) / parent`` and its
    bootstrap 95% interval (examples resampled with replacement, the same
    draw for every candidate), ranked by accept length, then accuracy, then
    the lower original layer index."""
    import numpy as np
    parent = np.array([r[0] for r in full_rows], dtype=np.float64)
    L = len(cand_rows)
    em = np.stack([np.array([r[0] for r in cand_rows[j]], dtype=np.float64) for j in range(L)], 1)
    acc = np.stack([np.array([r[1] for r in cand_rows[j]], dtype=np.float64) for j in range(L)], 1)
    n = len(parent)
    means, acc_means, pm = em.mean(0), acc.mean(0), float(parent.mean())
    damage = (pm - means) / pm
    rng = np.random.default_rng(bootstrap_seed)
    draws = []
    for start in range(0, bootstrap_samples, 256):
        idx = rng.integers(0, n, size=(min(256, bootstrap_samples - start), n))
        pb = parent[idx].mean(1)
        draws.append((pb[:, None] - em[idx].mean(1)) / pb[:, None])
    if draws:
        lo, hi = np.quantile(np.concatenate(draws, 0), [0.025, 0.975], axis=0)
    else:
        lo = hi = damage
    order = sorted(range(L), key=lambda j: (-means[j], -acc_means[j], retained_original[j]))
    rank = {j: i + 1 for i, j in enumerate(order)}
    rows = [{"rank": rank[j], "removed_compact_layer": j, "removed_original_layer": int(retained_original[j]),
             "selected": j == order[0], "parent_mean_accept_length": pm,
             "candidate_mean_accept_length": float(means[j]), "candidate_token_accuracy": float(acc_means[j]),
             "relative_acceptance_damage": float(damage[j]), "damage_ci95_low": float(lo[j]),
             "damage_ci95_high": float(hi[j])} for j in range(L)]
    return sorted(rows, key=lambda r: r["rank"])


def run_select(parent, examples_path, output_dir, *, split: str = "layer_selection", expected_samples: int = 512,
               block_size: int = 16, mask_token_id: Optional[int] = None, devices: Sequence[str] = ("cuda:0",),
               dtype: str = "bf16", bootstrap_samples: int = 10_000, bootstrap_seed: int = 42,
               synthetic_seed: int = 0) -> dict:
    """Score every single-layer deletion of ``parent`` on a tokenized split
    and write ``candidate_metrics.parquet``, ``candidate_summary.csv`` and
    ``selection.json`` into ``output_dir`` (``pruning/select_layer.py:168-264``).
    ``examples_path="synthetic"`` draws ``expected_samples`` random examples."""
    import time
    import pandas as pd
    import torch.distributed as dist
    from ..utils.io import write_json
    from .common import provenance, read_examples, resolve_mask_id
    started = time.time()
    parent = Path(parent).resolve()
    output = Path(output_dir).resolve()
    rank0 = not dist.is_initialized() or dist.get_rank() == 0
    if output.exists():
        raise FileExistsError(f"Refusing to overwrite {output}")
    if block_size < 2:
        raise ValueError("block size must be at least 2")
    if len(devices) != len(set(devices)):
        raise ValueError("--devices must be unique")
    mask_id = resolve_mask_id(parent, mask_token_id)
    if str(examples_path) == "synthetic":
        from ..config import ModelConfig
        cfg = ModelConfig.from_pretrained(parent)
        rng = random.Random(synthetic_seed)
        from .modeling import examples_from_sequences
        vocab = min(cfg.vocab_size, 151643) - 2
        seqs = [[rng.randrange(vocab) for _ in range(64 + block_size)] for _ in range(expected_samples)]
        exs = examples_from_sequences(seqs, block_size, 1, rng)
        ids = [str(i) for i in range(len(exs))]
    else:
        ids, exs = read_examples(examples_path, split, block_size)
    if expected_samples and len(exs) != expected_samples:
        raise ValueError(f"Expected {expected_samples} examples, found {len(exs)}")
    teacher, original_depth, retained = provenance(parent)
    full, cands = score_on_devices(str(parent), exs, list(devices), dtype, block_size, mask_id)
    summary = damage_table(full, cands, retained, bootstrap_samples, bootstrap_seed)
    best = summary[0]
    sel = best["removed_compact_layer"]
    selection = {
        "format_version": 1, "method": "progressive_single_layer_pruning", "parent_checkpoint": str(parent),
        "teacher_checkpoint": str(teacher), "original_depth": original_depth, "parent_depth": len(retained),
        "child_depth": len(retained) - 1, "parent_retained_original_layers": list(retained),
        "removed_compact_layer": sel, "removed_original_layer": int(retained[sel]),
        "child_retained_original_layers": [r for j, r in enumerate(retained) if j != sel],
        "block_size": block_size, "selection_samples": len(exs), "mask_token_id": mask_id,
        "selection_data": str(examples_path if str(examples_path) == "synthetic" else Path(examples_path).resolve()),
        "parent_mean_accept_length": best["parent_mean_accept_length"],
        "child_step0_mean_accept_length": best["candidate_mean_accept_length"],
        "relative_acceptance_damage": best["relative_acceptance_damage"],
        "elapsed_seconds": time.time() - started}
    if rank0:
        output.mkdir(parents=True)
        metrics = pd.DataFrame([{"analysis_id": ids[i], "removed_compact_layer": j,
                                 "parent_emitted_tokens": full[i][0], "candidate_emitted_tokens": cands[j][i][0],
                                 "parent_draft_token_accuracy": full[i][1],
                                 "candidate_draft_token_accuracy": cands[j][i][1]}
                                for j in sorted(cands) for i in range(len(exs))])
        metrics.sort_values(["removed_compact_layer", "analysis_id"]).to_parquet(
            output / "candidate_metrics.parquet", index=False)
        pd.DataFrame(summary).to_csv(output / "candidate_summary.csv", index=False)
        write_json(str(output / "selection.json"), selection)
        print(f"Selected compact layer {sel} (original layer {retained[sel]}) for D{len(retained)} -> "
              f"D{len(retained) - 1}.")
    return {"selection": selection, "summary": summary}
