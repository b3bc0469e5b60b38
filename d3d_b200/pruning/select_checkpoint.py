"""Pick the best recovery checkpoint by drafted accept length
(reference: ``pruning/select_checkpoint.py:84-158``): highest mean accept
length, then token accuracy, then the earliest step.

The stage (:func:`run_choose`) scores ``step-N`` checkpoints of a recovery
run (or a given list) on a tokenized validation split, one spawned process
per device (checkpoints ``i::n`` on device ``i``), or data-parallel over the
examples under ``torch.distributed.run``, and writes
``checkpoint_metrics.parquet``, ``checkpoint_summary.csv`` and
``selected_checkpoint.json``.
"""
from __future__ import annotations

import re
from pathlib import Path
from typing import List, Optional, Sequence

from ..checkpoint import load_model
from .modeling import EvalExample

_STEP = re.compile(r"step-(\d+)$")


def checkpoint_step(path) -> int:
    """``N`` of a ``step-N`` checkpoint directory, -1 for any other name."""
    m = _STEP.search(Path(path).name)
    return int(m.group(1)) if m else -1


def discover(run_dir=None, checkpoints: Optional[Sequence] = None) -> List[Path]:
    """Complete checkpoints (with a ``config.json``): the given list, or a
    run's ``step-*`` directories in step order."""
    if checkpoints:
        paths = [Path(p).resolve() for p in checkpoints]
    else:
        paths = sorted((p.resolve() for p in Path(run_dir).glob("step-*")), key=checkpoint_step)
    paths = [p for p in paths if (p / "config.json").is_file()]
    if not paths:
        raise ValueError("No complete checkpoints were found")
    return paths


def score_examples(model, examples: Sequence[EvalExample], block_size: int) -> list:
    """Per-example ``(accept length, token accuracy)`` of one drafter; under
    ``torch.distributed`` each rank scores examples rank::world and the rows
    are gathered in example order."""
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
    return gather_in_order(rs, world, rank)


def _score_worker(paths: List[str], examples: list, device: str, block_size: int, mask_token_id: Optional[int],
                  dtype: str) -> dict:
    import torch
    dt = {"bf16": torch.bfloat16, "fp32": torch.float32}[dtype]
    out = {}
    for p in paths:
        m = load_model(p, device=device, dtype=dt, mask_token_id=mask_token_id).eval()
        out[p] = score_examples(m, examples, block_size)
        del m
    return out


def score_checkpoints(paths: Sequence[str], examples: list, block_size: int, devices: Sequence[str] = ("cpu",),
                      mask_token_id: Optional[int] = None, dtype: str = "fp32") -> dict:
    """``{checkpoint: per-example rows}``."""
    import torch.distributed as dist
    paths = [str(p) for p in paths]
    n = len(devices)
    if n == 1 or (dist.is_initialized() and dist.get_world_size() > 1):
        return _score_worker(paths, examples, devices[0], block_size, mask_token_id, dtype)
    import concurrent.futures
    import multiprocessing
    jobs = [(paths[i::n], devices[i]) for i in range(n) if paths[i::n]]
    with concurrent.futures.ProcessPoolExecutor(max_workers=len(jobs),
                                                mp_context=multiprocessing.get_context("spawn")) as ex:
        futs = [ex.submit(_score_worker, ps, examples, d, block_size, mask_token_id, dtype) for ps, d in jobs]
        out = {}
        for f in futs:
            out.update(f.result())
    return {p: out[p] for p in paths}


def rank_checkpoints(rows: dict) -> List[dict]:
    table = []
    for p, rs in rows.items():
        table.append({"checkpoint": p, "mean_accept_length": sum(r[0] for r in rs) / len(rs),
                      "mean_draft_token_accuracy": sum(r[1] for r in rs) / len(rs), "samples": len(rs),
                      "step": checkpoint_step(p)})
    table.sort(key=lambda r: (-r["mean_accept_length"], -r["mean_draft_token_accuracy"], r["step"]))
    for i, r in enumerate(table):
        r["rank"] = i + 1
    return table


def choose(paths: List[str], examples: Sequence[EvalExample], block_size: int, device="cpu") -> dict:
    """In-process ranking of ``paths`` (no files written)."""
    table = rank_checkpoints(score_checkpoints(paths, list(examples), block_size, (str(device),)))
    return {"best": table[0], "ranking": table}


def run_choose(output_dir, examples_path, *, run_dir=None, checkpoints: Optional[Sequence] = None,
               split: str = "layer_validation", expected_samples: int = 512, block_size: int = 16,
               mask_token_id: Optional[int] = None, devices: Sequence[str] = ("cuda:0",), dtype: str = "bf16",
               synthetic_seed: int = 0) -> dict:
    import pandas as pd
    import torch.distributed as dist
    from ..utils.io import write_json
    from .common import read_examples
    output = Path(output_dir).resolve()
    if output.exists():
        raise FileExistsError(f"Refusing to overwrite {output}")
    if len(devices) != len(set(devices)):
        raise ValueError("--devices must be unique")
    paths = discover(run_dir, checkpoints)
    if str(examples_path) == "synthetic":
        import random
        from ..config import ModelConfig
        from .modeling import examples_from_sequences
        vocab = min(ModelConfig.from_pretrained(paths[0]).vocab_size, 151643) - 2
        rng = random.Random(synthetic_seed)
        seqs = [[rng.randrange(vocab) for _ in range(64 + block_size)] for _ in range(expected_samples)]
        exs = examples_from_sequences(seqs, block_size, 1, rng)
        ids = [str(i) for i in range(len(exs))]
    else:
        ids, exs = read_examples(examples_path, split, block_size)
    if expected_samples and len(exs) != expected_samples:
        raise ValueError(f"Expected {expected_samples} examples, found {len(exs)}")
    rows = score_checkpoints(paths, exs, block_size, devices, mask_token_id, dtype)
    table = rank_checkpoints(rows)
    best = table[0]
    chosen = {"format_version": 1, "selection_metric": "mean_accept_length",
              "selected_checkpoint": best["checkpoint"], "selected_step": best["step"],
              "mean_accept_length": best["mean_accept_length"],
              "mean_draft_token_accuracy": best["mean_draft_token_accuracy"], "samples": best["samples"]}
    if not dist.is_initialized() or dist.get_rank() == 0:
        output.mkdir(parents=True)
        metrics = pd.DataFrame([{"checkpoint": p, "analysis_id": ids[i], "emitted_tokens": r[0],
                                 "draft_token_accuracy": r[1]} for p, rs in rows.items() for i, r in enumerate(rs)])
        metrics.sort_values(["checkpoint", "analysis_id"]).to_parquet(output / "checkpoint_metrics.parquet",
                                                                      index=False)
        cols = ["rank", "checkpoint", "mean_accept_length", "mean_draft_token_accuracy", "samples", "step"]
        pd.DataFrame(table)[cols].to_csv(output / "checkpoint_summary.csv", index=False)
        write_json(str(output / "selected_checkpoint.json"), chosen)
        print(f"Selected {best['checkpoint']} with mean accept length {best['mean_accept_length']:.6f}.")
    return {"best": best, "ranking": table, "selected": chosen}
