"""``python -m d3d_b200.pruning {select,prune,train,choose}`` -- one stage of
progressive layer pruning, with the reference's flags and files
(``scripts/prune.sh``; ``pruning/select_layer.py``, ``prune.py``,
``train_recovery.py``, ``select_checkpoint.py``).

    select  --parent DIR --examples FILE --output-dir DIR [--devices cuda:0 cuda:1 ...]
            -> candidate_metrics.parquet, candidate_summary.csv, selection.json
    prune   --selection DIR/selection.json --output DIR
            -> the child checkpoint with layer_prune.json
    train   --student DIR --dataset FILE --output-dir DIR --max-steps N
            -> run_config.json, training_metrics.jsonl, step-N/, training_summary.json
            (multi-GPU: python -m torch.distributed.run --nproc-per-node G -m d3d_b200.pruning train ...)
    choose  (--run-dir DIR | --checkpoints DIR ...) --examples FILE --output-dir DIR
            -> checkpoint_metrics.parquet, checkpoint_summary.csv, selected_checkpoint.json

``--examples`` is a Parquet/JSONL/JSON file of ``prefix_ids`` / ``target_ids``
rows (optional ``analysis_id``, ``split``), or ``synthetic``.  ``select`` and
``choose`` also run data-parallel under ``torch.distributed.run`` (one
process per GPU, examples sharded, rows gathered in order).
"""
from __future__ import annotations

import argparse
import os
from pathlib import Path

import torch


def _cuda_default() -> str:
    return "cuda:0" if torch.cuda.is_available() else "cpu"


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="python -m d3d_b200.pruning", description=__doc__,
                                formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = p.add_subparsers(dest="stage", required=True)

    s = sub.add_parser("select", help="rank single-layer deletions on a tokenized split")
    s.add_argument("--parent", type=Path, required=True)
    s.add_argument("--examples", required=True, help="Parquet/JSONL/JSON of prefix_ids/target_ids, or 'synthetic'")
    s.add_argument("--output-dir", type=Path, required=True)
    s.add_argument("--split", default="layer_selection")
    s.add_argument("--expected-samples", type=int, default=512)
    s.add_argument("--block-size", type=int, default=16)
    s.add_argument("--mask-token-id", type=int, default=None)
    s.add_argument("--candidate-batch-size", type=int, default=2,
                   help="accepted for compatibility: every deletion reuses the shared layer prefix instead")
    s.add_argument("--devices", nargs="+", default=[_cuda_default()])
    s.add_argument("--dtype", choices=["bf16", "fp32"], default="bf16")
    s.add_argument("--bootstrap-samples", type=int, default=10_000)
    s.add_argument("--bootstrap-seed", type=int, default=42)

    s = sub.add_parser("prune", help="physically remove the layer recorded in selection.json")
    s.add_argument("--selection", type=Path, required=True)
    s.add_argument("--output", type=Path, required=True)

    s = sub.add_parser("train", help="fixed-budget recovery training of a pruned child")
    s.add_argument("--student", type=Path, required=True)
    s.add_argument("--dataset", required=True,
                   help="JSONL rows (chat, text or prompt_ids/response_ids), or 'synthetic'")
    s.add_argument("--output-dir", type=Path, required=True)
    s.add_argument("--data-cursor", type=int, default=0)
    s.add_argument("--max-steps", type=int, required=True)
    s.add_argument("--gradient-accumulation-steps", type=int, default=8)
    s.add_argument("--candidate-multiplier", type=float, default=2.0)
    s.add_argument("--anchors-per-example", type=int, default=0, help="default 2048 / block size")
    s.add_argument("--max-prompt-tokens", type=int, default=4096)
    s.add_argument("--max-sequence-tokens", type=int, default=8192)
    s.add_argument("--learning-rate", type=float, default=1e-5)
    s.add_argument("--min-lr", type=float, default=1e-6)
    s.add_argument("--warmup-ratio", type=float, default=0.01)
    s.add_argument("--gradient-clip", type=float, default=1.0)
    s.add_argument("--weight-decay", type=float, default=0.0)
    s.add_argument("--save-steps", type=int, default=500)
    s.add_argument("--log-steps", type=int, default=10)
    s.add_argument("--seed", type=int, default=42)
    s.add_argument("--optimizer", choices=["adamw8bit", "adamw"], default="adamw8bit")
    s.add_argument("--fsdp-cpu-offload", action="store_true",
                   help="fp32 master weights and moments in host memory, update on the CPU")
    s.add_argument("--fsdp", action="store_true",
                   help="shard the student's decoder layers over the ranks (gathered per layer over NVLink)")
    s.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")

    s = sub.add_parser("choose", help="pick the recovery checkpoint with the highest validation acceptance")
    src = s.add_mutually_exclusive_group(required=True)
    src.add_argument("--run-dir", type=Path)
    src.add_argument("--checkpoints", type=Path, nargs="+")
    s.add_argument("--examples", required=True)
    s.add_argument("--output-dir", type=Path, required=True)
    s.add_argument("--split", default="layer_validation")
    s.add_argument("--expected-samples", type=int, default=512)
    s.add_argument("--block-size", type=int, default=16)
    s.add_argument("--mask-token-id", type=int, default=None)
    s.add_argument("--devices", nargs="+", default=[_cuda_default()])
    s.add_argument("--dtype", choices=["bf16", "fp32"], default="bf16")
    return p


def _dist_devices(devices):
    """Under ``torch.distributed.run``: join the group; each rank uses its
    ``LOCAL_RANK`` GPU (or the CPU) and scores its share of the examples."""
    from ..train.trainer import _init_dist
    kind = torch.device(devices[0]).type
    rank, world = _init_dist(kind)
    if world > 1 and kind == "cuda":
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        return [f"cuda:{local}"]
    return list(devices)


def main(argv=None):
    a = parser().parse_args(argv)
    if a.stage == "select":
        from .select_layer import run_select
        return run_select(a.parent, a.examples, a.output_dir, split=a.split, expected_samples=a.expected_samples,
                          block_size=a.block_size, mask_token_id=a.mask_token_id, devices=_dist_devices(a.devices),
                          dtype=a.dtype, bootstrap_samples=a.bootstrap_samples, bootstrap_seed=a.bootstrap_seed)
    if a.stage == "prune":
        from .prune import prune_from_selection
        out = prune_from_selection(a.selection, a.output)
        print(f"Pruned checkpoint written to {out}")
        return out
    if a.stage == "choose":
        from .select_checkpoint import run_choose
        return run_choose(a.output_dir, a.examples, run_dir=a.run_dir, checkpoints=a.checkpoints, split=a.split,
                          expected_samples=a.expected_samples, block_size=a.block_size,
                          mask_token_id=a.mask_token_id, devices=_dist_devices(a.devices), dtype=a.dtype)
    from ..train.trainer import _init_dist
    from .recovery import run_recovery
    device = torch.device(a.device)
    rank, world = _init_dist(device.type)
    if device.type == "cuda":
        device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(device)
    return run_recovery(a, rank, world, device)


if __name__ == "__main__":
    main()
