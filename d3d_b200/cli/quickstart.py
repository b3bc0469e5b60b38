"""Ready-made runs with fixed defaults, extra flags appended (reference:
``scripts/quickstart_single.sh``, ``quickstart_concurrent.sh``,
``benchmark.sh``, ``train.sh``, ``prune.sh``, ``smoke_test.sh``).

    python -m d3d_b200.cli.quickstart single     [flags ...]   # one math500 prompt, 2 GPUs
    python -m d3d_b200.cli.quickstart concurrent [flags ...]   # CONCURRENCY (4) requests, paged engine
    python -m d3d_b200.cli.quickstart benchmark  [flags ...]   # every DATASETS set, 128 prompts each
    python -m d3d_b200.cli.quickstart train      [flags ...]   # NUM_GPUS (4) ranks of distillation
    python -m d3d_b200.cli.quickstart prune {select,prune,train,choose} [flags ...]
    python -m d3d_b200.cli.quickstart smoke                    # imports and hardware check

Models come from ``TARGET_MODEL`` / ``DRAFT_MODEL`` (presets or checkpoint
directories), evaluation sets from ``DATASETS``, training data from
``DATA_PATH``, outputs go under ``outputs/``.  Later flags override the
defaults (argparse keeps the last value).
"""
from __future__ import annotations

import os
import subprocess
import sys
from typing import List

SETS = "gsm8k math500 humaneval mbpp mt-bench aime25 livecodebench-v6"


def _models():
    return os.environ.get("TARGET_MODEL", "qwen3-8b"), os.environ.get("DRAFT_MODEL", "d3d-1.7b")


def plan(recipe: str, extra: List[str]) -> List[List[str]]:
    """The command lines a recipe runs (each a full ``argv``)."""
    py = [sys.executable, "-m"]
    target, draft = _models()
    tok = os.environ.get("TOKENIZER", target)
    if recipe == "single":
        return [py + ["d3d_b200.cli.single", "--verifier", target, "--drafter", draft, "--dataset", "math500",
                      "--tokenizer", tok, "--max-samples", "1", "--max-new-tokens", "128",
                      "--verifier-device", "cuda:0", "--draft-device", "cuda:1", "--temperature", "0",
                      "--block-size", "16", "--attention-mask-mode", "causal", "--anchor-num", "3",
                      "--packed-accepted-counts", "all", "--output-json", "outputs/single/result.json",
                      "--summary-json", "outputs/single/summary.json"] + extra]
    if recipe == "concurrent":
        c = int(os.environ.get("CONCURRENCY", "4"))
        return [py + ["d3d_b200.cli.serve", "--target", target, "--draft", draft, "--datasets", "math500",
                      "--tokenizer", tok, "--max-samples", "4", "--max-new-tokens", "128", "--concurrency", str(c),
                      "--anchor-num", "1" if c > 1 else "3", "--pages", "4096",
                      "--output", "outputs/concurrent/quickstart.json"] + extra]
    if recipe == "benchmark":
        return [py + ["d3d_b200.cli.single", "--verifier", target, "--drafter", draft, "--dataset", ds,
                      "--tokenizer", tok, "--max-samples", "128", "--max-new-tokens", "2048",
                      "--verifier-device", "cuda:0", "--draft-device", "cuda:1", "--temperature", "0",
                      "--block-size", "16", "--attention-mask-mode", "causal", "--anchor-num", "3",
                      "--packed-accepted-counts", "all", "--output-json", f"outputs/benchmark/{ds}.json",
                      "--summary-json", f"outputs/benchmark/{ds}.summary.json"] + extra
                for ds in os.environ.get("DATASETS", SETS).split()]
    if recipe == "train":
        n = os.environ.get("NUM_GPUS", "4")
        return [py + ["torch.distributed.run", "--nproc-per-node", n, "--master-addr", "127.0.0.1",
                      "--master-port", os.environ.get("MASTER_PORT", "29674"), "-m", "d3d_b200.train",
                      "--draft-model", draft, "--tokenizer-model", tok,
                      "--data-path", os.environ.get("DATA_PATH", "data/train.jsonl"),
                      "--output-dir", os.environ.get("OUTPUT_DIR", "outputs/d3d_b16_a128"),
                      "--objective", "ce", "--ce-weight", "1.0", "--ar-loss-weight", "1.0", "--block-size", "16",
                      "--parallel-anchors-per-example", "128", "--loss-decay-gamma", "7.75", "--batch-size", "1",
                      "--gradient-accumulation-steps", "8", "--epochs", "1", "--lr", "1e-5", "--min-lr-ratio",
                      "0.5", "--warmup-steps", "200", "--weight-decay", "0.0"] + extra]
    if recipe == "prune":
        if not extra or extra[0] not in ("select", "prune", "train", "choose"):
            raise SystemExit("prune needs a stage: select, prune, train or choose")
        if extra[0] == "train":
            n = os.environ.get("NUM_GPUS", "1")
            return [py + ["torch.distributed.run", "--nproc-per-node", n, "--master-addr", "127.0.0.1",
                          "-m", "d3d_b200.pruning"] + extra]
        return [py + ["d3d_b200.pruning"] + extra]
    if recipe == "smoke":
        return [[sys.executable, "-c", "import d3d_b200.cli.quickstart as q; q.smoke()"] + extra]
    raise SystemExit(f"unknown recipe {recipe!r}: single, concurrent, benchmark, train, prune or smoke")


def smoke(require_gpus: int = 2) -> None:
    """Import every module of the package, load the compiled extension and
    check the GPUs (two for the two-process layouts)."""
    import importlib
    import pkgutil
    import torch
    import d3d_b200
    for m in pkgutil.walk_packages(d3d_b200.__path__, "d3d_b200."):
        if not m.name.endswith("__main__"):
            importlib.import_module(m.name)
    if require_gpus:
        if not torch.cuda.is_available():
            raise SystemExit("CUDA is required for the smoke test")
        if torch.cuda.device_count() < require_gpus:
            raise SystemExit(f"{require_gpus} GPUs are required, found {torch.cuda.device_count()}")
        from .. import ops
        ops.ext()
    print("d3d_b200 import and hardware smoke test passed")


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] in ("-h", "--help"):
        print(__doc__)
        return 0
    for cmd in plan(argv[0], argv[1:]):
        os.makedirs("outputs", exist_ok=True)
        rc = subprocess.call(cmd)
        if rc:
            return rc
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
