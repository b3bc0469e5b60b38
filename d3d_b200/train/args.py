"""Training flags (names follow the reference's ``train/arguments.py``)."""
from __future__ import annotations

import argparse

import torch


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Block-diffusion drafter distillation")
    p.add_argument("--draft-model", required=True, help="checkpoint dir or preset (e.g. d3d-1.7b)")
    p.add_argument("--target-model", default="", help="frozen teacher checkpoint dir or preset")
    p.add_argument("--data-path", default="synthetic")
    p.add_argument("--output-dir", required=True)
    p.add_argument("--objective", default="kl_ce", help="ce | forward_kl | kl_ce")
    p.add_argument("--kl-weight", type=float, default=1.0)
    p.add_argument("--ce-weight", type=float, default=1.0)
    p.add_argument("--ce-on-target-greedy", action="store_true",
                   help="CE targets are the teacher's greedy tokens instead of the data")
    p.add_argument("--block-size", type=int, default=16)
    p.add_argument("--loss-decay-gamma", type=float, default=15.5)
    p.add_argument("--batch-size", type=int, default=4, help="sequences per rank per step")
    p.add_argument("--seq-len", type=int, default=2048, help="synthetic sequence length")
    p.add_argument("--tokenizer", default=None, help="tokenizer directory (chat / text JSONL rows)")
    p.add_argument("--max-examples", type=int, default=0, help="use the first N rows of the file (0 = all)")
    p.add_argument("--max-prompt-len", type=int, default=4096)
    p.add_argument("--max-seq-len", type=int, default=8192)
    p.add_argument("--enable-thinking-template", action="store_true")
    p.add_argument("--parallel-anchors-per-example", type=int, default=32)
    p.add_argument("--max-steps", type=int, default=10)
    p.add_argument("--lr", type=float, default=1e-4)
    p.add_argument("--min-lr-ratio", type=float, default=0.0)
    p.add_argument("--weight-decay", type=float, default=0.0)
    p.add_argument("--warmup-steps", type=int, default=0)
    p.add_argument("--grad-clip", type=float, default=1.0)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--dtype", choices=["bf16", "fp32"], default="bf16")
    p.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    p.add_argument("--draft-layers", type=int, default=None)
    p.add_argument("--mask-token-id", type=int, default=None)
    p.add_argument("--freeze-embeddings", action="store_true")
    p.add_argument("--gradient-checkpointing", action="store_true",
                   help="recompute each decoder layer in backward instead of keeping its activations "
                        "(the clean-prefix KV stays cached)")
    p.add_argument("--fsdp", action="store_true",
                   help="shard decoder-layer parameters over the ranks (gathered per layer, "
                        "recomputed in backward, gradients reduce-scattered per layer)")
    p.add_argument("--vocab-chunk", type=int, default=16384)
    p.add_argument("--save-every", type=int, default=0)
    p.add_argument("--save-final", action="store_true")
    p.add_argument("--resume", default=None, help="checkpoint directory written by --save-*")
    p.add_argument("--log-every", type=int, default=1)
    # auxiliary objectives on the student logits (off by default)
    p.add_argument("--hnce-weight", type=float, default=0.0, help="hard-negative CE weight")
    p.add_argument("--hnce-top-k", type=int, default=16)
    p.add_argument("--hnce-margin", type=float, default=0.0)
    p.add_argument("--margin-weight", type=float, default=0.0, help="top-k target margin weight")
    p.add_argument("--margin-top-k", type=int, default=16)
    p.add_argument("--margin-value", type=float, default=1.0)
    p.add_argument("--margin-hinge", action="store_true", help="hinge instead of softplus margin")
    p.add_argument("--ar-weight", type=float, default=0.0,
                   help="next-token CE of the student on the clean sequences (fused LM-head loss)")
    p.add_argument("--trajectory-weight", type=float, default=0.0,
                   help="hidden-trajectory (block relation) distillation weight; needs --target-model")
    return p
