"""Training flags: the reference's names and defaults (``train/arguments.py``,
``train/runtime.py:70-88``), plus this framework's own switches."""
from __future__ import annotations

import argparse

import torch


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Block-diffusion drafter distillation")
    p.add_argument("--draft-model", required=True, help="checkpoint dir or preset (e.g. d3d-1.7b)")
    p.add_argument("--draft-code-model", default="",
                   help="accepted for compatibility: the drafter's model code is this framework's")
    p.add_argument("--target-model", default="", help="frozen teacher checkpoint dir or preset")
    p.add_argument("--tokenizer-model", "--tokenizer", dest="tokenizer", default=None,
                   help="tokenizer directory (chat / text JSONL rows)")
    p.add_argument("--data-path", default="synthetic")
    p.add_argument("--output-dir", required=True)
    p.add_argument("--objective", default="ce", help="ce | forward_kl | reverse_kl | kl_ce (and aliases)")
    p.add_argument("--kl-weight", type=float, default=1.0)
    p.add_argument("--ce-weight", type=float, default=1.0)
    p.add_argument("--ce-on-target-greedy", action="store_true",
                   help="CE targets are the teacher's greedy tokens instead of the data")
    p.add_argument("--block-size", type=int, default=32)
    p.add_argument("--loss-decay-gamma", type=float, default=15.5)
    p.add_argument("--batch-size", type=int, default=1, help="sequences per rank per micro-step")
    p.add_argument("--parallel-anchors-per-example", type=int, default=32)
    p.add_argument("--seq-len", type=int, default=2048, help="synthetic sequence length")
    p.add_argument("--max-examples", type=int, default=0, help="use the first N rows of the file (0 = all)")
    p.add_argument("--max-prompt-len", type=int, default=4096)
    p.add_argument("--max-seq-len", type=int, default=8192)
    p.add_argument("--enable-thinking-template", dest="enable_thinking_template", action="store_true",
                   default=True)
    p.add_argument("--disable-thinking-template", dest="enable_thinking_template", action="store_false")
    p.add_argument("--fix-mistral-regex", action=argparse.BooleanOptionalAction, default=False,
                   help="load the tokenizer with transformers' fix_mistral_regex correction")
    # schedule
    p.add_argument("--epochs", type=int, default=1, help="passes over the data when --max-steps is 0")
    p.add_argument("--max-micro-steps", type=int, default=0, help="cap on micro-steps (0 = none)")
    p.add_argument("--max-steps", type=int, default=0,
                   help="optimizer steps (0 = from --epochs / --max-micro-steps and the data size)")
    p.add_argument("--gradient-accumulation-steps", type=int, default=1)
    p.add_argument("--lr", type=float, default=3.0e-6)
    p.add_argument("--min-lr-ratio", type=float, default=0.0)
    p.add_argument("--weight-decay", type=float, default=0.0)
    p.add_argument("--warmup-steps", type=int, default=200)
    p.add_argument("--grad-clip", type=float, default=1.0)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--dtype", choices=["bf16", "fp32"], default="bf16")
    p.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    # model
    p.add_argument("--attn-implementation", default=None, choices=["sdpa", "eager", "flash_attention_2"],
                   help="attention math of the student's PyTorch layers")
    p.add_argument("--gradient-checkpointing", action="store_true",
                   help="recompute each decoder layer in backward instead of keeping its activations "
                        "(the clean-prefix KV stays cached)")
    p.add_argument("--random-init", action="store_true",
                   help="start from a seeded random init of the drafter's configuration instead of its weights")
    p.add_argument("--mask-token", default="<MASK>",
                   help="token whose id is the mask when neither the checkpoint nor --mask-token-id sets one")
    p.add_argument("--mask-token-id", type=int, default=None,
                   help="existing embedding row used as the mask (Qwen3 default 151669)")
    p.add_argument("--draft-layers", type=int, default=None, help="preset drafters only")
    p.add_argument("--freeze-embeddings", action="store_true")
    p.add_argument("--vocab-chunk", type=int, default=16384,
                   help="vocabulary columns per pass of the fused LM-head loss")
    # data loading
    p.add_argument("--workers", type=int, default=8,
                   help="host threads packing batches ahead of the device (0 = pack inline)")
    p.add_argument("--prefetch", type=int, default=2, help="batches packed ahead per worker")
    p.add_argument("--persistent-workers", dest="persistent_workers", action="store_true", default=True)
    p.add_argument("--no-persistent-workers", dest="persistent_workers", action="store_false")
    p.add_argument("--pin-memory", dest="pin_memory", action="store_true", default=True)
    p.add_argument("--no-pin-memory", dest="pin_memory", action="store_false")
    # sharding
    p.add_argument("--fsdp", dest="fsdp", action="store_true", default=False,
                   help="shard decoder-layer parameters over the ranks (gathered per layer over NVLink, "
                        "recomputed in backward, gradients reduce-scattered per layer); off by default: a "
                        "replicated drafter with sharded optimizer state is faster and fits")
    p.add_argument("--no-fsdp", dest="fsdp", action="store_false")
    p.add_argument("--fsdp-cpu-offload", action="store_true",
                   help="fp32 master weights and Adam moments in host memory, update on the CPU")
    p.add_argument("--fsdp-reshard-after-forward", dest="fsdp_reshard_after_forward", action="store_true",
                   default=True, help="sharded layers are gathered again in backward (the only mode)")
    p.add_argument("--no-fsdp-reshard-after-forward", dest="fsdp_reshard_after_forward", action="store_false")
    p.add_argument("--fsdp-transformer-layer-cls", action="append", default=None,
                   help="layer class to shard (decoder layers: D3DDecoderLayer / Qwen3DecoderLayer)")
    # checkpoints and logging
    p.add_argument("--save-every", type=int, default=200)
    p.add_argument("--save-final", action="store_true")
    p.add_argument("--resume", default=None, help="checkpoint directory written by --save-*")
    p.add_argument("--log-every", type=int, default=1)
    p.add_argument("--wandb-project", default="")
    p.add_argument("--wandb-name", default="")
    p.add_argument("--disable-wandb", action="store_true")
    # auxiliary objectives on the student logits (off by default)
    p.add_argument("--hnce-weight", type=float, default=0.0, help="hard-negative CE weight")
    p.add_argument("--hnce-top-k", type=int, default=16)
    p.add_argument("--hnce-margin", type=float, default=0.0)
    p.add_argument("--margin-weight", type=float, default=0.0, help="top-k target margin weight")
    p.add_argument("--margin-top-k", type=int, default=4)
    p.add_argument("--margin-value", type=float, default=0.5)
    p.add_argument("--margin-smooth", action="store_true", help="softplus instead of hinge margin")
    p.add_argument("--ar-loss-weight", "--ar-weight", dest="ar_weight", type=float, default=0.0,
                   help="next-token CE of the student on the clean sequences (fused LM-head loss)")
    p.add_argument("--ar-logit-chunk-size", type=int, default=512,
                   help="accepted for compatibility: the fused LM-head loss never materialises AR logits")
    # trajectory distillation
    p.add_argument("--trajectory-weight", type=float, default=0.0,
                   help="hidden-trajectory (block relation) distillation weight")
    p.add_argument("--trajectory-teacher-model", default="",
                   help="teacher of the trajectory term (default: --target-model)")
    p.add_argument("--trajectory-teacher-code-model", default="",
                   help="accepted for compatibility: the teacher's model code is this framework's")
    p.add_argument("--trajectory-gradient-probe-steps", type=int, default=0,
                   help="for the first N micro-steps, record the gradient norms of the unit trajectory term "
                        "and of the CE term at the student's final hidden states")
    p.add_argument("--trajectory-shuffle-teacher-blocks", action="store_true",
                   help="negative control: shuffle teacher relation targets among selected blocks of equal "
                        "active length")
    return p
