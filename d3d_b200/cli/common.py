"""Shared CLI plumbing: model/engine construction and prompt loading."""
from __future__ import annotations

import argparse
from pathlib import Path
from typing import List, Optional

import torch

from .. import config as C
from ..utils.data import load_jsonl_prompts, synthetic_prompts


def add_model_args(p: argparse.ArgumentParser, target_flag: str, draft_flag: str) -> None:
    p.add_argument(target_flag, dest="target", required=True,
                   help="target checkpoint directory or preset name")
    p.add_argument(draft_flag, dest="draft", required=True, help="drafter checkpoint directory or preset name")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--dtype", default="bf16", choices=["bf16"])
    p.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    p.add_argument("--mask-token-id", type=int, default=None)
    p.add_argument("--draft-layers", type=int, default=None, help="preset drafters only")


def add_data_args(p: argparse.ArgumentParser) -> None:
    p.add_argument("--dataset", default="synthetic", help="'synthetic' or a JSONL file of prompts")
    p.add_argument("--max-samples", type=int, default=8)
    p.add_argument("--prompt-min", type=int, default=128)
    p.add_argument("--prompt-max", type=int, default=512)
    p.add_argument("--tokenizer", default=None, help="tokenizer directory for text prompts")


def load_prompts(args) -> List[List[int]]:
    if args.dataset == "synthetic":
        vocab = min(151643, model_config(args.target).vocab_size - 2)
        return synthetic_prompts(args.max_samples, args.prompt_min, args.prompt_max, seed=1000 + args.seed,
                                 vocab=vocab)
    tok = None
    if args.tokenizer:
        from transformers import AutoTokenizer
        tok = AutoTokenizer.from_pretrained(args.tokenizer)
    return load_jsonl_prompts(args.dataset, tok, args.max_samples)


def is_preset(name: str) -> bool:
    return name in C.PRESETS and not Path(name).is_dir()


def model_config(name: str, draft_layers: Optional[int] = None) -> C.ModelConfig:
    if is_preset(name):
        cfg = C.PRESETS[name]()
        if draft_layers and cfg.d3d_draft:
            cfg = cfg.replace(num_hidden_layers=draft_layers)
        return cfg
    return C.ModelConfig.from_pretrained(name)


def load_fast_weights(name: str, device, seed: int, draft_layers: Optional[int] = None,
                      mask_token_id: Optional[int] = None):
    from ..models.fast import FastWeights
    if is_preset(name):
        return FastWeights.random(model_config(name, draft_layers), seed=seed, device=device)
    from ..checkpoint import load_model
    m = load_model(name, device="cpu", mask_token_id=mask_token_id)
    return FastWeights.from_module(m, device)


def load_module(name: str, device, seed: int, draft_layers: Optional[int] = None,
                mask_token_id: Optional[int] = None):
    from ..models.qwen3 import build_model
    if is_preset(name):
        return build_model(model_config(name, draft_layers), seed=seed, device=device)
    from ..checkpoint import load_model
    return load_model(name, device=device, mask_token_id=mask_token_id)


def build_engine(args, decode, max_seqs: int, max_context: int, pages: Optional[int] = None):
    from ..api import D3DEngine
    dev = torch.device(args.device)
    if dev.type == "cuda":
        tw = load_fast_weights(args.target, dev, args.seed)
        dw = load_fast_weights(args.draft, dev, args.seed, args.draft_layers, args.mask_token_id)
        return D3DEngine.from_weights(tw, dw, decode, max_seqs=max_seqs, max_context=max_context,
                                      target_pages=pages, draft_pages=None if pages is None else None,
                                      device=dev)
    t = load_module(args.target, dev, args.seed)
    d = load_module(args.draft, dev, args.seed, args.draft_layers, args.mask_token_id)
    return D3DEngine.from_modules(t, d, decode)
