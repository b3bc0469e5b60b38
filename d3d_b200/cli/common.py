"""Shared CLI plumbing: model/engine construction and prompt loading."""
from __future__ import annotations

import argparse
from pathlib import Path
from typing import List, Optional, Sequence

import torch

from .. import config as C
from ..utils.data import load_jsonl_prompts, synthetic_prompts


def add_model_args(p: argparse.ArgumentParser, target_flag: str, draft_flag: str,
                   dtypes: Sequence[str] = ("bf16",)) -> None:
    p.add_argument(target_flag, dest="target", required=True,
                   help="target checkpoint directory or preset name")
    p.add_argument(draft_flag, dest="draft", required=True, help="drafter checkpoint directory or preset name")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--dtype", default="bf16", choices=list(dtypes))
    p.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    p.add_argument("--mask-token-id", type=int, default=None)
    p.add_argument("--draft-layers", type=int, default=None, help="preset drafters only")


def add_data_args(p: argparse.ArgumentParser, max_samples: Optional[int] = None) -> None:
    """Prompt-source flags.  ``--max-samples`` defaults to ``max_samples``;
    ``None`` reads every example of a file or evaluation set (and draws 8
    synthetic prompts)."""
    p.add_argument("--dataset", default="synthetic",
                   help="'synthetic', a JSONL file of prompts, or an evaluation set by name "
                        "(gsm8k, math500, aime25, humaneval, mbpp, mt-bench, livecodebench-v6; read from "
                        "$D3D_DATA_CACHE / $D3D_ANSWER_CACHE, rendered with the tokenizer's chat template)")
    p.add_argument("--enable-thinking", action="store_true", help="evaluation sets: thinking chat template")
    p.add_argument("--max-samples", type=int, default=max_samples)
    p.add_argument("--prompt-min", type=int, default=128)
    p.add_argument("--prompt-max", type=int, default=512)
    p.add_argument("--tokenizer", default=None, help="tokenizer directory for text prompts")


def load_prompts(args) -> List[List[int]]:
    if args.dataset == "synthetic":
        vocab = min(151643, model_config(args.target).vocab_size - 2)
        n = args.max_samples if args.max_samples else 8
        return synthetic_prompts(n, args.prompt_min, args.prompt_max, seed=1000 + args.seed,
                                 vocab=vocab)
    tok = None
    if args.tokenizer:
        from transformers import AutoTokenizer
        tok = AutoTokenizer.from_pretrained(args.tokenizer)
    from ..utils.benchsets import SETS, load_set
    if args.dataset in SETS and not Path(args.dataset).is_file():
        if tok is None:
            raise ValueError(f"--dataset {args.dataset} needs --tokenizer (questions are text)")
        from ..utils.text import chat_prompt
        exs, meta = load_set(args.dataset, args.max_samples)
        args.eval_examples, args.eval_meta, args.eval_tokenizer = exs, meta, tok
        return [tok.encode(chat_prompt(tok, e.question, thinking=getattr(args, "enable_thinking", False)),
                           add_special_tokens=False) for e in exs]
    return load_jsonl_prompts(args.dataset, tok, args.max_samples)


def load_selected_prompts(args) -> List[List[int]]:
    """``load_prompts``, restricted to example ``args.sample_index`` when set
    (an evaluation set's own example index; the position otherwise)."""
    idx = getattr(args, "sample_index", None)
    if idx is None:
        return load_prompts(args)
    args.max_samples = idx + 1 if args.dataset == "synthetic" else None
    prompts = load_prompts(args)
    exs = getattr(args, "eval_examples", None)
    keep = [i for i in range(len(prompts)) if (exs[i].index if exs else i) == idx][:1]
    if not keep:
        raise ValueError(f"--sample-index {idx} not found in {args.dataset}")
    if exs:
        args.eval_examples = [exs[i] for i in keep]
    return [prompts[i] for i in keep]


def score_outputs(args, outputs: List[List[int]]) -> Optional[dict]:
    """Exact-answer accuracy of decoded outputs on a scored evaluation set
    (``None`` for other prompt sources); fills ``pred`` / ``correct`` per row."""
    exs = getattr(args, "eval_examples", None)
    if not exs:
        return None
    from ..utils.benchsets import score
    tok = args.eval_tokenizer
    rows, hits, scored = [], 0, 0
    for e, toks in zip(exs, outputs):
        pred, ok = score(e.dataset, tok.decode(toks, skip_special_tokens=True), e.gold)
        rows.append({"index": e.index, "gold": e.gold, "pred": pred, "correct": ok})
        if ok is not None:
            scored += 1
            hits += bool(ok)
    return {"set": args.eval_meta, "scored": scored, "correct": hits,
            "accuracy": hits / scored if scored else None, "rows": rows}


def check_devices(*devices) -> None:
    """Exit with a clear message when a requested GPU does not exist (the
    reference's hardware check, ``common/runtime.py:31-43``)."""
    for d in devices:
        dev = torch.device(d)
        if dev.type == "cuda" and (not torch.cuda.is_available() or (dev.index or 0) >= torch.cuda.device_count()):
            raise SystemExit(f"device {dev} is not available ({torch.cuda.device_count()} CUDA devices)")


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
                                      target_pages=pages, device=dev)
    t = load_module(args.target, dev, args.seed)
    d = load_module(args.draft, dev, args.seed, args.draft_layers, args.mask_token_id)
    return D3DEngine.from_modules(t, d, decode)


def hf_greedy_agreement(target: str, device, prompts: List[List[int]], outputs: List[List[int]],
                        budgets: List[int]) -> dict:
    """Greedy continuations of ``transformers``' own Qwen3 implementation for
    the same checkpoint (the reference's validation oracle): the fraction of
    requests whose output is identical, and each request's first divergent
    position (``None`` when identical).  On bf16 kernels an early divergence
    can be a near-tie, not an error; fp32 models agree exactly."""
    import transformers
    dt = torch.bfloat16 if torch.device(device).type == "cuda" else torch.float32
    hf = transformers.AutoModelForCausalLM.from_pretrained(target, dtype=dt).to(device).eval()
    first = []
    for p, o, n in zip(prompts, outputs, budgets):
        with torch.no_grad():
            ref = hf.generate(torch.tensor([p], device=device), max_new_tokens=int(n), do_sample=False,
                              pad_token_id=0)[0, len(p):].tolist()
        k = next((i for i, (x, y) in enumerate(zip(o, ref)) if x != y), None)
        if k is None and len(o) != len(ref):
            k = min(len(o), len(ref))
        first.append(k)
    same = sum(k is None for k in first)
    return {"identical": same, "requests": len(first), "rate": same / max(1, len(first)),
            "first_divergence": first}


def parse_cpu_list(value: Optional[str]) -> List[int]:
    """CPU ids from a list such as ``"0-3,8,10-11"`` (empty for ``None``)."""
    out: List[int] = []
    for part in (value or "").replace(" ", "").split(","):
        if not part:
            continue
        if "-" in part:
            lo, hi = (int(x) for x in part.split("-", 1))
            if hi < lo:
                raise ValueError(f"bad CPU range {part!r}")
            out.extend(range(lo, hi + 1))
        else:
            out.append(int(part))
    return sorted(set(out))


def pin_host_threads(*cpu_lists: Optional[str]) -> Optional[List[int]]:
    """Restrict this process to the union of the given CPU lists (the
    reference pins its verifier and drafter processes; here the target's
    host work runs in the coordinator's process, so both sets apply to it)."""
    import os
    cpus = sorted(set(c for v in cpu_lists for c in parse_cpu_list(v)))
    if not cpus:
        return None
    os.sched_setaffinity(0, set(cpus))
    return cpus
