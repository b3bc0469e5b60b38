"""Concurrent paged-KV serving benchmark (reference: ``serving/bench.py``).

    python -m d3d_b200.cli.serve --target qwen3-8b --draft d3d-1.7b --pages 4096 \\
        --concurrency 1,4,8,16 --max-new-tokens 512 --validate --output-json out/serve.json

Requests arrive all at once (closed loop); throughput is end to end
(prefill and admission included), as in the reference.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import time
from typing import Dict

from ..engine.controlled import ControlledAcceptance, rate_for_mean_accept
from ..engine.spec import DecodeConfig
from ..utils.io import write_json
from ..utils.runtime import check_paged_capacity, runtime_metadata
from .common import (add_data_args, add_model_args, build_engine, hf_greedy_agreement, is_preset,
                     load_prompts, score_outputs)


def parser():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    add_model_args(p, "--target", "--draft")
    add_data_args(p, max_samples=128)
    p.add_argument("--datasets", nargs="+", default=None,
                   help="several prompt sources in one run (names or files, as --dataset); one row per "
                        "(dataset, concurrency, repeat)")
    p.add_argument("--pages", type=int, default=4096)
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--concurrency", default="1,4,8,16")
    p.add_argument("--max-new-tokens", type=int, default=2048)
    p.add_argument("--max-new-tokens-range", default=None,
                   help="LO,HI: per-request output budgets drawn uniformly (seeded), e.g. 128,512")
    p.add_argument("--repeats", type=int, default=1, help="timed runs per (dataset, concurrency)")
    p.add_argument("--block-size", type=int, default=16)
    p.add_argument("--anchor-num", type=int, default=3)
    p.add_argument("--draft-microbatch", type=int, default=4)
    p.add_argument("--ignore-eos", action="store_true")
    p.add_argument("--backup", choices=["neural", "fast", "fast_legacy"], default="neural",
                   help="on a branch miss: redraft (neural) or verify a random block at once (fast: the "
                        "block's drafts cover commit length 1 only; fast_legacy: every commit length)")
    p.add_argument("--fast-miss-anchors", type=int, default=0,
                   help="fast backup: anchors drafted after a random block (0 = --anchor-num)")
    p.add_argument("--validate", action="store_true",
                   help="check token identity against AR decoding (an error when any request differs)")
    p.add_argument("--validate-hf", action="store_true",
                   help="compare the outputs with transformers' greedy generate on the target checkpoint")
    p.add_argument("--validate-draft", action="store_true",
                   help="compare the engine's drafter with the PyTorch drafter module on the first prompt "
                        "(recovery block equal, packed drafts >= 99%% equal)")
    p.add_argument("--baseline", action="store_true", help="AR baseline at each concurrency")
    p.add_argument("--controlled-accept-mean", type=float, default=None)
    p.add_argument("--output-json", "--output", dest="output_json", default=None)
    return p


def _load_sets(a) -> Dict[str, dict]:
    """Prompts (and evaluation-set scoring state) of every requested source."""
    sets, first = {}, a.dataset
    for name in a.datasets or [a.dataset]:
        a.dataset = name
        for k in ("eval_examples", "eval_meta", "eval_tokenizer"):
            if hasattr(a, k):
                delattr(a, k)
        prompts = load_prompts(a)
        if not prompts:
            raise ValueError(f"dataset {name} has no prompts")
        sets[name] = {"prompts": prompts, "eval": {k: getattr(a, k) for k in
                                                   ("eval_examples", "eval_meta", "eval_tokenizer")
                                                   if hasattr(a, k)}}
    a.dataset = first
    return sets


def main(argv=None):
    a = parser().parse_args(argv)
    conc = [int(c) for c in a.concurrency.split(",")]
    if min(conc + [a.max_samples, a.max_new_tokens, a.repeats, a.pages]) < 1:
        raise SystemExit("concurrency, samples, token count, repeats and pages must be positive")
    sets = _load_sets(a)
    budgets = {}
    if a.max_new_tokens_range:
        import random
        lo, hi = (int(x) for x in a.max_new_tokens_range.split(","))
        rng = random.Random(a.seed + 17)
        budgets = {n: [rng.randint(lo, hi) for _ in d["prompts"]] for n, d in sets.items()}
        a.max_new_tokens = hi
    lens = [len(p) for d in sets.values() for p in d["prompts"]]
    check_paged_capacity(lens, a.max_new_tokens, conc, a.pages, a.page_size, a.block_size, a.anchor_num)
    decode = DecodeConfig(block_size=a.block_size, anchor_num=a.anchor_num, max_new_tokens=a.max_new_tokens,
                          draft_microbatch=a.draft_microbatch, ignore_eos=a.ignore_eos, backup=a.backup,
                          fast_miss_anchors=a.fast_miss_anchors)
    eng = build_engine(a, decode, max_seqs=max(conc), max_context=max(lens) + a.max_new_tokens + 64, pages=a.pages)
    rows, warm = [], False
    draft_check = None
    if a.validate_draft:
        import copy
        from ..engine.validation import validate_draft
        # the oracle holds exactly the engine drafter's weights: unpacked from the
        # kernel layout on a GPU, a copy of the PyTorch module on the CPU
        d = eng.decoder.d
        oracle = d.w.to_module() if hasattr(d, "w") else copy.deepcopy(d.model)
        first = next(iter(sets.values()))["prompts"][0]
        draft_check = validate_draft(eng.decoder, oracle, first)
        del oracle
        print({k: v for k, v in draft_check.items() if k != "differences"}, flush=True)
    for name, d in sets.items():
        prompts, bud = d["prompts"], budgets.get(name)
        digest = hashlib.sha256(json.dumps(prompts).encode()).hexdigest()
        for k, v in d["eval"].items():
            setattr(a, k, v)
        if not d["eval"]:
            a.eval_examples = None
        ar = None
        if a.validate or a.baseline or a.controlled_accept_mean is not None:
            ar = eng.generate_ar(prompts, concurrency=max(conc), max_new=bud)
        ctl = None
        if a.controlled_accept_mean is not None:
            rate = rate_for_mean_accept(a.controlled_accept_mean, a.block_size)
            ctl = (lambda ps, outs: lambda i: ControlledAcceptance(ps[i] + outs[i], rate, int(eng.draft.vocab_size),
                                                                   seed=a.seed, stream=i))(prompts, ar["outputs"])
        if not warm:
            eng.generate(prompts[:1], max_new_tokens=16, controlled=ctl)           # warm-up
            warm = True
        for c in conc:
            ar_tps = None
            if a.baseline:
                t0 = time.perf_counter()
                b = eng.generate_ar(prompts, concurrency=c, max_new=bud)
                ar_tps = b["output_tokens"] / (time.perf_counter() - t0)
            for rep in range(a.repeats):
                r = eng.generate(prompts, concurrency=c, controlled=ctl, max_new=bud)
                row = {"dataset": name, "concurrency": c, "repeat": rep, "requests": len(prompts), "tps": r["tps"],
                       "elapsed_s": r["elapsed_s"], "output_tokens": r["output_tokens"],
                       "mean_accept_length": r["mean_accept_length"], "accept_length": r["mean_accept_length"],
                       "miss_rounds": r["miss_rounds"],
                       "max_batch": max(r["decode_batch_sizes"]) if r["decode_batch_sizes"] else 0,
                       "max_active": max(r["decode_batch_sizes"]) if r["decode_batch_sizes"] else 0,
                       "timing_boundary": "end to end: admission, prefill, decode and release",
                       "input_sha256": digest}
                if ar is not None:
                    row["token_identical_to_ar"] = all(o.tokens == ar["outputs"][o.index] for o in r["outputs"])
                outs = [o.tokens for o in sorted(r["outputs"], key=lambda o: o.index)]
                if a.validate_hf and rep == 0:
                    if is_preset(a.target):
                        raise SystemExit("--validate-hf needs a target checkpoint directory, not a preset")
                    row["hf_greedy"] = hf_greedy_agreement(a.target, a.device, prompts, outs,
                                                           bud or [a.max_new_tokens] * len(prompts))
                scores = score_outputs(a, outs)
                if scores is not None:
                    row["accuracy"] = scores["accuracy"]
                    row["scored"] = scores["scored"]
                if ar_tps is not None:
                    row["ar_tps"] = row["baseline_tps"] = ar_tps
                    row["speedup"] = row["tps"] / ar_tps if ar_tps else None
                rows.append(row)
                print(row, flush=True)
    write_json(a.output_json, {"rows": rows, "config": {k: v for k, v in vars(a).items() if not k.startswith("eval_")},
                               "eval_sets": {n: d["eval"].get("eval_meta") for n, d in sets.items()},
                               "draft_validation": draft_check,
                               "runtime": runtime_metadata({"target": a.target, "draft": a.draft})})
    if a.validate and not all(r.get("token_identical_to_ar", True) for r in rows):
        raise RuntimeError("speculative output differs from AR decoding; see token_identical_to_ar in the JSON")
    return rows


if __name__ == "__main__":
    main()
