"""Concurrent paged-KV serving benchmark (reference: ``serving/bench.py``).

    python -m d3d_b200.cli.serve --target qwen3-8b --draft d3d-1.7b --pages 4096 \\
        --concurrency 1,4,8,16 --max-new-tokens 512 --validate --output-json out/serve.json

Requests arrive all at once (closed loop); throughput is end to end
(prefill and admission included), as in the reference.
"""
from __future__ import annotations

import argparse
import time

from ..engine.controlled import ControlledAcceptance, rate_for_mean_accept
from ..engine.spec import DecodeConfig
from ..utils.io import write_json
from ..utils.runtime import check_paged_capacity
from .common import (add_data_args, add_model_args, build_engine, hf_greedy_agreement, is_preset,
                     load_prompts, score_outputs)


def parser():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    add_model_args(p, "--target", "--draft")
    add_data_args(p)
    p.add_argument("--pages", type=int, default=4096)
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--concurrency", default="1,4,8,16")
    p.add_argument("--max-new-tokens", type=int, default=256)
    p.add_argument("--max-new-tokens-range", default=None,
                   help="LO,HI: per-request output budgets drawn uniformly (seeded), e.g. 128,512")
    p.add_argument("--block-size", type=int, default=16)
    p.add_argument("--anchor-num", type=int, default=1)
    p.add_argument("--draft-microbatch", type=int, default=4)
    p.add_argument("--ignore-eos", action="store_true")
    p.add_argument("--backup", choices=["neural", "fast"], default="neural",
                   help="on a branch miss: redraft (neural) or verify a random block at once (fast)")
    p.add_argument("--validate", action="store_true", help="check token identity against AR decoding")
    p.add_argument("--validate-hf", action="store_true",
                   help="compare the outputs with transformers' greedy generate on the target checkpoint")
    p.add_argument("--baseline", action="store_true", help="AR baseline at each concurrency")
    p.add_argument("--controlled-accept-mean", type=float, default=None)
    p.add_argument("--output-json", default=None)
    return p


def main(argv=None):
    a = parser().parse_args(argv)
    conc = [int(c) for c in a.concurrency.split(",")]
    prompts = load_prompts(a)
    budgets = None
    if a.max_new_tokens_range:
        import random
        lo, hi = (int(x) for x in a.max_new_tokens_range.split(","))
        rng = random.Random(a.seed + 17)
        budgets = [rng.randint(lo, hi) for _ in prompts]
        a.max_new_tokens = hi
    check_paged_capacity([len(p) for p in prompts], a.max_new_tokens, conc, a.pages, a.page_size,
                         a.block_size, a.anchor_num)
    decode = DecodeConfig(block_size=a.block_size, anchor_num=a.anchor_num, max_new_tokens=a.max_new_tokens,
                          draft_microbatch=a.draft_microbatch, ignore_eos=a.ignore_eos, backup=a.backup)
    eng = build_engine(a, decode, max_seqs=max(conc), max_context=max(len(p) for p in prompts) + a.max_new_tokens + 64,
                       pages=a.pages)
    ar = None
    if a.validate or a.baseline or a.controlled_accept_mean is not None:
        ar = eng.generate_ar(prompts, concurrency=max(conc), max_new=budgets)
    ctl = None
    if a.controlled_accept_mean is not None:
        rate = rate_for_mean_accept(a.controlled_accept_mean, a.block_size)
        ctl = lambda i: ControlledAcceptance(prompts[i] + ar["outputs"][i], rate, int(eng.draft.vocab_size),
                                             seed=a.seed, stream=i)
    eng.generate(prompts[:1], max_new_tokens=16, controlled=ctl)           # warm-up
    rows = []
    for c in conc:
        r = eng.generate(prompts, concurrency=c, controlled=ctl, max_new=budgets)
        row = {"concurrency": c, "tps": r["tps"], "elapsed_s": r["elapsed_s"], "output_tokens": r["output_tokens"],
               "mean_accept_length": r["mean_accept_length"], "miss_rounds": r["miss_rounds"],
               "max_batch": max(r["decode_batch_sizes"]) if r["decode_batch_sizes"] else 0}
        if ar is not None:
            row["token_identical_to_ar"] = all(o.tokens == ar["outputs"][o.index] for o in r["outputs"])
        outs = [o.tokens for o in sorted(r["outputs"], key=lambda o: o.index)]
        if a.validate_hf:
            if is_preset(a.target):
                raise SystemExit("--validate-hf needs a target checkpoint directory, not a preset")
            row["hf_greedy"] = hf_greedy_agreement(a.target, a.device, prompts, outs,
                                                   budgets or [a.max_new_tokens] * len(prompts))
        scores = score_outputs(a, outs)
        if scores is not None:
            scores.pop("rows")
            row["accuracy"] = scores["accuracy"]
            row["scored"] = scores["scored"]
        if a.baseline:
            t0 = time.perf_counter()
            b = eng.generate_ar(prompts, concurrency=c, max_new=budgets)
            row["ar_tps"] = b["output_tokens"] / (time.perf_counter() - t0)
            row["speedup"] = row["tps"] / row["ar_tps"] if row["ar_tps"] else None
        rows.append(row)
        print(row, flush=True)
    write_json(a.output_json, {"rows": rows, "config": {k: v for k, v in vars(a).items() if not k.startswith("eval_")},
                               "eval_set": getattr(a, "eval_meta", None)})
    return rows


if __name__ == "__main__":
    main()
