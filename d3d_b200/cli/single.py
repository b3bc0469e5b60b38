"""Single-request asynchronous speculative decoding
(reference: ``single/eval_async_packed.py``, flags 1773-1812).

    python -m d3d_b200.cli.single --verifier qwen3-8b --drafter d3d-1.7b \\
        --block-size 16 --anchor-num 3 --max-new-tokens 512 --baseline \\
        --output-json out/result.json --summary-json out/summary.json
"""
from __future__ import annotations

import argparse
import os
import json
import statistics
import time

import torch

from ..engine.controlled import ControlledAcceptance, rate_for_mean_accept
from ..engine.spec import EOS_DEFAULT, DecodeConfig
from ..utils.io import label, write_json
from ..utils.runtime import runtime_metadata
from ..utils.metrics import headline, source_stats, steps_from_output, summarize_acceptance
from .common import (add_data_args, add_model_args, build_engine, check_devices, load_selected_prompts,
                     pin_host_threads, score_outputs)


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    add_model_args(p, "--verifier", "--drafter")
    add_data_args(p)
    p.add_argument("--max-new-tokens", type=int, default=2048)
    p.add_argument("--block-size", type=int, default=32)
    p.add_argument("--anchor-num", type=int, default=0,
                   help="non-primary anchors per rejection position (0: unanchored outcomes)")
    p.add_argument("--attention-mask-mode", choices=["causal", "block_causal"], default="block_causal")
    p.add_argument("--packed-accepted-counts", default="all",
                   help="'all' or a comma list of commit lengths to pre-draft")
    p.add_argument("--temperature", type=float, default=0.0)
    p.add_argument("--proposal-top-k", type=int, default=0)
    p.add_argument("--proposal-top-p", type=float, default=1.0)
    p.add_argument("--target-top-k", type=int, default=0, help="target sampling truncation (kernel path: 1..4)")
    p.add_argument("--target-top-p", type=float, default=1.0)
    p.add_argument("--collect-stage-timings", action="store_true",
                   help="host time per coordinator phase and device time per captured forward")
    p.add_argument("--ignore-eos", action="store_true")
    p.add_argument("--backup", choices=["neural", "fast", "fast_legacy"], default="neural",
                   help="on a branch miss: redraft (neural) or verify a random block at once (fast: the "
                        "block's drafts cover commit length 1 only; fast_legacy: every commit length)")
    p.add_argument("--fast-miss-anchors", type=int, default=0,
                   help="fast backup: anchors drafted after a random block (0 = --anchor-num)")
    p.add_argument("--baseline", action=argparse.BooleanOptionalAction, default=True,
                   help="also run target-only AR decoding (on the verifier) and report the speedup")
    p.add_argument("--controlled-accept-mean", type=float, default=None,
                   help="acceptance-controlled mode (needs --baseline's AR oracle)")
    p.add_argument("--warmup-new-tokens", type=int, default=32)
    p.add_argument("--output-json", default=None)
    p.add_argument("--summary-json", default=None)
    p.add_argument("--verifier-cpu-affinity", default=None, help="CPU list, e.g. 0-7 (host threads)")
    p.add_argument("--draft-cpu-affinity", default=None, help="CPU list, e.g. 8-15 (host threads)")
    p.add_argument("--verifier-device", default=None,
                   help="target device (default: --device); a different --draft-device runs the target in "
                        "its own process on its own GPU, linked over NVLink")
    p.add_argument("--draft-device", default=None, help="drafter device (default: the verifier's)")
    p.add_argument("--verifier-process", action="store_true",
                   help="run the target in its own process even on one device (CPU only)")
    p.add_argument("--model-type", default=None, choices=["d3d"], help="drafter family (D3D drafters only)")
    p.add_argument("--drafter-tag", default=None, help="label recorded in the summary (default: the drafter)")
    p.add_argument("--sample-index", type=int, default=None, help="decode only this example of the set")
    p.add_argument("--draft-tokens", type=int, default=None,
                   help="drafted tokens per block for the acceptance summary (default: block size - 1)")
    p.add_argument("--eos-token-id", type=int, action="append", default=None,
                   help="stop token (repeatable; default: Qwen3's end tokens)")
    p.add_argument("--verbose", action="store_true", help="print one line per prompt")
    p.add_argument("--async-blocks", type=int, default=1,
                   help="block-size chunks drafted per packed outcome; this engine drafts one (the reference's "
                        "default)")
    p.add_argument("--use-kvcache", action="store_true", default=True,
                   help="accepted for compatibility: the asynchronous engine always keeps paged KV caches")
    p.add_argument("--denoising-steps", type=int, default=1,
                   help="must be 1: asynchronous drafting is single-step (as in the reference)")
    p.add_argument("--remasking-strategy", default="low_confidence", choices=["low_confidence", "dynamic"],
                   help="no effect with one denoising step (recorded)")
    p.add_argument("--confidence-threshold", type=float, default=0.9, help="no effect with one denoising step")
    p.add_argument("--target-attn-implementation", default=os.environ.get("TARGET_ATTN_IMPLEMENTATION"),
                   choices=["sdpa", "eager", "flash_attention_2"],
                   help="PyTorch backends (CPU) only; the GPU path runs this framework's attention kernels")
    p.add_argument("--draft-attn-implementation", default=os.environ.get("DRAFT_ATTN_IMPLEMENTATION"),
                   choices=["sdpa", "eager", "flash_attention_2"])
    return p


def _check(a) -> None:
    if a.denoising_steps != 1:
        raise SystemExit("--denoising-steps must be 1: asynchronous drafting denoises in one step "
                         "(multi-step denoising runs in python -m d3d_b200.cli.sync)")
    if a.async_blocks != 1:
        raise SystemExit("--async-blocks: only 1 is supported (each packed outcome drafts one block)")
    if a.draft_tokens is not None and a.draft_tokens <= 0:
        raise SystemExit("--draft-tokens must be positive")


def _engine(a, decode, max_context):
    """Co-located engine, or the drafter here and the target in a verifier
    process when the devices differ (or ``--verifier-process``)."""
    vdev = torch.device(a.verifier_device or a.device)
    ddev = torch.device(a.draft_device or vdev)
    check_devices(vdev, ddev)
    if vdev == ddev and not a.verifier_process:
        a.device = str(vdev)
        eng = build_engine(a, decode, max_seqs=2, max_context=max_context)
        for be, impl in ((eng.target, a.target_attn_implementation), (eng.draft, a.draft_attn_implementation)):
            if impl is not None and hasattr(be, "model"):
                be.model.set_attn_implementation(impl)
        return eng, None
    if vdev == ddev and vdev.type == "cuda":
        raise SystemExit("--verifier-process on one GPU is not supported: the two processes' kernels would wait "
                         "on each other on one device; give --draft-device another GPU")
    from .pair import VerifierProcess
    vp = VerifierProcess(a, decode, max_seqs=2, max_context=max_context)
    return vp.engine, vp


def main(argv=None):
    a = parser().parse_args(argv)
    _check(a)
    pin_host_threads(a.verifier_cpu_affinity, a.draft_cpu_affinity)
    counts = None if a.packed_accepted_counts == "all" else tuple(int(x) for x in a.packed_accepted_counts.split(","))
    eos = tuple(sorted(set(a.eos_token_id))) if a.eos_token_id else EOS_DEFAULT
    decode = DecodeConfig(block_size=a.block_size, anchor_num=a.anchor_num, attention_mask_mode=a.attention_mask_mode,
                          max_new_tokens=a.max_new_tokens, temperature=a.temperature, top_k=a.proposal_top_k,
                          top_p=a.proposal_top_p, ignore_eos=a.ignore_eos, packed_accepted_counts=counts,
                          target_top_k=a.target_top_k, target_top_p=a.target_top_p, backup=a.backup,
                          fast_miss_anchors=a.fast_miss_anchors, eos=eos)
    prompts = load_selected_prompts(a)
    eng, vp = _engine(a, decode, max(len(p) for p in prompts) + a.max_new_tokens + 64)
    try:
        return _run(a, eng, prompts)
    finally:
        if vp is not None:
            vp.close()


def _run(a, eng, prompts):
    ar = None
    baseline_tps = None
    if a.baseline or a.controlled_accept_mean is not None:
        ar = eng.generate_ar(prompts)
        # decode-only, as the single-request metric: the prefill and its first token excluded
        dec_t = sum(ar["decode_s"])
        baseline_tps = sum(max(len(o) - 1, 0) for o in ar["outputs"]) / dec_t if dec_t > 0 else 0.0
    ctl = None
    if a.controlled_accept_mean is not None:
        rate = rate_for_mean_accept(a.controlled_accept_mean, a.block_size)
        vocab = int(eng.draft.vocab_size)      # drafter and target share the vocabulary
        ctl = lambda i: ControlledAcceptance(prompts[i] + ar["outputs"][i], rate, vocab, seed=a.seed, stream=i)
    if a.warmup_new_tokens:
        eng.generate(prompts[:1], max_new_tokens=a.warmup_new_tokens, controlled=ctl)
    if a.collect_stage_timings:
        eng.decoder.prof.enabled = True
        eng.decoder.prof.reset()
    per, outs = [], []
    draft_tokens = a.draft_tokens if a.draft_tokens is not None else a.block_size - 1
    t0 = time.perf_counter()
    for i, p in enumerate(prompts):
        s0 = time.perf_counter()
        r = eng.generate([p], max_new_tokens=a.max_new_tokens,
                         controlled=(lambda j, i=i: ctl(i)) if ctl else None)
        o = r["outputs"][0]
        outs.append(o)
        wall = time.perf_counter() - s0
        dt = o.decode_s             # after the prefill (which emits the first token) to the last token
        steps = steps_from_output(o.accepts, a.block_size, o.tokens)
        per.append({"index": i, "input_tokens": len(p), "output_tokens": len(o.tokens),
                    "decode_tokens": max(len(o.tokens) - 1, 0), "decode_elapsed_s": dt, "wall_s": wall,
                    "tokens_per_s": max(len(o.tokens) - 1, 0) / dt if dt > 0 else 0.0,
                    "tokens": o.tokens, "hits": o.hits, "recoveries": o.recoveries,
                    "summary": summarize_acceptance(steps, draft_tokens),
                    "sources": source_stats(o.sources, [a.block_size] * len(o.accepts), o.accepts),
                    "matches_ar": (o.tokens == ar["outputs"][i]) if ar else None})
        if a.verbose:
            print(json.dumps({"index": i, "output_tokens": len(o.tokens), "decode_elapsed_s": dt,
                              **per[-1]["summary"]}), flush=True)
    elapsed = time.perf_counter() - t0
    dec = sum(x["decode_tokens"] for x in per)
    dtime = sum(x["decode_elapsed_s"] for x in per)
    tps = dec / dtime if dtime > 0 else 0.0
    acc = statistics.fmean(s for x in per for s in [x["summary"]["avg_accept_length"]]) if per else 0.0
    summary = {"headline": headline(tps, baseline_tps or 0.0, acc), "elapsed_s": elapsed,
               "token_identical_to_ar": all(x["matches_ar"] for x in per) if ar else None,
               "drafter_tag": label(a.drafter_tag or a.draft), "draft_tokens": draft_tokens, "model_type": "d3d",
               "layout": "verifier_process" if hasattr(eng.target, "links") else "colocated"}
    hits = sum(x["hits"] for x in per)
    recov = sum(x["recoveries"] for x in per)
    verifies = sum(x["summary"]["num_verify_steps"] for x in per)
    all_src = [src for o in outs for src in o.sources]
    all_acc = [n for o in outs for n in o.accepts]
    summary["async"] = {"verify_steps": verifies, "packed_outcome_hits": hits, "redraft_steps": recov,
                        "packed_hit_rate": hits / max(1, hits + recov),
                        "all_pass_steps": sum(1 for n in all_acc if n == a.block_size),
                        "sources": source_stats(all_src, [a.block_size] * len(all_acc), all_acc)}
    if a.collect_stage_timings:
        summary["stage_timings"] = eng.decoder.prof.summary()
    scores = score_outputs(a, [x["tokens"] for x in per])
    if scores is not None:
        for x, r in zip(per, scores.pop("rows")):
            x.update(pred=r["pred"], gold=r["gold"], correct=r["correct"])
        summary["accuracy"] = scores
    summary["config"] = {k: v for k, v in vars(a).items() if not k.startswith("eval_")}
    write_json(a.output_json, {"summary": summary, "per_prompt": per,
                               "runtime": runtime_metadata({"target": a.target, "draft": a.draft})})
    write_json(a.summary_json, summary)
    print(summary["headline"])
    return summary


if __name__ == "__main__":
    main()
