"""Synchronous multi-step denoising decode (reference: ``single/eval_sync.py``).

    python -m d3d_b200.cli.sync --verifier tiny-target --drafter tiny-drafter \\
        --block-size 8 --denoising-steps 2 --remasking-strategy low_confidence

Per prompt: draft a block in ``--denoising-steps`` drafter forwards, verify it
with one target forward, commit, repeat.  ``--use-kvcache`` keeps KV caches on
both models (the default here; ``--no-kvcache`` recomputes the prefix every
step, the reference's default).  ``--draft-device`` puts the drafter on its
own GPU.  Outputs: one row per prompt with its acceptance summary and timing,
an overall summary, evaluation-set accuracy where the set has answers.
"""
from __future__ import annotations

import argparse
import os
import json
import time

import torch

from ..engine.backends import TorchTarget
from ..engine.spec import EOS_DEFAULT, ar_generate
from ..engine.sync import sync_generate, sync_generate_nocache
from ..utils.io import label, write_json
from ..utils.metrics import AcceptanceStep, step_dicts, summarize_acceptance, summarize_timing
from ..utils.runtime import resolve_dtype, runtime_metadata
from .common import (add_data_args, add_model_args, check_devices, load_module, load_selected_prompts,
                     score_outputs)

DTYPES = ("auto", "bf16", "bfloat16", "fp16", "float16", "fp32", "float32")


def parser():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    add_model_args(p, "--verifier", "--drafter", dtypes=DTYPES)
    add_data_args(p)
    p.add_argument("--model-type", default=None, choices=["d3d"],
                   help="drafter family (read from the drafter's config when omitted; D3D drafters only)")
    p.add_argument("--drafter-tag", default=None, help="label recorded in the summary (default: the drafter name)")
    p.add_argument("--sample-index", type=int, default=None, help="decode only this example of the set")
    p.add_argument("--max-new-tokens", type=int, default=2048)
    p.add_argument("--draft-tokens", type=int, default=None,
                   help="drafted tokens per block for the acceptance summary (default: block size - 1)")
    p.add_argument("--block-size", type=int, default=32)
    p.add_argument("--denoising-steps", type=int, default=1)
    p.add_argument("--remasking-strategy", default="low_confidence", choices=["low_confidence", "dynamic"])
    p.add_argument("--confidence-threshold", type=float, default=0.9)
    p.add_argument("--attention-mask-mode", default="block_causal", choices=["causal", "block_causal"])
    p.add_argument("--temperature", type=float, default=0.0)
    p.add_argument("--proposal-top-k", type=int, default=0)
    p.add_argument("--proposal-top-p", type=float, default=1.0)
    p.add_argument("--target-top-k", type=int, default=0)
    p.add_argument("--target-top-p", type=float, default=1.0)
    p.add_argument("--verifier-device", default=None, help="target device (default: --device)")
    p.add_argument("--draft-device", default=None, help="drafter device (default: the verifier's)")
    p.add_argument("--eos-token-id", type=int, action="append", default=None,
                   help="stop token (repeatable; default: the tokenizer's EOS and Qwen3's end tokens)")
    cache = p.add_mutually_exclusive_group()
    cache.add_argument("--use-kvcache", dest="kvcache", action="store_true", default=True)
    cache.add_argument("--no-kvcache", dest="kvcache", action="store_false")
    p.add_argument("--target-attn-implementation", default=os.environ.get("TARGET_ATTN_IMPLEMENTATION"),
                   choices=["sdpa", "eager", "flash_attention_2"])
    p.add_argument("--draft-attn-implementation", default=os.environ.get("DRAFT_ATTN_IMPLEMENTATION"),
                   choices=["sdpa", "eager", "flash_attention_2"])
    p.add_argument("--collect-stage-timings", action="store_true",
                   help="per-verify records with wall and device time of each draft and verify")
    p.add_argument("--baseline", action="store_true", help="also run target-only AR decoding")
    p.add_argument("--output-json", default=None)
    p.add_argument("--summary-json", default=None, help="compact summary (one object)")
    p.add_argument("--verbose", action="store_true", help="print one line per prompt")
    return p


def _steps(st, n_out: int):
    """Acceptance steps of one request; emitted counts stop at the output's end
    (a stop token or the token budget)."""
    out, left = [], n_out
    for d, t, e, a, s in zip(st.draft_blocks, st.target_blocks, st.emitted_blocks, st.acceptance_lengths,
                             st.stopped):
        emitted = e[:max(left, 0)]
        left -= len(e)
        out.append(AcceptanceStep(accepted_draft_tokens=a - 1, accept_length=a, emitted_count=len(emitted),
                                  emitted_tokens=emitted, draft_tokens=d, target_tokens=t, stopped=s))
    return out


def _stop_ids(a):
    if a.eos_token_id:
        return sorted(set(a.eos_token_id))
    ids = set(EOS_DEFAULT)
    tok = getattr(a, "eval_tokenizer", None)
    if tok is not None and tok.eos_token_id is not None:
        ids.add(int(tok.eos_token_id))
    return sorted(ids)


def main(argv=None):
    a = parser().parse_args(argv)
    if a.block_size <= 1 and a.draft_tokens is None:
        raise SystemExit("--block-size must be > 1 when --draft-tokens is omitted")
    if a.draft_tokens is not None and a.draft_tokens <= 0:
        raise SystemExit("--draft-tokens must be positive")
    draft_tokens = a.draft_tokens if a.draft_tokens is not None else a.block_size - 1
    vdev = torch.device(a.verifier_device or a.device)
    ddev = torch.device(a.draft_device or vdev)
    check_devices(vdev, ddev)
    t = load_module(a.target, vdev, a.seed).eval()
    d = load_module(a.draft, ddev, a.seed, a.draft_layers, a.mask_token_id).eval()
    if not getattr(d.cfg, "d3d_draft", False) and d.cfg.mask_token_id is None:
        raise SystemExit("the drafter is not a D3D drafter (no mask token); --model-type d3d only")
    if a.dtype != "auto":
        t.to(resolve_dtype(a.dtype))
        d.to(resolve_dtype(a.dtype))
    attn = {"target": t.set_attn_implementation(a.target_attn_implementation),
            "draft": d.set_attn_implementation(a.draft_attn_implementation)}
    prompts = load_selected_prompts(a)
    stop = _stop_ids(a)
    ar = ar_generate(TorchTarget(t), prompts, a.max_new_tokens, eos=tuple(stop)) if a.baseline else None
    run = sync_generate if a.kvcache else sync_generate_nocache
    rows, all_steps, t0 = [], [], time.perf_counter()
    for i, pr in enumerate(prompts):
        st = run(t, d, pr, a.max_new_tokens, block_size=a.block_size, denoising_steps=a.denoising_steps,
                 remasking=a.remasking_strategy, threshold=a.confidence_threshold, temperature=a.temperature,
                 top_k=a.proposal_top_k, top_p=a.proposal_top_p, target_top_k=a.target_top_k,
                 target_top_p=a.target_top_p, mode=a.attention_mask_mode, stop_ids=stop, seed=a.seed + i,
                 collect_stage_timings=a.collect_stage_timings)
        steps = _steps(st, len(st.output_tokens))
        all_steps += steps
        n = len(st.output_tokens)
        nsteps = max(len(steps), 1)
        row = {"index": i, "input_tokens": st.num_input_tokens, "output_tokens": n, "tokens": st.output_tokens,
               "summary": summarize_acceptance(steps, draft_tokens), "steps": step_dicts(steps),
               "decode_elapsed_s": st.decode_elapsed_s,
               "tokens_per_s": n / st.decode_elapsed_s if st.decode_elapsed_s > 0 else 0.0,
               "time_per_output_token": st.time_per_output_token,
               "timing": {"draft_time": st.draft_s, "draft_gpu_time": st.draft_gpu_s,
                          "draft_prefill_time": st.draft_prefill_s, "verify_time": st.verify_s,
                          "verify_gpu_time": st.verify_gpu_s, "verifier_prefill_time": st.verifier_prefill_s,
                          "mean_draft_time_per_step": st.draft_s / nsteps,
                          "mean_draft_gpu_time_per_step": st.draft_gpu_s / nsteps,
                          "mean_verify_time_per_step": st.verify_s / nsteps,
                          "mean_verify_gpu_time_per_step": st.verify_gpu_s / nsteps,
                          "collect_stage_timings": a.collect_stage_timings},
               "stage_timings": st.stage_records,
               "matches_ar": (st.output_tokens == ar["outputs"][i]) if ar else None}
        rows.append(row)
        if a.verbose:
            print(json.dumps({"index": i, "output_tokens": n, "decode_elapsed_s": st.decode_elapsed_s,
                              **row["summary"]}), flush=True)
    elapsed = time.perf_counter() - t0
    scores = score_outputs(a, [r["tokens"] for r in rows])
    if scores is not None:
        for r, sc in zip(rows, scores.pop("rows")):
            r.update(pred=sc["pred"], gold=sc["gold"], correct=sc["correct"])
    summary = summarize_acceptance(all_steps, draft_tokens)
    summary.update(dataset=a.dataset, eval_set=getattr(a, "eval_meta", None), model_type="d3d",
                   drafter_tag=label(a.drafter_tag or a.draft), num_prompts=len(rows),
                   total_output_tokens=sum(r["output_tokens"] for r in rows), elapsed_s=elapsed,
                   **summarize_timing(rows, elapsed_s=elapsed), target_model=a.target, draft_model=a.draft,
                   draft_tokens=draft_tokens, block_size=a.block_size, denoising_steps=a.denoising_steps,
                   remasking_strategy=a.remasking_strategy, confidence_threshold=a.confidence_threshold,
                   attention_mask_mode=a.attention_mask_mode, max_new_tokens=a.max_new_tokens,
                   eos_token_ids=stop, temperature=a.temperature, proposal_top_k=a.proposal_top_k,
                   proposal_top_p=a.proposal_top_p, target_top_k=a.target_top_k, target_top_p=a.target_top_p,
                   use_kvcache=a.kvcache, collect_stage_timings=a.collect_stage_timings,
                   verifier_device=str(vdev), draft_device=str(ddev), attn_implementation=attn,
                   accuracy=None if scores is None else scores["accuracy"],
                   matches_ar=None if ar is None else all(r["matches_ar"] for r in rows))
    config = {k: v for k, v in vars(a).items() if not k.startswith("eval_")}
    write_json(a.output_json, {"summary": summary, "rows": rows, "accuracy": scores, "config": config,
                               "runtime": runtime_metadata({"target": a.target, "draft": a.draft})})
    compact = {k: summary[k] for k in ("dataset", "drafter_tag", "num_prompts", "total_output_tokens",
                                       "avg_accept_length", "avg_accepted_draft_tokens", "draft_accept_rate",
                                       "aggregate_decode_tokens_per_s", "mean_time_per_output_token",
                                       "accuracy", "matches_ar", "use_kvcache", "block_size", "denoising_steps")}
    write_json(a.summary_json, compact)
    print(json.dumps(compact, indent=2), flush=True)
    return rows


if __name__ == "__main__":
    main()
