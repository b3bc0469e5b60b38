"""Synchronous multi-step denoising decode (reference: ``single/eval_sync.py``).

    python -m d3d_b200.cli.sync --verifier tiny-target --drafter tiny-drafter \\
        --block-size 8 --denoising-steps 2 --remasking-strategy low_confidence
"""
from __future__ import annotations

import argparse

from ..engine.spec import ar_generate
from ..engine.backends import TorchTarget
from ..engine.sync import sync_generate, sync_generate_nocache
from ..utils.io import write_json
from ..utils.metrics import steps_from_output, summarize_acceptance
from .common import add_data_args, add_model_args, load_module, load_prompts, score_outputs


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    add_model_args(p, "--verifier", "--drafter")
    add_data_args(p)
    p.add_argument("--max-new-tokens", type=int, default=128)
    p.add_argument("--block-size", type=int, default=32)
    p.add_argument("--denoising-steps", type=int, default=1)
    p.add_argument("--remasking-strategy", default="low_confidence", choices=["low_confidence", "dynamic"])
    p.add_argument("--confidence-threshold", type=float, default=0.9)
    p.add_argument("--attention-mask-mode", default="block_causal", choices=["causal", "block_causal"])
    p.add_argument("--temperature", type=float, default=0.0)
    p.add_argument("--proposal-top-k", type=int, default=0)
    p.add_argument("--no-kvcache", action="store_true")
    p.add_argument("--baseline", action="store_true")
    p.add_argument("--output-json", default=None)
    a = p.parse_args(argv)
    t = load_module(a.target, a.device, a.seed).eval()
    d = load_module(a.draft, a.device, a.seed, a.draft_layers, a.mask_token_id).eval()
    prompts = load_prompts(a)
    ar = ar_generate(TorchTarget(t), prompts, a.max_new_tokens) if a.baseline else None
    rows = []
    for i, pr in enumerate(prompts):
        kw = dict(block_size=a.block_size, denoising_steps=a.denoising_steps, remasking=a.remasking_strategy,
                  threshold=a.confidence_threshold, mode=a.attention_mask_mode)
        st = (sync_generate_nocache(t, d, pr, a.max_new_tokens, **kw) if a.no_kvcache else
              sync_generate(t, d, pr, a.max_new_tokens, temperature=a.temperature, top_k=a.proposal_top_k, **kw))
        rows.append({"index": i, "tokens": st.output_tokens, "decode_elapsed_s": st.decode_elapsed_s,
                     "summary": summarize_acceptance(steps_from_output(st.acceptance_lengths, a.block_size,
                                                                       st.output_tokens), a.block_size - 1),
                     "matches_ar": (st.output_tokens == ar["outputs"][i]) if ar else None})
    scores = score_outputs(a, [r["tokens"] for r in rows])
    if scores is not None:
        for r, sc in zip(rows, scores.pop("rows")):
            r.update(pred=sc["pred"], gold=sc["gold"], correct=sc["correct"])
    write_json(a.output_json, {"rows": rows, "accuracy": scores,
                               "config": {k: v for k, v in vars(a).items() if not k.startswith("eval_")}})
    print({"samples": len(rows), "matches_ar": [r["matches_ar"] for r in rows]})
    return rows


if __name__ == "__main__":
    main()
