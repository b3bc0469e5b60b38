"""Breakdown of one speculative decode step on the headline configuration.

    python -m d3d_b200.benchmarks.step_profile [--requests 2] [--max-new 256]

Runs a few controlled-acceptance requests and prints host time per phase of
the coordinator and device time of each captured forward (CUDA events on the
forward's own stream).
"""
from __future__ import annotations

import argparse
import json
import random
import time

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--requests", type=int, default=2)
    ap.add_argument("--max-new", type=int, default=256)
    ap.add_argument("--accept-mean", type=float, default=5.0)
    ap.add_argument("--anchor-num", type=int, default=1)
    ap.add_argument("--draft-layers", type=int, default=28)
    ap.add_argument("--two-streams", action="store_true")
    a = ap.parse_args()
    from d3d_b200 import config as C
    from d3d_b200.api import D3DEngine
    from d3d_b200.engine.controlled import ControlledAcceptance, rate_for_mean_accept
    from d3d_b200.engine.spec import DecodeConfig
    from d3d_b200.models.fast import FastWeights

    tw = FastWeights.random(C.qwen3_8b(), seed=0)
    dw = FastWeights.random(C.d3d_1p7b(num_layers=a.draft_layers), seed=0)
    dec = DecodeConfig(block_size=16, anchor_num=a.anchor_num, max_new_tokens=a.max_new)
    eng = D3DEngine.from_weights(tw, dw, dec, max_seqs=4, max_context=512 + a.max_new + 32,
                                 shared_stream=not a.two_streams)
    rng = random.Random(0)
    prompts = [[rng.randrange(0, 151643) for _ in range(rng.randint(128, 512))]
               for _ in range(a.requests + 1)]
    ar = eng.generate_ar(prompts)["outputs"]
    rate = rate_for_mean_accept(a.accept_mean, 16)
    ctl = lambda i: ControlledAcceptance(prompts[i] + ar[i], rate, 151936, stream=i)
    eng.generate(prompts[:1], controlled=ctl)          # warm-up / graph capture
    eng.decoder.prof.enabled = True
    eng.decoder.prof.reset()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    outs = []
    for i in range(1, a.requests + 1):
        r = eng.generate([prompts[i]], controlled=lambda j, i=i: ctl(i))
        outs += r["outputs"]
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    steps = sum(len(o.accepts) for o in outs)
    toks = sum(len(o.tokens) for o in outs)
    summ = eng.decoder.prof.summary()
    summ.update(wall_s=round(wall, 3), steps=steps, tokens=toks, tps=round(toks / wall, 1),
                ms_per_step=round(1e3 * wall / max(1, steps), 3),
                recoveries=sum(o.recoveries for o in outs), hits=sum(o.hits for o in outs))
    print(json.dumps(summ, indent=1))


if __name__ == "__main__":
    main()
