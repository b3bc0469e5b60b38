#!/usr/bin/env python3
"""Headline benchmark: decode tokens/s (and speedup vs AR) of asynchronous
speculative decoding, Qwen3-8B target + 1.7B-layout D3D drafter, bf16,
random-init weights, synthetic seeded prompts, acceptance-controlled drafts.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One *step* is one request decoded end to end at concurrency 1 (prompt of
128-512 random non-special tokens -> 512 new tokens, greedy): prefill, the
async draft/verify loop, output read back.  W requests are decoded untimed
(CUDA-graph capture, allocator warm-up), then exactly K requests are timed
with CUDA events between two barrier+synchronize points; the device time is
the max over ranks and ``value`` is the whole-job token rate (every rank
decodes its own requests: weak scaling).  The same K requests are decoded
target-only (AR) on the same kernels for the speedup, and once more through
the public API with wall-clock timing for the ``e2e`` figure.

For N > 1 launch with ``python -m torch.distributed.run --nproc-per-node N``.
"""
from __future__ import annotations

import argparse
import json
import os
import random
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BASELINE_TPS = 501.60   # published headline: SGLang Hybrid aggregate TPS, 2xH800 (README.md:251-253 of the reference)
BASELINE_NOTE = ("vs_baseline divides by 501.60 tok/s, the reference's published SGLang-Hybrid aggregate over 7 real "
                 "datasets with a trained drafter and natural acceptance on 2xH800: a different workload, acceptance "
                 "regime, GPU count and GPU; the same-box comparison is the --impl reference arm")
METRIC = "decode tokens/s + speedup vs AR, Qwen3-8B target/1.7B draft, concurrency 1–8"
EOS = (151643, 151645)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=4)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--max-new-tokens", type=int, default=512)
    p.add_argument("--accept-mean", type=float, default=5.0,
                   help="controlled mean accepted length; 0 = natural acceptance (no injection)")
    p.add_argument("--block-size", type=int, default=16)
    p.add_argument("--anchor-num", type=int, default=1)
    p.add_argument("--concurrency", type=int, default=1)
    p.add_argument("--prompt-min", type=int, default=128)
    p.add_argument("--prompt-max", type=int, default=512)
    p.add_argument("--target", default="qwen3-8b")
    p.add_argument("--draft-layers", type=int, default=28)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--json-out", default=None)
    p.add_argument("--watchdog-s", type=float, default=1500.0,
                   help="N>1: dump stacks and exit a rank still running after this many seconds")
    p.add_argument("--layout", choices=["auto", "replica", "disagg", "tp"], default="auto",
                   help="N>1: 'tp' = target tensor-parallel over N/2 GPUs + one drafter per other GPU; "
                        "'disagg' = pairs of GPUs (target GPU + drafter GPU, NVLink handoff); "
                        "'replica' = target and drafter co-located on every GPU; "
                        "auto = replica for N=1, disagg pairs for even N (the tp layout's bench run at "
                        "N=4 stopped during target set-up, before serving, in its last run)")
    return p.parse_args()


from d3d_b200.utils.benchutil import ClockSampler, barrier, dist_max, dist_setup, dist_sum  # noqa: E402


def make_prompts(n, lo, hi, seed):
    rng = random.Random(seed)
    return [[rng.randrange(0, 151643) for _ in range(rng.randint(lo, hi))] for _ in range(n)]


# ------------------------------------------------------------------- ours
def run_ours(args, rank, world, local):
    import torch
    from d3d_b200 import config as C
    from d3d_b200.api import D3DEngine
    from d3d_b200.engine.controlled import ControlledAcceptance, rate_for_mean_accept
    from d3d_b200.engine.spec import DecodeConfig
    from d3d_b200.models.fast import FastWeights
    from d3d_b200.utils import launches

    dev = torch.device("cuda", local)
    tcfg = C.PRESETS[args.target]()
    dcfg = C.d3d_1p7b(num_layers=args.draft_layers)
    tw = FastWeights.random(tcfg, seed=args.seed, device=dev)
    dw = FastWeights.random(dcfg, seed=args.seed, device=dev)
    decode = DecodeConfig(block_size=args.block_size, anchor_num=args.anchor_num,
                          attention_mask_mode="causal", max_new_tokens=args.max_new_tokens,
                          eos=EOS)
    max_ctx = args.prompt_max + args.max_new_tokens + 2 * args.block_size
    eng = D3DEngine.from_weights(tw, dw, decode, max_seqs=max(4, args.concurrency),
                                 max_context=max_ctx, device=dev)
    n = args.warmup + args.steps
    prompts = make_prompts(n * args.concurrency, args.prompt_min, args.prompt_max,
                           seed=1000 + 7919 * rank + args.seed)
    groups = [prompts[i * args.concurrency:(i + 1) * args.concurrency] for i in range(n)]

    # --- AR oracle (also the AR baseline: same kernels, target only)
    ar_out = {}
    ar_time = 0.0
    ar_tokens = 0
    for gi, g in enumerate(groups):
        if gi == args.warmup:
            barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0.record()
        r = eng.generate_ar(g, concurrency=args.concurrency)
        t1.record()
        torch.cuda.synchronize()
        for j, o in enumerate(r["outputs"]):
            ar_out[gi * args.concurrency + j] = o
        if gi >= args.warmup:
            ar_time += t0.elapsed_time(t1) / 1e3
            ar_tokens += sum(len(o) for o in r["outputs"])
    rate = rate_for_mean_accept(args.accept_mean, args.block_size) if args.accept_mean > 0 else 0.0

    def ctl_for(base):
        if args.accept_mean <= 0:     # natural acceptance: the drafter's own proposals
            return None
        def ctl(i):
            k = base + i
            return ControlledAcceptance(oracle=prompts[k] + ar_out[k], rate=rate,
                                        vocab_size=tcfg.vocab_size, seed=args.seed, stream=k,
                                        exclude=(151669,) + EOS)
        return ctl

    # --- warm-up
    for gi in range(args.warmup):
        eng.generate(groups[gi], concurrency=args.concurrency, controlled=ctl_for(gi * args.concurrency))

    # --- timed region
    barrier()
    launches.reset()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    tokens = 0
    accepts = []
    ident = True
    with ClockSampler(local) as clk:
        barrier()
        ev0.record()
        for gi in range(args.warmup, n):
            r = eng.generate(groups[gi], concurrency=args.concurrency,
                             controlled=ctl_for(gi * args.concurrency))
            for j, o in enumerate(r["outputs"]):
                tokens += len(o.tokens)
                accepts.extend(o.accepts)
                ident &= o.tokens == ar_out[gi * args.concurrency + j]
        torch.cuda.synchronize()
        ev1.record()
        barrier()
    n_launch = launches.count()
    dev_s = ev0.elapsed_time(ev1) / 1e3

    # --- end-to-end pass through the public API (pinned inputs, host outputs)
    e2e = None
    if not args.no_e2e:
        pinned = [[torch.tensor(p, dtype=torch.int64).pin_memory() for p in g] for g in groups]
        bi = bo = 0
        e2e_tokens = 0
        barrier()
        w0 = time.perf_counter()
        for gi in range(args.warmup, n):
            r = eng.generate([p.tolist() for p in pinned[gi]], concurrency=args.concurrency,
                             controlled=ctl_for(gi * args.concurrency))
            for o in r["outputs"]:
                e2e_tokens += len(o.tokens)
                bo += 8 * len(o.tokens)
            bi += sum(8 * p.numel() for p in pinned[gi])
        barrier()
        w1 = time.perf_counter()
        e2e_s = dist_max(w1 - w0)
        e2e = {"value": dist_sum(e2e_tokens) / e2e_s, "unit": "tokens/s",
               "h2d_bytes_per_step": bi / args.steps, "d2h_bytes_per_step": bo / args.steps,
               "timing": "wall clock around the public D3DEngine.generate calls"}

    dev_s_max = dist_max(dev_s)
    all_tokens = dist_sum(tokens)
    ar_s_max = dist_max(ar_time)
    ar_all = dist_sum(ar_tokens)
    value = all_tokens / dev_s_max
    ar_value = ar_all / ar_s_max if ar_s_max > 0 else None
    ident_all = dist_sum(1.0 if ident else 0.0) == world
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * dev_s_max / args.steps, 3),
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(value / BASELINE_TPS, 4), "vs_baseline_note": BASELINE_NOTE, "dtype": "bf16",
        "data": "synthetic seeded random-token prompts, random-init weights (seed 0), "
                "acceptance-controlled drafts",
        "config": {"model": "Qwen3-8B-layout target + D3D-1.7B-layout drafter (28 layers, block 16)",
                   "global_batch": args.concurrency * world, "seq_len": f"prompt {args.prompt_min}-"
                   f"{args.prompt_max} + {args.max_new_tokens} new",
                   "parallelism": f"replica per GPU x{world} (target + drafter co-located, one stream)",
                   "concurrency": args.concurrency, "anchor_num": args.anchor_num,
                   "controlled_accept_mean": args.accept_mean,
                   "measured_accept_mean": round(statistics.fmean(accepts), 3) if accepts else None,
                   "l2": "inputs larger than L2: every verify streams ~16 GB of target weights",
                   "step": "one request, prefill through last token"},
        "ar_tokens_per_s": round(ar_value, 2) if ar_value else None,
        "speedup_vs_ar": round(value / ar_value, 3) if ar_value else None,
        "token_identical_to_ar": bool(ident_all),
        "gpu_launches": int(dist_sum(n_launch)),
        "clocks": clk.summary(),
        "e2e": e2e,
        "impl": "ours",
    }
    return out


# ------------------------------------------------------- ours, disaggregated
def run_disagg(args, rank, world, local):
    """Pairs of GPUs: even rank = target server, odd rank = drafter + coordinator.
    Each pair decodes its own requests (concurrency ``args.concurrency``)."""
    import torch
    import torch.distributed as dist
    from d3d_b200 import config as C
    from d3d_b200.api import D3DEngine, open_pair_link, target_server
    from d3d_b200.engine.controlled import ControlledAcceptance, rate_for_mean_accept
    from d3d_b200.engine.spec import DecodeConfig, ar_generate
    from d3d_b200.models.fast import FastWeights
    from d3d_b200.utils import launches

    dev = torch.device("cuda", local)
    is_target = rank % 2 == 0
    pair, pairs = rank // 2, world // 2
    link = open_pair_link(rank ^ 1, dev)
    tcfg = C.PRESETS[args.target]()
    dcfg = C.d3d_1p7b(num_layers=args.draft_layers)
    decode = DecodeConfig(block_size=args.block_size, anchor_num=args.anchor_num,
                          attention_mask_mode="causal", max_new_tokens=args.max_new_tokens, eos=EOS)
    max_ctx = args.prompt_max + args.max_new_tokens + 2 * args.block_size
    n = args.warmup + args.steps
    cc = args.concurrency
    prompts = make_prompts(n * cc, args.prompt_min, args.prompt_max, seed=1000 + 7919 * pair + args.seed)
    groups = [prompts[i * cc:(i + 1) * cc] for i in range(n)]
    ar_out, ar_time, ar_tokens = {}, 0.0, 0
    if is_target:
        srv = target_server(FastWeights.random(tcfg, seed=args.seed, device=dev), link,
                            max_seqs=max(4, cc), max_context=max_ctx, device=dev)
        # AR oracle and AR baseline: target only, on this GPU, same kernels
        for gi, g in enumerate(groups):
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            t0.record()
            r = ar_generate(srv.be, g, args.max_new_tokens, eos=EOS, concurrency=cc)
            torch.cuda.synchronize()
            t1.record()
            torch.cuda.synchronize()
            for j, o in enumerate(r["outputs"]):
                ar_out[gi * cc + j] = o
            if gi >= args.warmup:
                ar_time += t0.elapsed_time(t1) / 1e3
                ar_tokens += sum(len(o) for o in r["outputs"])
    else:
        eng = D3DEngine.from_remote_target(FastWeights.random(dcfg, seed=args.seed, device=dev), link,
                                           tcfg.hidden_size, decode, max_seqs=max(4, cc),
                                           max_context=max_ctx, device=dev)
    shared = [None] * world
    dist.all_gather_object(shared, ar_out if is_target else None)
    ar_out = shared[2 * pair]
    rate = rate_for_mean_accept(args.accept_mean, args.block_size) if args.accept_mean > 0 else 0.0

    def ctl_for(base):
        if args.accept_mean <= 0:     # natural acceptance: the drafter's own proposals
            return None
        def ctl(i):
            k = base + i
            return ControlledAcceptance(oracle=prompts[k] + ar_out[k], rate=rate, vocab_size=tcfg.vocab_size,
                                        seed=args.seed, stream=k, exclude=(151669,) + EOS)
        return ctl

    def phase(ids, check=None):
        """The drafter decodes groups ``ids``; the target serves until told to stop."""
        if is_target:
            srv.serve()
            return
        for gi in ids:
            r = eng.generate(groups[gi], concurrency=cc, controlled=ctl_for(gi * cc))
            if check is not None:
                check(gi, r)
        eng.close()

    phase(range(args.warmup))
    tokens, accepts, ident, dsteps = 0, [], True, 0

    def check(gi, r):
        nonlocal tokens, ident, dsteps
        dsteps += r["steps"]
        for j, o in enumerate(r["outputs"]):
            tokens += len(o.tokens)
            accepts.extend(o.accepts)
            ident &= o.tokens == ar_out[gi * cc + j]

    # device timers (CUDA events around each captured forward) for the
    # exposed-handoff figure: step time minus the slower of verify and draft
    from d3d_b200.utils.timing import StepProfiler
    prof = StepProfiler(True)
    if is_target:
        srv.be.prof = prof
    else:
        eng.decoder.prof = prof
        for be in (eng.decoder.t, eng.decoder.d):
            if hasattr(be, "prof"):
                be.prof = prof

    barrier()
    launches.reset()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        ev0.record()
        phase(range(args.warmup, n), check)
        torch.cuda.synchronize()
        ev1.record()
        barrier()
    n_launch = launches.count()
    dev_s = ev0.elapsed_time(ev1) / 1e3
    if is_target:
        srv.be.prof = StepProfiler(False)
    else:
        eng.decoder.prof = StepProfiler(False)
        for be in (eng.decoder.t, eng.decoder.d):
            if hasattr(be, "prof"):
                be.prof = eng.decoder.prof

    def _busiest(prefix):
        dev = prof.summary()["device"]
        rows = [v for k, v in dev.items() if k.startswith(prefix)]
        return max(rows, key=lambda v: v["n"])["ms_each"] if rows else 0.0

    mine = (_busiest("verify_") if is_target else _busiest("draft_"), dsteps, dev_s)
    timers = [None] * world
    dist.all_gather_object(timers, mine)
    verify_ms = statistics.fmean(t[0] for i, t in enumerate(timers) if i % 2 == 0)
    draft_ms = statistics.fmean(t[0] for i, t in enumerate(timers) if i % 2 == 1)
    step_ms = statistics.fmean(1e3 * t[2] / max(1, t[1]) for i, t in enumerate(timers) if i % 2 == 1)
    handoff = {"step_ms": round(step_ms, 3), "verify_ms": round(verify_ms, 3), "draft_ms": round(draft_ms, 3),
               "exposed_ms": round(step_ms - max(verify_ms, draft_ms), 3),
               "note": "per decode step: step time minus the slower of the concurrent verify and packed "
                       "draft forwards (CUDA events), averaged over pairs"}

    e2e = None
    if not args.no_e2e:
        pinned = [[torch.tensor(p, dtype=torch.int64).pin_memory() for p in g] for g in groups]
        e2e_tokens, bi, bo = 0, 0, 0

        def e2e_check(gi, r):
            nonlocal e2e_tokens, bo
            for o in r["outputs"]:
                e2e_tokens += len(o.tokens)
                bo += 8 * len(o.tokens)

        barrier()
        w0 = time.perf_counter()
        if is_target:
            srv.serve()
        else:
            for gi in range(args.warmup, n):
                r = eng.generate([p.tolist() for p in pinned[gi]], concurrency=cc, controlled=ctl_for(gi * cc))
                e2e_check(gi, r)
                bi += sum(8 * p.numel() for p in pinned[gi])
            eng.close()
        barrier()
        w1 = time.perf_counter()
        e2e_s = dist_max(w1 - w0)
        e2e = {"value": dist_sum(e2e_tokens) / e2e_s, "unit": "tokens/s",
               "h2d_bytes_per_step": dist_sum(bi) / args.steps / pairs,
               "d2h_bytes_per_step": dist_sum(bo) / args.steps / pairs,
               "timing": "wall clock around the public D3DEngine.generate calls (drafter ranks) "
                         "while the target ranks serve"}

    dev_s_max = dist_max(dev_s)
    all_tokens = dist_sum(tokens)
    ar_s_max = dist_max(ar_time)
    ar_all = dist_sum(ar_tokens)
    value = all_tokens / dev_s_max
    ar_value = ar_all / ar_s_max if ar_s_max > 0 else None
    ident_all = dist_sum(0.0 if (not is_target and not ident) else 1.0) == world
    acc_all = [None] * world
    dist.all_gather_object(acc_all, accepts)
    accepts = [a for lst in acc_all for a in lst]
    n_launch_all = int(dist_sum(n_launch))
    link.close()
    return {
        "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * dev_s_max / args.steps, 3),
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(value / BASELINE_TPS, 4), "vs_baseline_note": BASELINE_NOTE, "dtype": "bf16",
        "data": "synthetic seeded random-token prompts, random-init weights (seed 0), "
                "acceptance-controlled drafts",
        "config": {"model": "Qwen3-8B-layout target + D3D-1.7B-layout drafter (28 layers, block 16)",
                   "global_batch": cc * pairs, "seq_len": f"prompt {args.prompt_min}-"
                   f"{args.prompt_max} + {args.max_new_tokens} new",
                   "parallelism": f"disaggregated pairs x{pairs}: target GPU + drafter GPU per request "
                                  "stream, NVLink mailbox handoff (fused accept+send kernel)",
                   "concurrency": cc, "anchor_num": args.anchor_num,
                   "controlled_accept_mean": args.accept_mean,
                   "measured_accept_mean": round(statistics.fmean(accepts), 3) if accepts else None,
                   "l2": "inputs larger than L2: every verify streams ~16 GB of target weights",
                   "step": "one request per pair, prefill through last token"},
        "ar_tokens_per_s": round(ar_value, 2) if ar_value else None,
        "speedup_vs_ar": round(value / ar_value, 3) if ar_value else None,
        "speedup_note": "per pair (2 GPUs) vs target-only AR on one GPU, as the reference reports it",
        "handoff": handoff,
        "token_identical_to_ar": bool(ident_all),
        "gpu_launches": n_launch_all,
        "clocks": clk.summary(),
        "e2e": e2e,
        "impl": "ours",
    }


# --------------------------------------- ours, tensor-parallel target + drafters
def run_tp_layout(args, rank, world, local):
    """N GPUs: the target tensor-parallel over ranks 0..T-1 (T = N/2) and one
    drafter + coordinator on each of the other D = N - T ranks, each decoding
    its own request stream (concurrency ``args.concurrency`` per drafter).
    Every drafter sends its requests to every target rank over NVLink
    mailboxes; the target batches the drafters' verifies into one forward per
    round and rank 0's fused accept+send kernel answers each drafter in its
    own mailbox.  Weak scaling: per-GPU work is fixed as N grows."""
    import torch
    import torch.distributed as dist
    from d3d_b200 import config as C
    from d3d_b200.api import D3DEngine
    from d3d_b200.engine.controlled import ControlledAcceptance, rate_for_mean_accept
    from d3d_b200.engine.disagg import DEFAULT_SLOT_BYTES, BatchedTargetServer
    from d3d_b200.engine.fast import FastTarget
    from d3d_b200.engine.spec import DecodeConfig, ar_generate
    from d3d_b200.models.fast import FastWeights
    from d3d_b200.parallel.p2p import Link
    from d3d_b200.parallel.tp import TPGroup, random_shard
    from d3d_b200.utils import launches
    from d3d_b200.utils.timing import StepProfiler

    T = world // 2
    D = world - T
    dev = torch.device("cuda", local)
    is_target = rank < T
    me = rank - T                      # drafter index on drafter ranks
    tp_group = dist.new_group(list(range(T)))
    pair = {(t, d): dist.new_group([t, T + d]) for t in range(T) for d in range(D)}
    tcfg = C.PRESETS[args.target]()
    dcfg = C.d3d_1p7b(num_layers=args.draft_layers)
    decode = DecodeConfig(block_size=args.block_size, anchor_num=args.anchor_num,
                          attention_mask_mode="causal", max_new_tokens=args.max_new_tokens, eos=EOS)
    max_ctx = args.prompt_max + args.max_new_tokens + 2 * args.block_size
    n = args.warmup + args.steps
    cc = args.concurrency
    prompts = [make_prompts(n * cc, args.prompt_min, args.prompt_max, seed=1000 + 7919 * d + args.seed)
               for d in range(D)]
    groups = [[p[i * cc:(i + 1) * cc] for i in range(n)] for p in prompts]
    ar_out, ar_time, ar_tokens = {}, 0.0, 0
    if is_target:
        grp = TPGroup(rank, T, dev, group=tp_group, num_layers=tcfg.num_hidden_layers) if T > 1 else None
        w = random_shard(tcfg, T, rank, seed=args.seed, device=dev) if T > 1 else \
            FastWeights.random(tcfg, seed=args.seed, device=dev)
        links = [Link(1, DEFAULT_SLOT_BYTES, dev, group=pair[(rank, d)]) for d in range(D)]
        seqs = max(4, D * cc)
        tgt = FastTarget(w, pages=seqs * (max_ctx + 64 + 16) // 16 + 8, max_seqs=seqs, max_context=max_ctx,
                         device=dev, tp=grp)
        # AR oracle and AR baseline: target only on the T ranks, every drafter's
        # requests of a step decoded together (batch-invariant kernels)
        for gi in range(n):
            batch = [p for d in range(D) for p in groups[d][gi]]
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            r = ar_generate(tgt, batch, args.max_new_tokens, eos=EOS, concurrency=D * cc)
            e1.record()
            torch.cuda.synchronize()
            for j, o in enumerate(r["outputs"]):
                ar_out[(j // cc, gi * cc + j % cc)] = o
            if gi >= args.warmup:
                ar_time += e0.elapsed_time(e1) / 1e3
                ar_tokens += sum(len(o) for o in r["outputs"])
        srv = BatchedTargetServer(tgt, links, replies="all" if rank == 0 else "ack")
    else:
        links = [Link(0, DEFAULT_SLOT_BYTES, dev, group=pair[(t, me)]) for t in range(T)]
        eng = D3DEngine.from_remote_target(FastWeights.random(dcfg, seed=args.seed, device=dev), links,
                                           tcfg.hidden_size, decode, max_seqs=max(4, cc), max_context=max_ctx,
                                           device=dev)
    shared = [None] * world
    dist.all_gather_object(shared, ar_out if rank == 0 else None)
    ar_out = shared[0]
    rate = rate_for_mean_accept(args.accept_mean, args.block_size) if args.accept_mean > 0 else 0.0

    def ctl_for(base):
        if args.accept_mean <= 0:     # natural acceptance: the drafter's own proposals
            return None
        def ctl(i):
            k = base + i
            return ControlledAcceptance(oracle=prompts[me][k] + ar_out[(me, k)], rate=rate,
                                        vocab_size=tcfg.vocab_size, seed=args.seed, stream=7919 * me + k,
                                        exclude=(151669,) + EOS)
        return ctl

    def phase(ids, check=None, pinned=None):
        if is_target:
            srv.serve()
            return
        for gi in ids:
            g = groups[me][gi] if pinned is None else [p.tolist() for p in pinned[gi]]
            r = eng.generate(g, concurrency=cc, controlled=ctl_for(gi * cc))
            if check is not None:
                check(gi, r)
        eng.close()

    phase(range(args.warmup))
    tokens, accepts, ident, dsteps = 0, [], True, 0

    def check(gi, r):
        nonlocal tokens, ident, dsteps
        dsteps += r["steps"]
        for j, o in enumerate(r["outputs"]):
            tokens += len(o.tokens)
            accepts.extend(o.accepts)
            ident &= o.tokens == ar_out[(me, gi * cc + j)]

    prof = StepProfiler(True)
    if is_target:
        tgt.prof = prof
    else:
        eng.decoder.prof = prof
        eng.draft.prof = prof
    barrier()
    launches.reset()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        ev0.record()
        phase(range(args.warmup, n), check)
        torch.cuda.synchronize()
        ev1.record()
        barrier()
    n_launch = launches.count()
    dev_s = ev0.elapsed_time(ev1) / 1e3
    off = StepProfiler(False)
    if is_target:
        tgt.prof = off
    else:
        eng.decoder.prof = off
        eng.draft.prof = off

    def _busiest(prefix):
        rows = [v for k, v in prof.summary()["device"].items() if k.startswith(prefix)]
        return max(rows, key=lambda v: v["n"])["ms_each"] if rows else 0.0

    mine = (_busiest("verify_") if is_target else _busiest("draft_"), dsteps, dev_s)
    timers = [None] * world
    dist.all_gather_object(timers, mine)
    verify_ms = timers[0][0]
    draft_ms = statistics.fmean(t[0] for i, t in enumerate(timers) if i >= T)
    step_ms = statistics.fmean(1e3 * t[2] / max(1, t[1]) for i, t in enumerate(timers) if i >= T)
    handoff = {"step_ms": round(step_ms, 3), "verify_ms": round(verify_ms, 3), "draft_ms": round(draft_ms, 3),
               "exposed_ms": round(step_ms - max(verify_ms, draft_ms), 3),
               "note": "per decode step: step time minus the slower of the batched verify (target rank 0) "
                       "and the packed draft forward (CUDA events), averaged over drafters"}

    e2e = None
    if not args.no_e2e:
        pinned = None if is_target else [[torch.tensor(p, dtype=torch.int64).pin_memory() for p in g]
                                         for g in groups[me]]
        e2e_tokens, bi, bo = 0, 0, 0

        def e2e_check(gi, r):
            nonlocal e2e_tokens, bi, bo
            bi += sum(8 * p.numel() for p in pinned[gi])
            for o in r["outputs"]:
                e2e_tokens += len(o.tokens)
                bo += 8 * len(o.tokens)

        barrier()
        w0 = time.perf_counter()
        phase(range(args.warmup, n), e2e_check, pinned)
        barrier()
        e2e_s = dist_max(time.perf_counter() - w0)
        e2e = {"value": dist_sum(e2e_tokens) / e2e_s, "unit": "tokens/s",
               "h2d_bytes_per_step": dist_sum(bi) / args.steps, "d2h_bytes_per_step": dist_sum(bo) / args.steps,
               "timing": "wall clock around the public D3DEngine.generate calls (drafter ranks) while the "
                         "target ranks serve"}

    dev_s_max = dist_max(dev_s)
    all_tokens = dist_sum(tokens)
    ar_s_max = dist_max(ar_time)
    ar_all = dist_sum(ar_tokens if rank == 0 else 0)
    value = all_tokens / dev_s_max
    ar_value = ar_all / ar_s_max if ar_s_max > 0 else None
    ident_all = dist_sum(0.0 if (not is_target and not ident) else 1.0) == world
    acc_all = [None] * world
    dist.all_gather_object(acc_all, accepts)
    accepts = [a for lst in acc_all for a in lst]
    n_launch_all = int(dist_sum(n_launch))
    status = int(grp.status.item()) if (is_target and T > 1) else 0
    status_all = dist_sum(status)
    for i, lk in enumerate(links):
        lk.close(pair[(rank, i)] if is_target else pair[(i, me)])
    if is_target and T > 1:
        grp.close()
    return {
        "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * dev_s_max / args.steps, 3),
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(value / BASELINE_TPS, 4), "vs_baseline_note": BASELINE_NOTE, "dtype": "bf16",
        "data": "synthetic seeded random-token prompts, random-init weights (seed 0), "
                "acceptance-controlled drafts",
        "config": {"model": "Qwen3-8B-layout target + D3D-1.7B-layout drafter (28 layers, block 16)",
                   "global_batch": cc * D, "seq_len": f"prompt {args.prompt_min}-"
                   f"{args.prompt_max} + {args.max_new_tokens} new",
                   "parallelism": f"target tensor-parallel TP={T} (ranks 0..{T - 1}) + {D} drafter GPUs, one "
                                  "request stream each; the drafters' verifies batched into one target forward "
                                  "per round; NVLink mailbox handoff, fused accept+send replies",
                   "concurrency": cc * D, "anchor_num": args.anchor_num,
                   "controlled_accept_mean": args.accept_mean,
                   "measured_accept_mean": round(statistics.fmean(accepts), 3) if accepts else None,
                   "l2": "inputs larger than L2: every verify streams the target's weight shard",
                   "step": f"{D} requests (one per drafter GPU), prefill through last token"},
        "ar_tokens_per_s": round(ar_value, 2) if ar_value else None,
        "speedup_vs_ar": round(value / ar_value, 3) if ar_value else None,
        "speedup_note": f"all {world} GPUs vs target-only AR on the {T} target GPUs at concurrency {cc * D}",
        "handoff": handoff,
        "token_identical_to_ar": bool(ident_all),
        "tp_exchange_status": status_all,
        "gpu_launches": n_launch_all,
        "clocks": clk.summary(),
        "e2e": e2e,
        "impl": "ours",
    }


# -------------------------------------------------------------- reference
def run_reference(args, rank, world, local):
    from baseline import reference_arm
    return reference_arm.run(args, rank, world, local)


def main():
    args = parse()
    rank, world, local = dist_setup()
    if world > 1:
        # a rank stuck past the watchdog prints every thread's stack and exits,
        # so a multi-GPU run never holds its GPUs silently
        import faulthandler
        faulthandler.dump_traceback_later(args.watchdog_s, exit=True)
    try:
        if args.impl == "reference":
            try:
                out = run_reference(args, rank, world, local)
            except ImportError as e:
                out = {"impl": "reference", "unavailable": f"reference arm not importable: {e}"}
        else:
            layout = args.layout
            if layout == "auto":
                layout = "replica" if world == 1 or world % 2 else "disagg"
            if layout in ("disagg", "tp") and (world < 2 or world % 2):
                raise SystemExit(f"--layout {layout} needs an even number of GPUs")
            run = {"disagg": run_disagg, "tp": run_tp_layout, "replica": run_ours}[layout]
            out = run(args, rank, world, local)
        if rank == 0 and out is not None:
            line = json.dumps(out)
            print(line, flush=True)
            if args.json_out:
                with open(args.json_out, "w") as f:
                    f.write(line + "\n")
    except BaseException:
        if world > 1:
            # say why at once and leave: the other ranks' next collective
            # fails instead of every rank waiting out the process-group timeout
            import traceback
            print(f"[rank {rank}] bench failed:", file=sys.stderr)
            traceback.print_exc()
            sys.stderr.flush()
            sys.stdout.flush()
            os._exit(1)
        raise
    finally:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
