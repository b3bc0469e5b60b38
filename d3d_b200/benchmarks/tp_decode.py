"""Tensor-parallel target + disaggregated drafter (the Qwen3-32B configuration).

    python -m torch.distributed.run --nnodes=1 --nproc-per-node <T+1> --master-addr 127.0.0.1 \\
        -m d3d_b200.benchmarks.tp_decode --tp T [--target qwen3-32b] [--draft-layers 24]

Ranks ``0..T-1`` hold the target, tensor-parallel (column-parallel QKV /
gate-up, row-parallel o / down whose all-reduce is fused into the residual +
RMSNorm kernel, vocab-parallel LM head), and serve verify requests; rank
``T`` runs the drafter (a pruned 24-layer D3D-1.7B layout) and the
coordinator.  Requests go to every target rank through NVLink mailboxes;
rank 0's fused acceptance kernel writes the result into the drafter GPU's
mailbox.  Random-init weights, seeded random prompts of ``--prompt-len``
tokens, ``--max-new-tokens`` greedy tokens, acceptance-controlled drafts
(mean ``--accept-mean``); the AR baseline runs target-only on the same T
ranks.  Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import random
import statistics
import time

import torch
import torch.distributed as dist

EOS = (151643, 151645)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--target", default="qwen3-32b")
    p.add_argument("--draft-layers", type=int, default=24)
    p.add_argument("--prompt-len", type=int, default=512)
    p.add_argument("--max-new-tokens", type=int, default=512)
    p.add_argument("--requests", type=int, default=3)
    p.add_argument("--warmup", type=int, default=1)
    p.add_argument("--accept-mean", type=float, default=5.0)
    p.add_argument("--concurrency", type=int, default=1)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--target-path", default=None, help="HF checkpoint (each rank reads only its slices)")
    p.add_argument("--draft-path", default=None, help="HF checkpoint of the drafter")
    return p.parse_args()


def main():
    a = parse()
    from d3d_b200 import config as C
    from d3d_b200.engine.controlled import ControlledAcceptance, rate_for_mean_accept
    from d3d_b200.engine.disagg import DEFAULT_SLOT_BYTES, P2PTarget, P2PTargetServer
    from d3d_b200.engine.fast import FastDraft, FastTarget
    from d3d_b200.engine.layout import paged_draft_branch_tokens
    from d3d_b200.engine.spec import DecodeConfig, SpecDecoder, ar_generate
    from d3d_b200.models.fast import FastWeights
    from d3d_b200.parallel.p2p import Link
    from d3d_b200.parallel.tp import TPGroup, random_shard
    from d3d_b200.utils import launches
    from d3d_b200.utils.benchutil import ClockSampler, barrier, dist_max, dist_setup, dist_sum

    rank, world, local = dist_setup()
    T = a.tp
    if world != T + 1:
        raise SystemExit(f"--tp {T} needs {T + 1} processes (one drafter rank)")
    dev = torch.device("cuda", local)
    drafter = rank == T
    tp_group = dist.new_group(list(range(T)))
    pairs = [dist.new_group([j, T]) for j in range(T)]
    tcfg = C.ModelConfig.from_pretrained(a.target_path) if a.target_path else C.PRESETS[a.target]()
    dcfg = C.d3d_1p7b(num_layers=a.draft_layers)
    K = 16
    decode = DecodeConfig(block_size=K, anchor_num=1, max_new_tokens=a.max_new_tokens, eos=EOS)
    max_ctx = a.prompt_len + a.max_new_tokens + 2 * K
    cc = a.concurrency
    n = a.warmup + a.requests
    rng = random.Random(1000 + a.seed)
    prompts = [[rng.randrange(0, 151643) for _ in range(a.prompt_len)] for _ in range(n * cc)]
    groups = [prompts[i * cc:(i + 1) * cc] for i in range(n)]

    ar_out, ar_time, ar_tokens = {}, 0.0, 0
    if not drafter:
        grp = TPGroup(rank, T, dev, group=tp_group, num_layers=tcfg.num_hidden_layers) if T > 1 else None
        if a.target_path:
            from d3d_b200.api import load_target_shard
            w = load_target_shard(a.target_path, T, rank, device=dev)
        else:
            w = random_shard(tcfg, T, rank, seed=a.seed, device=dev) if T > 1 else \
                FastWeights.random(tcfg, seed=a.seed, device=dev)
        link = Link(1, DEFAULT_SLOT_BYTES, dev, group=pairs[rank])
        pages = max(4, cc) * (max_ctx + 64 + 16) // 16 + 8
        tgt = FastTarget(w, pages=pages, max_seqs=max(4, cc), max_context=max_ctx, device=dev, tp=grp)
        for gi, g in enumerate(groups):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            r = ar_generate(tgt, g, a.max_new_tokens, eos=EOS, concurrency=cc)
            torch.cuda.synchronize()
            e1.record()
            torch.cuda.synchronize()
            for j, o in enumerate(r["outputs"]):
                ar_out[gi * cc + j] = o
            if gi >= a.warmup:
                ar_time += e0.elapsed_time(e1) / 1e3
                ar_tokens += sum(len(o) for o in r["outputs"])
        srv = P2PTargetServer(tgt, link, replies="all" if rank == 0 else "ack")
    else:
        links = [Link(0, DEFAULT_SLOT_BYTES, dev, group=pairs[j]) for j in range(T)]
        if a.draft_path:
            from d3d_b200.checkpoint import load_model
            dw = FastWeights.from_module(load_model(a.draft_path), dev)
        else:
            dw = FastWeights.random(dcfg, seed=a.seed, device=dev)
        packed_q = paged_draft_branch_tokens(K, 1)
        dp = max(4, cc) * (max_ctx + packed_q + 16) // 16 + 8
        d = FastDraft(dw, pages=dp, max_seqs=max(4, cc), max_context=max_ctx, packed_q=packed_q, device=dev)
        remote = P2PTarget(links, tcfg.hidden_size, dev, want_hidden=False, draft_stream=d.stream)
        dec = SpecDecoder(remote, d, decode)
    shared = [None] * world
    dist.all_gather_object(shared, ar_out if rank == 0 else None)
    ar_out = shared[0]
    rate = rate_for_mean_accept(a.accept_mean, K)

    def ctl_for(base):
        def ctl(i):
            k = base + i
            return ControlledAcceptance(oracle=prompts[k] + ar_out[k], rate=rate, vocab_size=tcfg.vocab_size,
                                        seed=a.seed, stream=k, exclude=(151669,) + EOS)
        return ctl

    tokens, accepts, ident, steps = 0, [], True, 0

    def phase(ids, record):
        nonlocal tokens, ident, steps
        if not drafter:
            srv.serve()
            return
        for gi in ids:
            r = dec.generate(groups[gi], concurrency=cc, controlled=ctl_for(gi * cc))
            if record:
                steps += r["steps"]
                for j, o in enumerate(r["outputs"]):
                    tokens += len(o.tokens)
                    accepts.extend(o.accepts)
                    ident &= o.tokens == ar_out[gi * cc + j]
        remote.close()

    phase(range(a.warmup), False)
    barrier()
    launches.reset()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        ev0.record()
        phase(range(a.warmup, n), True)
        torch.cuda.synchronize()
        ev1.record()
        barrier()
    dev_s = dist_max(ev0.elapsed_time(ev1) / 1e3)
    all_tokens = dist_sum(tokens)
    all_steps = dist_sum(steps)
    ar_s = dist_max(ar_time)
    ar_tok = dist_sum(ar_tokens if rank == 0 else 0)
    ident_all = dist_sum(0.0 if (drafter and not ident) else 1.0) == world
    acc = [None] * world
    dist.all_gather_object(acc, accepts)
    accepts = [x for lst in acc for x in lst]
    n_launch = int(dist_sum(launches.count()))
    status = int(grp.status.item()) if (not drafter and grp is not None) else 0
    status_all = dist_sum(status)
    value = all_tokens / dev_s
    ar_value = ar_tok / ar_s if ar_s > 0 else None
    if not drafter:
        link.close(pairs[rank])
    else:
        for j, lk in enumerate(links):
            lk.close(pairs[j])
    if not drafter and grp is not None:
        grp.close()
    if rank == 0:
        print(json.dumps({
            "metric": "decode tokens/s + speedup vs AR (tensor-parallel target)",
            "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
            "ms_per_step": round(1e3 * dev_s / max(1.0, all_steps), 3),
            "config": {"target": f"{a.target} layout, TP={T}", "drafter": f"D3D-1.7B layout, {a.draft_layers} layers",
                       "prompt_len": a.prompt_len, "max_new_tokens": a.max_new_tokens, "concurrency": cc,
                       "requests": a.requests, "controlled_accept_mean": a.accept_mean,
                       "measured_accept_mean": round(statistics.fmean(accepts), 3) if accepts else None,
                       "parallelism": f"target TP={T} (fused row-parallel all-reduce) + drafter on 1 GPU, "
                                      "NVLink mailbox handoff"},
            "ar_tokens_per_s": round(ar_value, 2) if ar_value else None,
            "speedup_vs_ar": round(value / ar_value, 3) if ar_value else None,
            "token_identical_to_ar": bool(ident_all), "exchange_status": status_all,
            "gpu_launches": n_launch, "clocks": clk.summary(), "dtype": "bf16",
            "data": "synthetic seeded random-token prompts, random-init weights, acceptance-controlled drafts"}),
            flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
