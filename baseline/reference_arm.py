"""Reference arm of ``bench.py``: the unmodified reference (installed under
``baseline/_ref``) decoding the same synthetic workload through its own public
API and stock code path.

* Models: random-init checkpoints of the same architectures (Qwen3-8B layout
  target; D3D-1.7B layout drafter with ``d3d_draft: true``) built with the
  reference's own classes / Hugging Face ``transformers`` and saved in HF
  layout; the reference loads them with its own loader (``_load_model``).
* Target: the reference's ``VerifierProcessClient`` (a spawned process holding
  the target, talking over a Pipe).  Drafter: ``_load_model`` in this process.
  With one GPU both sit on ``cuda:<local rank>``.
* Decode: ``run_d3d_generate_async`` with block 16, one anchor, causal draft
  mask, greedy — the reference's quick-start settings except the anchor count.
* The AR oracle/baseline is target-only decoding through the same verifier
  client (prefill + one-token verify, the loop of the reference's
  ``run_ar_baseline``), which also yields the oracle tokens of the
  acceptance-controlled mode.
* Controlled acceptance: the reference's two draft functions are wrapped so
  their outputs are rewritten by the same injection rules as ours
  (``d3d_b200.engine.controlled``), keyed by absolute position.  Nothing else
  on the reference path is touched.
* Timing: CUDA events on this process's stream with a synchronize on both
  sides of the timed requests (the reference loop is synchronous per step).
"""
from __future__ import annotations

import json
import os
import statistics
import sys
import time
from pathlib import Path

REF_ROOT = Path(__file__).resolve().parent / "_ref"
BASELINE_TPS = 501.60
EOS = (151643, 151645)
MASK_ID = 151669


def _ckpt_dir() -> Path:
    for cand in ("/dev/shm", "/tmp"):
        try:
            st = os.statvfs(cand)
            if st.f_bavail * st.f_frsize > 40e9:
                return Path(cand) / "d3d_ref_ckpt"
        except OSError:
            continue
    return Path("/tmp/d3d_ref_ckpt")


def _build_checkpoints(root: Path, device, draft_layers: int, seed: int):
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM
    tgt, drf = root / "target", root / "draft"
    if (tgt / "config.json").exists() and (drf / "config.json").exists():
        return tgt, drf
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        torch.manual_seed(seed)
        cfg = Qwen3Config(vocab_size=151936, hidden_size=4096, intermediate_size=12288,
                          num_hidden_layers=36, num_attention_heads=32, num_key_value_heads=8,
                          head_dim=128, rope_theta=1e6, max_position_embeddings=40960,
                          tie_word_embeddings=False, rms_norm_eps=1e-6)
        with torch.device(device):
            m = Qwen3ForCausalLM(cfg)
        m.save_pretrained(str(tgt), safe_serialization=True)
        del m
        torch.cuda.empty_cache()
        from models.d3d.configuration_d3d import D3DConfig
        from models.d3d.modeling_d3d import D3DForCausalLM
        dc = D3DConfig(vocab_size=151936, hidden_size=2048, intermediate_size=6144,
                       num_hidden_layers=draft_layers, num_attention_heads=16, num_key_value_heads=8,
                       head_dim=128, rope_theta=1e6, max_position_embeddings=40960,
                       tie_word_embeddings=True, rms_norm_eps=1e-6)
        dc.mask_token_id = MASK_ID
        with torch.device(device):
            d = D3DForCausalLM(dc)
        d.save_pretrained(str(drf), safe_serialization=True)
        del d
        torch.cuda.empty_cache()
    finally:
        torch.set_default_dtype(old)
    return tgt, drf


def run(args, rank, world, local):
    import torch
    import torch.distributed as dist

    if not (REF_ROOT / "single" / "eval_async_packed.py").exists():
        return {"impl": "reference", "unavailable": "reference not installed under baseline/_ref"}
    sys.path.insert(0, str(REF_ROOT))
    # The image ships transformers 5.5; the reference pins 4.57, whose
    # cache_utils still exported SlidingWindowCache.  models/d3d/modeling_d3d.py
    # imports that name (it never uses it on the decode path), so the missing
    # name is aliased in the dependency before the reference is imported.  The
    # reference's own files are not modified.
    import transformers.cache_utils as _cu
    if not hasattr(_cu, "SlidingWindowCache"):
        _cu.SlidingWindowCache = _cu.DynamicCache
    import single.eval_async_packed as ea
    import single.eval_sync as es

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    from bench import BASELINE_NOTE, ClockSampler, barrier, dist_max, dist_sum, make_prompts, METRIC
    from d3d_b200.engine.controlled import ControlledAcceptance, rate_for_mean_accept

    dev = f"cuda:{local}"
    root = _ckpt_dir()
    if rank == 0:
        _build_checkpoints(root, dev, args.draft_layers, args.seed)
    if dist.is_initialized():
        dist.barrier()
    tgt_path, drf_path = root / "target", root / "draft"

    # the reference's stock attention implementation (its CLI default) is
    # FlashAttention-2 for both models; SDPA is the fallback when it is absent
    try:
        import flash_attn  # noqa: F401
        attn = "flash_attention_2"
    except ImportError:
        attn = "sdpa"
    # Layout: with an even number of GPUs the reference runs in its stock
    # two-GPU arrangement (its CLI defaults: verifier on one GPU, drafter on
    # another), one pair per two ranks: the even rank drives the decode with
    # its verifier process on the partner GPU, the odd rank only joins the
    # collectives.  One GPU (or --layout replica): both on the rank's GPU.
    layout = getattr(args, "layout", "auto")
    pairs = world > 1 and world % 2 == 0 and layout in ("auto", "disagg")
    active = not pairs or rank % 2 == 0
    verifier_dev = f"cuda:{local + 1}" if pairs else dev
    n = args.warmup + args.steps
    if not active:
        return _idle_rank(args, world, local, pairs, attn, barrier, dist_max, dist_sum, ClockSampler)
    visible, worker_dev = ea._isolated_cuda_device(verifier_dev)
    verifier = ea.VerifierProcessClient(str(tgt_path), worker_dev, "bf16", attn, (), visible)
    drafter = es._load_model(str(drf_path), torch.bfloat16, attn_implementation=attn).to(dev).eval()
    es._disable_default_cache(drafter)
    verifier.wait_ready()

    prompts = make_prompts(n, args.prompt_min, args.prompt_max,
                           seed=1000 + 7919 * (rank // 2 if pairs else rank) + args.seed)
    ids = [torch.tensor([p], dtype=torch.long) for p in prompts]

    # --- AR baseline: target-only decoding through the reference verifier
    # (the loop of its run_ar_baseline: prefill, then one-token verifies)
    ar_time, ar_tokens = 0.0, 0
    for i in range(args.warmup, n):
        anchor, _, kv_len = verifier.prefill(ids[i], 0.0, 0, 1.0)
        gen = [int(anchor[0])]
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        while len(gen) < args.max_new_tokens and gen[-1] not in EOS:
            verifier.submit_verify(torch.tensor([[gen[-1]]]), None, int(kv_len), 0.0, 0, 1.0)
            _, _, corr, _ = verifier.receive_verify()
            kv_len += 1
            gen.append(int(corr[0]))
        ar_time += time.perf_counter() - t0
        ar_tokens += len(gen)

    # --- oracle for the controlled mode: the target's greedy continuation
    # computed with block-sized (16-token) verifies, i.e. with the same GEMM
    # shapes the speculative loop verifies with.  The reference's kernels are
    # not batch-invariant, so a one-token AR continuation would disagree with
    # its own block verification and corrupt the injected acceptance rate.
    oracle = {}
    filler = [MASK_ID] * (args.block_size - 1)
    for i, x in enumerate(ids):
        anchor, _, kv_len = verifier.prefill(x, 0.0, 0, 1.0)
        gen = [int(anchor[0])]
        while len(gen) < args.max_new_tokens and gen[-1] not in EOS:
            verifier.submit_verify(torch.tensor([[gen[-1]] + filler]), None, int(kv_len), 0.0, 0, 1.0)
            post, _, _, _ = verifier.receive_verify()
            kv_len += 1
            gen.append(int(post[0][0]))
        oracle[i] = gen

    # --- identical controlled-acceptance injection on the reference's draft outputs
    rate = rate_for_mean_accept(args.accept_mean, args.block_size) if args.accept_mean > 0 else 0.0
    current = {"i": 0}

    def ctl():
        i = current["i"]
        return ControlledAcceptance(oracle=prompts[i] + oracle[i], rate=rate, vocab_size=151936,
                                    seed=args.seed, stream=i, exclude=(MASK_ID,) + EOS)

    orig_anchor = ea.d3d_draft_from_anchor
    orig_packed = ea.d3d_draft_all_outcomes_packed

    def draft_from_anchor(drafter_, **kw):
        block, top, probs = orig_anchor(drafter_, **kw)
        c = ctl()
        b = block[0].clone().cpu()
        t = top[0].clone().cpu() if top is not None else None
        c.override(b, t, int(kw["prefix_len"]))
        block[0].copy_(b.to(block.device))
        if top is not None:
            top[0].copy_(t.to(top.device))
        return block, top, probs

    def all_outcomes(drafter_, **kw):
        cands, tops, probs = orig_packed(drafter_, **kw)
        c = ctl()
        base = int(kw["draft_kv_len"])
        for key, blk in cands.items():
            b = blk[0].clone().cpu()
            t = tops[key][0].clone().cpu() if key in tops else None
            c.override(b, t, base + int(key[0]))
            blk[0].copy_(b.to(blk.device))
            if t is not None:
                tops[key][0].copy_(t.to(tops[key].device))
        return cands, tops, probs

    if args.accept_mean > 0:     # 0 = natural acceptance: the reference's drafts as they are
        ea.d3d_draft_from_anchor = draft_from_anchor
        ea.d3d_draft_all_outcomes_packed = all_outcomes

    opts = dict(block_size=args.block_size, denoising_steps=1, threshold=0.9, remasking="low_confidence",
                top_k=0, top_p=1.0, target_top_k=0, target_top_p=1.0, return_stats=True,
                verifier_device=verifier_dev, draft_device=dev, async_blocks=1, attention_mask_mode="causal",
                anchor_num=args.anchor_num, packed_accepted_counts=None)

    def one(i):
        current["i"] = i
        st = ea.run_d3d_generate_async(drafter, verifier, ids[i].to(dev), args.max_new_tokens, list(EOS),
                                       0.0, **opts)
        out = st.output_ids[0, st.num_input_tokens:].tolist()
        return out, [int(x) for x in st.acceptance_lengths]

    for i in range(args.warmup):
        one(i)
    barrier()
    tokens, accepts, ident = 0, [], True
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        ev0.record()
        for i in range(args.warmup, n):
            out, acc = one(i)
            tokens += len(out)
            accepts += acc
            ident &= out == oracle[i][: len(out)]
        ev1.record()
        barrier()
    dev_s = ev0.elapsed_time(ev1) / 1e3
    verifier.close()

    dev_max = dist_max(dev_s)
    value = dist_sum(tokens) / dev_max
    ar_all, ar_max = dist_sum(ar_tokens), dist_max(ar_time)   # every rank, same order
    ar_value = ar_all / ar_max if ar_max > 0 else None
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * dev_max / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(value / BASELINE_TPS, 4), "vs_baseline_note": BASELINE_NOTE, "dtype": "bf16",
        "data": "synthetic seeded random-token prompts, random-init weights, acceptance-controlled drafts",
        "config": {"model": "Qwen3-8B-layout target + D3D-1.7B-layout drafter (reference classes)",
                   "global_batch": world // 2 if pairs else world,
                   "seq_len": f"prompt {args.prompt_min}-{args.prompt_max} + {args.max_new_tokens} new",
                   "parallelism": (f"reference two-GPU pairs x{world // 2} (verifier process on one GPU, "
                                   "drafter on the partner GPU)") if pairs else
                   f"replica per GPU x{world} (reference verifier process + drafter on the same GPU)",
                   "concurrency": 1, "anchor_num": args.anchor_num,
                   "controlled_accept_mean": args.accept_mean,
                   "measured_accept_mean": round(statistics.fmean(accepts), 3) if accepts else None,
                   "attn_implementation": attn, "oracle": "greedy continuation from 16-token verifies",
                   "step": "one request, prefill through last token"},
        "ar_tokens_per_s": round(ar_value, 2) if ar_value else None,
        "ar_timing": "host perf_counter around each request's one-token verify loop (the reference's "
                     "run_ar_baseline is synchronous per token), after a synchronize",
        "speedup_vs_ar": round(value / ar_value, 3) if ar_value else None,
        "token_identical_to_ar": bool(dist_sum(1.0 if ident else 0.0) == world),
        "token_identical_note": "the reference's outputs against its own greedy continuation from 16-token "
                                "verifies (its kernels are not batch-invariant, so one-token AR can differ)",
        "clocks": clk.summary(),
    }


def _idle_rank(args, world, local, pairs, attn, barrier, dist_max, dist_sum, ClockSampler):
    """The odd rank of a pair: its GPU hosts the partner's verifier process;
    it joins the same collectives as the active rank, with nothing to add."""
    barrier()
    with ClockSampler(local) as clk:
        barrier()
        barrier()
    dist_max(0.0)
    dist_sum(0)
    dist_sum(0)
    dist_max(0.0)
    dist_sum(1.0)
    return None
