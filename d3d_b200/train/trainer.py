"""Distillation of the block-diffusion drafter against a frozen target
(reference: ``train/trainer.py``).

One micro-step: pack anchor+MASK blocks (:mod:`.blocks`), prefill the clean
sequence through the student without gradient, run the packed block forward
against that KV, take the target's hidden states at the supervising
positions, and minimise ``alpha_kl * KL(p_target || p_draft) + alpha_ce *
CE(target greedy / response token)`` with position-decayed weights through
the fused LM-head loss (:func:`.losses.lmhead_distill_loss`).  Gradients are
reduce-scattered and applied by the sharded fused AdamW (:mod:`.optim`).

Launch (one process per GPU):

    python -m torch.distributed.run --nproc-per-node 8 -m d3d_b200.train \\
        --draft-model d3d-1.7b --target-model qwen3-8b --data-path synthetic \\
        --output-dir out/train --seq-len 2048 --batch-size 4 --lr 1e-4
"""
from __future__ import annotations

import datetime
import json
import os
import random
import time
from pathlib import Path
from typing import Optional

import torch
import torch.distributed as dist

from ..checkpoint import expected_keys, write_state
from .data import IndexedExamples, Prefetcher, RowLimits, worker_rng
from .blocks import build_packed_block_batch, synthetic_examples
from . import trajectory
from .losses import ce_aux_per_token, decay_weights, lmhead_distill_loss, normalize_objective
from .model_utils import clean_prefill, student_hidden, teacher_hidden
from .optim import ShardedAdamW, cosine_lr


def _init_dist(device_type: str):
    if dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        backend = "nccl" if device_type == "cuda" else "gloo"
        kw = {}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=600), **kw)
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def _all_sum(x: float, device) -> float:
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t)
    return float(t.item())


def _batch_source(args, rank: int, world: int, vocab: int, rng: random.Random, mask_id: int, cursor: int,
                  tok=None, n_micro: int = 1):
    """``make(micro_step) -> (examples, packed batch, cursor after)``, called
    in micro-step order (on the prefetch thread unless ``--workers 0``).
    ``synthetic`` draws seeded random sequences; a JSONL path goes through
    the byte-offset index (rank-strided rows, chat-template split,
    ``train/dataset.py:157-231``)."""
    state = {"cursor": cursor}
    if args.data_path == "synthetic":
        # a bounded pool of seeded sequences, read cyclically (long synthetic runs
        # would otherwise hold every step's tokens in host memory)
        pool = synthetic_examples(min(args.batch_size * max(1, n_micro), 1024), args.seq_len, 0.25, vocab, rng)

        def take(c, n):
            return [pool[(c + i) % len(pool)] for i in range(n)], c + n
    else:
        src = IndexedExamples(args.data_path, rank, world, tok,
                              RowLimits(args.max_prompt_len, args.max_seq_len, args.enable_thinking_template),
                              args.max_examples)
        take = src.take
    pin = bool(getattr(args, "pin_memory", True)) and torch.cuda.is_available() and args.device.startswith("cuda")

    def make(step):
        exs, state["cursor"] = take(state["cursor"], args.batch_size)
        batch = build_packed_block_batch(exs, block_size=args.block_size, mask_token_id=mask_id,
                                         max_anchors=args.parallel_anchors_per_example,
                                         rng=worker_rng(args.seed, rank, step)) if exs else None
        if batch is not None and pin:
            batch = batch.pin()
        return exs, batch, state["cursor"]
    return make


def _rows(args) -> int:
    """Rows of the training file (after ``--max-examples``); 0 for synthetic."""
    if args.data_path == "synthetic":
        return 0
    from .data import JsonlIndex
    return JsonlIndex(args.data_path, 0, 1, args.max_examples).total_rows


def _build(name: str, device, dtype, seed: int, layers: Optional[int] = None, mask_id: Optional[int] = None,
           random_init: bool = False):
    from ..cli.common import is_preset, model_config
    from ..models.qwen3 import build_model
    if is_preset(name):
        return build_model(model_config(name, layers), seed=seed, dtype=dtype, device=device)
    if random_init:
        from ..config import ModelConfig
        return build_model(ModelConfig.from_pretrained(name, mask_token_id=mask_id), seed=seed, dtype=dtype,
                           device=device)
    from ..checkpoint import load_model
    return load_model(name, device=device, dtype=dtype, mask_token_id=mask_id)


def save_checkpoint(model, opt: ShardedAdamW, out_dir: Path, step: int, cursor: int, z3=None) -> None:
    """HF-layout FP32 safetensors from the fp32 master shards (gathered),
    plus this rank's optimizer shard and the trainer state, written atomically.
    With sharded decoder layers (``z3``) their master shards are gathered too
    and each rank also keeps its layer-shard optimizer state."""
    rank = opt.rank
    full = torch.empty(opt.padded, dtype=torch.float32, device=opt.master.device)
    if opt.world > 1:
        dist.all_gather_into_tensor(full, opt.master, group=opt.group)
    else:
        full[: opt.shard] = opt.master
    layers = z3.full_state("model.layers.") if z3 is not None else {}
    ck = out_dir / f"step_{step:07d}"
    tmp = out_dir / f".step_{step:07d}.tmp"
    if rank == 0:
        tmp.mkdir(parents=True, exist_ok=True)
        state, off = {}, 0
        names = [n for n, p in model.named_parameters() if p.requires_grad]
        for n, p in zip(names, opt.params):
            state[n] = full[off:off + p.numel()].view(p.shape).cpu().clone()
            off += p.numel()
        state.update(layers)
        for n, p in model.named_parameters():
            if n not in state:
                state[n] = p.detach().float().cpu()
        if model.cfg.tie_word_embeddings:
            state.pop("lm_head.weight", None)
        keep = set(expected_keys(model.cfg))
        write_state({k: v for k, v in state.items() if k in keep}, tmp)
        model.cfg.save(tmp)
        (tmp / "trainer_state.json").write_text(json.dumps({"step": step, "data_cursor": cursor,
                                                            "world": opt.world}))
    if dist.is_initialized():
        dist.barrier()
    if rank == 0:
        os.replace(tmp, ck)
    if dist.is_initialized():
        dist.barrier()
    torch.save(opt.state_dict(), ck / f"optim_rank{rank:03d}.pt")
    if z3 is not None:
        torch.save(z3.state_dict(), ck / f"layers_rank{rank:03d}.pt")


def validate_args(args) -> None:
    """The reference's checks of the training flags (``train/trainer.py:470-515``)."""
    checks = [
        (args.block_size > 1, "--block-size must be > 1"),
        (args.batch_size > 0, "--batch-size must be > 0"),
        (args.parallel_anchors_per_example > 0, "--parallel-anchors-per-example must be > 0"),
        (args.workers >= 0, "--workers must be >= 0"),
        (args.workers == 0 or args.prefetch > 0, "--prefetch must be > 0 when workers are enabled"),
        (args.loss_decay_gamma > 0, "--loss-decay-gamma must be > 0"),
        (args.gradient_accumulation_steps > 0, "--gradient-accumulation-steps must be > 0"),
        (0.0 <= args.min_lr_ratio <= 1.0, "--min-lr-ratio must be in [0, 1]"),
        (args.ce_weight >= 0 and args.kl_weight >= 0, "--ce-weight / --kl-weight must be >= 0"),
        (args.hnce_weight >= 0 and args.hnce_top_k > 0, "--hnce-weight must be >= 0 and --hnce-top-k > 0"),
        (args.margin_weight >= 0 and args.margin_top_k > 0, "--margin-weight must be >= 0 and --margin-top-k > 0"),
        (args.ar_weight >= 0 and args.ar_logit_chunk_size >= 0,
         "--ar-loss-weight and --ar-logit-chunk-size must be >= 0"),
        (args.trajectory_weight >= 0, "--trajectory-weight must be >= 0"),
        (not args.trajectory_shuffle_teacher_blocks or args.trajectory_weight > 0,
         "--trajectory-shuffle-teacher-blocks requires --trajectory-weight > 0"),
        (args.epochs > 0 and args.max_micro_steps >= 0 and args.max_steps >= 0,
         "--epochs must be > 0, --max-micro-steps and --max-steps >= 0"),
    ]
    for ok, msg in checks:
        if not ok:
            raise ValueError(msg)


def _tokenizer(args):
    """The data tokenizer: ``--tokenizer-model``, else the target's or the
    drafter's checkpoint directory when it holds one (the reference's
    fallback order); ``None`` for synthetic data without one."""
    from ..cli.common import is_preset
    path = getattr(args, "tokenizer", None)
    if not path:
        for cand in (args.target_model, args.draft_model):
            if cand and not is_preset(cand) and (Path(cand) / "tokenizer_config.json").is_file():
                path = cand
                break
    if not path:
        return None
    from transformers import AutoTokenizer
    kw = {"fix_mistral_regex": True} if getattr(args, "fix_mistral_regex", False) else {}
    return AutoTokenizer.from_pretrained(path, **kw)


def _mask_id(args, tok) -> Optional[int]:
    """``--mask-token-id``, else the checkpoint's own id (``None`` here), else
    the id of ``--mask-token`` in the tokenizer when the checkpoint has none."""
    if args.mask_token_id is not None:
        return int(args.mask_token_id)
    from ..cli.common import is_preset
    if tok is None or not getattr(args, "mask_token", "") or is_preset(args.draft_model):
        return None
    cfg = json.loads((Path(args.draft_model) / "config.json").read_text())
    if cfg.get("mask_token_id") is not None:
        return None
    tid = tok.convert_tokens_to_ids(args.mask_token)
    if tid is None or tid == tok.unk_token_id:
        return None
    return int(tid)


def _schedule(args, rows: int, world: int) -> int:
    """Optimizer steps of the run: ``--max-steps``, else ``--epochs`` passes
    over this rank's share of ``rows`` (``--batch-size`` per micro-step),
    capped at ``--max-micro-steps``, over ``--gradient-accumulation-steps``."""
    accum = max(1, int(args.gradient_accumulation_steps))
    if args.max_steps > 0:
        return int(args.max_steps)
    micro = None
    if rows > 0:
        per_rank = -(-rows // world)
        micro = max(1, args.epochs) * -(-per_rank // max(1, args.batch_size))
    if args.max_micro_steps > 0:
        micro = args.max_micro_steps if micro is None else min(micro, args.max_micro_steps)
    if micro is None:
        raise ValueError("synthetic data needs --max-steps or --max-micro-steps")
    return max(1, micro // accum)


class _Inline:
    """``Prefetcher``'s interface without a thread (``--workers 0``)."""

    def __init__(self, make, start: int, stop: int):
        self.make, self.s, self.stop = make, start, stop

    def get(self):
        if self.s >= self.stop:
            raise StopIteration
        s = self.s
        self.s += 1
        return s, self.make(s)

    def close(self):
        pass


def _reverse_kl(h_s, w_s, h_t, w_t, weights, rows: int = 256) -> torch.Tensor:
    """``sum_n weights[n] KL(p_s || p_t)[n]`` over row chunks of materialised
    logits (``objective=reverse_kl``)."""
    from .losses import reverse_kl_per_token
    total = h_s.new_zeros((), dtype=torch.float32)
    for i in range(0, h_s.shape[0], rows):
        sl = h_s[i:i + rows].float() @ w_s.float().t()
        with torch.no_grad():
            tl = h_t[i:i + rows].float() @ w_t.float().t()
        total = total + (weights[i:i + rows] * reverse_kl_per_token(sl, tl)).sum()
    return total


def _wandb_run(args, rank: int):
    """A W&B run when a project is named and W&B is importable (rank 0);
    the JSONL metrics file is written either way."""
    if rank != 0 or args.disable_wandb or not args.wandb_project:
        return None
    try:
        import wandb
    except ImportError:
        print("wandb is not installed: metrics go to training_metrics.jsonl only", flush=True)
        return None
    return wandb.init(project=args.wandb_project, name=args.wandb_name or None,
                      config={k: v for k, v in vars(args).items() if isinstance(v, (int, float, str, bool))})


class _TensorBoard:
    """Scalars of every step record under ``<output>/tensorboard`` (rank 0,
    when TensorBoard is installed), as the reference's writer does."""

    def __init__(self, log_dir: Path, rank: int):
        self.w = None
        if rank != 0:
            return
        try:
            from torch.utils.tensorboard import SummaryWriter
        except ImportError:
            return
        self.w = SummaryWriter(log_dir=str(log_dir))

    def log(self, rec: dict, step: int) -> None:
        if self.w is None:
            return
        for k, v in rec.items():
            if isinstance(v, (int, float)) and not isinstance(v, bool) and v is not None and k != "step":
                self.w.add_scalar(f"train/{k}", float(v), step)

    def close(self) -> None:
        if self.w is not None:
            self.w.close()


def train(args) -> dict:
    device = torch.device(args.device)
    rank, world = _init_dist(device.type)
    if device.type == "cuda":
        device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(device)
    torch.manual_seed(args.seed + rank)
    rng = random.Random(args.seed * 1000 + rank)
    cdt = torch.bfloat16 if (device.type == "cuda" and args.dtype == "bf16") else torch.float32
    validate_args(args)
    accum = max(1, int(getattr(args, "gradient_accumulation_steps", 1)))
    objective = normalize_objective(args.objective)
    if objective in ("forward_kl", "reverse_kl") and not args.target_model:
        raise ValueError(f"objective {objective} needs --target-model")
    probe_steps = int(getattr(args, "trajectory_gradient_probe_steps", 0) or 0)
    if probe_steps < 0:
        raise ValueError("--trajectory-gradient-probe-steps must be >= 0")
    if probe_steps and not getattr(args, "trajectory_weight", 0.0):
        raise ValueError("--trajectory-gradient-probe-steps requires --trajectory-weight > 0")
    if getattr(args, "trajectory_weight", 0.0) and not (args.target_model or args.trajectory_teacher_model):
        raise ValueError("--trajectory-weight needs --trajectory-teacher-model or --target-model")
    cls = getattr(args, "fsdp_transformer_layer_cls", None) or []
    if any(c not in ("D3DDecoderLayer", "Qwen3DecoderLayer", "DecoderLayer") for c in cls):
        raise ValueError("--fsdp-transformer-layer-cls: only the decoder layers can be sharded")
    if getattr(args, "fsdp", False) and not getattr(args, "fsdp_reshard_after_forward", True):
        raise ValueError("sharded decoder layers are always gathered again in backward "
                         "(--no-fsdp-reshard-after-forward is not supported)")
    tok = _tokenizer(args)
    mask_override = _mask_id(args, tok)
    # resuming starts from the checkpoint's weights (its fp32 master values);
    # the optimizer shards and moments come from its per-rank files below
    student = (_build(args.resume, device, cdt, args.seed, None, mask_override) if args.resume else
               _build(args.draft_model, device, cdt, args.seed, args.draft_layers, mask_override,
                      random_init=getattr(args, "random_init", False)))
    student.train()
    if getattr(args, "attn_implementation", None):
        student.set_attn_implementation(args.attn_implementation)

    def frozen_teacher(name, seed):
        t = _build(name, device, cdt, seed).eval()
        for p in t.parameters():
            p.requires_grad_(False)
        if device.type == "cuda" and os.environ.get("D3D_FAST_TEACHER", "1") != "0":
            # the frozen teacher's forward runs on the sm_100a inference kernels
            from .model_utils import FastTeacher
            max_len = args.seq_len if args.data_path == "synthetic" else args.max_seq_len
            t = FastTeacher(t, max(1, args.batch_size), max_len, device)
        return t

    teacher = frozen_teacher(args.target_model, args.seed + 1) if args.target_model else None
    traj_teacher = teacher
    if getattr(args, "trajectory_weight", 0.0) and getattr(args, "trajectory_teacher_model", ""):
        traj_teacher = frozen_teacher(args.trajectory_teacher_model, args.seed + 2)
    if args.freeze_embeddings:
        student.model.embed_tokens.weight.requires_grad_(False)
    student.gradient_checkpointing = bool(getattr(args, "gradient_checkpointing", False))
    z3 = None
    if getattr(args, "fsdp", False):
        # decoder layers live as per-rank shards; the optimizer below sees the rest
        from ..parallel.zero3 import Zero3Layers
        student.gradient_checkpointing = False      # the sharded layers recompute already
        z3 = Zero3Layers(student.model.layers, lr=args.lr, weight_decay=args.weight_decay)
    offload = bool(getattr(args, "fsdp_cpu_offload", False))
    if device.type == "cuda" and world > 1 and not offload and os.environ.get("D3D_FUSED_OPT", "1") != "0":
        # reduce-scatter + AdamW + all-gather fused into kernels over NVLink peer memory
        from ..parallel.fsdp import FusedShardedAdamW
        opt = FusedShardedAdamW(student.parameters(), lr=args.lr, weight_decay=args.weight_decay)
    else:
        opt = ShardedAdamW(student.parameters(), lr=args.lr, weight_decay=args.weight_decay, offload=offload)
    total = _schedule(args, _rows(args), world)
    start, cursor0 = 0, None
    if args.resume:
        ck = Path(args.resume)
        opt.load_state_dict(torch.load(ck / f"optim_rank{rank:03d}.pt"))
        if z3 is not None:
            z3.load_state_dict(torch.load(ck / f"layers_rank{rank:03d}.pt"))
        st = json.loads((ck / "trainer_state.json").read_text())
        start, cursor0 = st["step"], st.get("data_cursor")
    mask_id = int(student.cfg.mask_token_id)
    vocab = min(student.cfg.vocab_size, 151643) - 2
    make_batch = _batch_source(args, rank, world, vocab, rng, mask_id,
                               start * accum * args.batch_size if cursor0 is None else cursor0, tok, total * accum)
    workers = int(getattr(args, "workers", 1))
    prefetch = (Prefetcher(make_batch, start * accum, total * accum,
                           depth=max(1, int(getattr(args, "prefetch", 2))) * max(1, workers))
                if workers > 0 else _Inline(make_batch, start * accum, total * accum))
    out_dir = Path(args.output_dir)
    if rank == 0:
        out_dir.mkdir(parents=True, exist_ok=True)
        (out_dir / "args.json").write_text(json.dumps({**{k: v for k, v in vars(args).items()
                                                          if isinstance(v, (int, float, str, bool, list, type(None)))},
                                                       "world_size": world}, indent=2, sort_keys=True))
    run = _wandb_run(args, rank)
    tb = _TensorBoard(out_dir / "tensorboard", rank)
    a_kl = args.kl_weight if (teacher is not None and objective in ("forward_kl", "kl_ce")) else 0.0
    a_rkl = args.kl_weight if (teacher is not None and objective == "reverse_kl") else 0.0
    a_ce = args.ce_weight if objective in ("ce", "kl_ce") else 0.0
    probe_left = int(getattr(args, "trajectory_gradient_probe_steps", 0) or 0)
    shuffle = (torch.Generator().manual_seed(args.seed + 7 * rank)
               if getattr(args, "trajectory_shuffle_teacher_blocks", False) else None)
    log = []
    cursor = start * accum * args.batch_size if cursor0 is None else cursor0
    t_start = time.perf_counter()
    for step in range(start, total):
        if device.type == "cuda":
            torch.cuda.synchronize()
        t0 = time.perf_counter()
        tot = {"loss": 0.0, "kl": 0.0, "ce": 0.0, "tokens": 0.0}
        empty, probe = 0, None
        for _ in range(accum):
            _, (exs, batch, cursor) = prefetch.get()   # packed on the host, ahead of the device
            if batch is None:
                # nothing to supervise on this rank in this micro-step: take part in
                # every collective with zeros, so the ranks stay matched (the
                # reference runs a dummy forward/backward, train/trainer.py:103-146)
                _all_sum(0.0, device)
                if getattr(args, "ar_weight", 0.0):
                    _all_sum(0.0, device)
                if getattr(args, "trajectory_weight", 0.0) and traj_teacher is not None:
                    _all_sum(0.0, device)
                if z3 is not None:
                    passes = 1 + (1 if getattr(args, "ar_weight", 0.0) else 0)
                    z3.idle_exchanges(passes * len(z3.specs))
                empty += 1
                continue
            batch = batch.to(device)
            cache = clean_prefill(student, batch)
            hs = student_hidden(student, batch, cache)
            act = batch.active
            w = decay_weights(batch.offsets[act], args.loss_decay_gamma)
            z = _all_sum(float(w.sum()), device)
            w = w / max(z, 1e-6)
            h_t = w_t = None
            targets = batch.target_ids[act]
            th_all = None
            if teacher is not None:
                th_all = teacher_hidden(teacher, batch)
                th = th_all[act]
                h_t, w_t = th, teacher.lm_weight
                if args.ce_on_target_greedy:
                    targets = (teacher.logits(th).argmax(-1) if device.type != "cuda" else
                               _greedy(th, w_t))
            loss, kl, ce = lmhead_distill_loss(hs[act], student.lm_weight, h_t, w_t, targets,
                                               (a_kl * w) if a_kl else None, (a_ce * w) if a_ce else None,
                                               chunk=args.vocab_chunk)
            if a_rkl:
                loss = loss + _reverse_kl(hs[act], student.lm_weight, h_t, w_t, a_rkl * w)
            if getattr(args, "hnce_weight", 0.0) or getattr(args, "margin_weight", 0.0):
                # auxiliary objectives on materialised student logits of the supervised rows
                logits = hs[act].float() @ student.lm_weight.float().t()
                aux, _, _, _ = ce_aux_per_token(logits, targets, ce_weight=0.0, hnce_weight=args.hnce_weight,
                                                hnce_top_k=args.hnce_top_k, hnce_margin=args.hnce_margin,
                                                margin_weight=args.margin_weight, margin_top_k=args.margin_top_k,
                                                margin_value=args.margin_value, margin_smooth=args.margin_smooth)
                loss = loss + (w * aux).sum()
            if getattr(args, "ar_weight", 0.0):
                # clean autoregressive loss (reference: train/losses.py:380-468), mean over
                # every rank's valid next-token positions, through the fused LM-head CE
                hc = student(batch.clean_ids)[:, :-1]
                pos = torch.arange(hc.shape[1], device=device)[None]
                valid = pos < (batch.clean_lens[:, None] - 1)
                n_ar = _all_sum(float(valid.sum()), device)
                w_ar = torch.full((int(valid.sum()),), args.ar_weight / max(n_ar, 1.0), device=device)
                ar_loss, _, _ = lmhead_distill_loss(hc[valid], student.lm_weight, None, None,
                                                    batch.clean_ids[:, 1:][valid], None, w_ar,
                                                    chunk=args.vocab_chunk)
                loss = loss + ar_loss
            if getattr(args, "trajectory_weight", 0.0) and traj_teacher is not None:
                tt_all = th_all if traj_teacher is teacher else teacher_hidden(traj_teacher, batch)
                unit = _trajectory_term(student, traj_teacher, batch, hs, tt_all, device, world, shuffle)
                if probe_left > 0:
                    # gradient scale of the unit trajectory term against the data CE at
                    # the student's final hidden states
                    ce_only, _, _ = lmhead_distill_loss(hs[act], student.lm_weight, None, None, targets, None, w,
                                                        chunk=args.vocab_chunk)
                    g_t = torch.autograd.grad(unit, hs, retain_graph=True, allow_unused=True)[0]
                    g_c = torch.autograd.grad(ce_only, hs, retain_graph=True, allow_unused=True)[0]
                    nt = float(g_t.float().norm()) if g_t is not None else 0.0
                    nc = float(g_c.float().norm()) if g_c is not None else 0.0
                    probe = {"trajectory_grad_norm": nt, "ce_grad_norm": nc,
                             "trajectory_to_ce_grad_ratio": nt / nc if nc > 0 else None}
                    probe_left -= 1
                    if rank == 0:
                        print(f"  trajectory_grad | ce_hidden {nc:.6e} | unit_traj_hidden {nt:.6e} | "
                              f"unit/ce {probe['trajectory_to_ce_grad_ratio'] or 0.0:.4f}", flush=True)
                loss = loss + args.trajectory_weight * unit
            (loss / accum).backward()
            tot["loss"] += float(loss.item())
            tot["kl"] += float((kl * w).sum().item())
            tot["ce"] += float((ce * w).sum().item())
            tot["tokens"] += float(act.sum().item())
        lr = cosine_lr(step, args.lr, args.warmup_steps, total, args.min_lr_ratio)
        gnorm = _opt_step(opt, z3, args.grad_clip, lr)
        opt.zero_grad()
        if device.type == "cuda":
            torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        rec = {"step": step + 1, "loss": _all_sum(tot["loss"] / accum, device),
               "kl": _all_sum(tot["kl"] / accum, device), "ce": _all_sum(tot["ce"] / accum, device),
               "grad_norm": gnorm, "lr": lr, "tokens": int(_all_sum(tot["tokens"], device)), "step_s": dt}
        if empty == accum:
            rec["empty_rank"] = True
        if probe is not None:
            rec.update(probe)
        log.append(rec)
        if rank == 0:
            with open(out_dir / "training_metrics.jsonl", "a") as f:
                f.write(json.dumps(rec) + "\n")
            if run is not None:
                run.log(rec, step=step + 1)
            tb.log(rec, step + 1)
            if args.log_every and (step + 1) % args.log_every == 0:
                print(json.dumps(rec), flush=True)
        if args.save_every and (step + 1) % args.save_every == 0:
            save_checkpoint(student, opt, out_dir, step + 1, cursor, z3)
    if args.save_final:
        save_checkpoint(student, opt, out_dir, total, cursor, z3)
    prefetch.close()
    if run is not None:
        run.finish()
    tb.close()
    if z3 is not None:
        z3.close()
    return {"log": log, "elapsed_s": time.perf_counter() - t_start, "world": world, "steps": total}


def _opt_step(opt, z3, grad_clip: float, lr: float) -> float:
    """Optimizer step of the replicated parameters and, with sharded decoder
    layers, of their shards -- one gradient norm and clip factor for both."""
    if z3 is None:
        return opt.step(grad_clip, lr)
    gnorm = opt.step(grad_clip, lr, extra_sumsq=z3.sumsq())
    z3.step(opt.last_scale, lr)
    z3.zero_grad()
    return gnorm


def _argmax_rows(h: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    if h.is_cuda:
        return _greedy(h, w)
    return (h.float() @ w.float().t()).argmax(-1)


def _trajectory_term(student, teacher, batch, hs, th_all, device, world, shuffle=None) -> torch.Tensor:
    """Block-relation distillation over blocks the teacher drafts better
    (``train/trajectory.py``), normalised by the global selected-block count."""
    K = batch.block_size
    B, Q = batch.active.shape
    with torch.no_grad():
        s_pred = _argmax_rows(hs.reshape(B * Q, -1).detach(), student.lm_weight).view(B, Q)
        t_pred = _argmax_rows(th_all.reshape(B * Q, -1), teacher.lm_weight).view(B, Q)
    valid = trajectory.by_block(batch.active, K)
    tgt = trajectory.by_block(batch.target_ids, K)
    s_acc = trajectory.block_accept_lengths(trajectory.by_block(s_pred, K)[..., 1:], tgt[..., 1:], valid[..., 1:])
    t_acc = trajectory.block_accept_lengths(trajectory.by_block(t_pred, K)[..., 1:], tgt[..., 1:], valid[..., 1:])
    sel = trajectory.selection_mask(t_acc, s_acc, valid.sum(-1), batch.block_keep)
    lsum, cnt = trajectory.relational_loss(trajectory.by_block(hs, K), trajectory.by_block(th_all, K), valid, sel,
                                           shuffle)
    return trajectory.distributed_block_mean(lsum, _all_sum(float(cnt), device), world)


def _greedy(h, w) -> torch.Tensor:
    from .. import ops
    ov, oi = ops.gemm_topk(h.to(torch.bfloat16).contiguous(), w.contiguous(), 1)
    return oi[:, 0]
