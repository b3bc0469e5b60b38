"""Fixed-budget recovery training of a pruned drafter
(reference: ``pruning/train_recovery.py``).

The frozen teacher is the ORIGINAL full-depth drafter recorded in the
child's ``layer_prune.json``.  Per example, on ``[anchor, MASK x (K-1)]``
blocks placed at seeded response offsets (:mod:`d3d_b200.train.blocks`):

``loss = 1.0 * AR + 1.0 * CE + 1.0 * corrected KL + 10.0 * boundary MSE``

(the reference's fixed coefficients, ``train_recovery.py:33-36``).  AR is the
student's next-token cross-entropy over the response of the clean sequence.
CE, corrected KL and the boundary term weight block offset ``o`` by
``exp(-(o - 1) / decay)`` (decay 7.75 for K=16 and 15.5 for K=32).  The
boundary term is the RMS-normalised MSE between every student layer's output
and the teacher's output of the original layer it descends from, the last
one taken before the final norm.  Embeddings and the LM head stay frozen.

:func:`run_recovery` is the stage: a data window of the permuted JSONL rows
(``cursor .. cursor + multiplier x steps x accumulation x world``, rank-strided),
gradient accumulation, warm-up + cosine learning rate, gradient clipping,
``training_metrics.jsonl``, atomic ``step-N`` checkpoints with
``recovery_info.json``, ``run_config.json`` and ``training_summary.json``
(with the next data cursor).  All ranks stop together with an error when any
rank runs out of data before the step budget.
"""
from __future__ import annotations

import json
import math
import os
import random
import shutil
import tempfile
import time
from pathlib import Path
from typing import Dict, Optional, Sequence

import torch
import torch.distributed as dist

from ..engine.layout import rows_to_dense
from ..models.qwen3 import Qwen3LM
from ..train.blocks import Example, PackedTrainBatch, build_packed_block_batch
from ..train.model_utils import clean_prefill
from .losses import boundary_hidden_mse, corrected_kl, masked_mean, target_ce

LAMBDA_AR, LAMBDA_CE, LAMBDA_KL, LAMBDA_H = 1.0, 1.0, 1.0, 10.0
_DECAY = {16: 7.75, 32: 15.5}


def position_decay(block_size: int) -> float:
    """Decay length of the position weights; block sizes other than 16 and 32
    (which the reference refuses) use ``(K - 1) / 2``."""
    return _DECAY.get(int(block_size), (block_size - 1) / 2.0)


def learning_rate(step: int, total: int, base: float, minimum: float, warmup_ratio: float) -> float:
    """Learning rate of optimizer step ``step`` (1-based): linear from
    ``minimum`` to ``base`` over the warm-up steps, then a half cosine back
    down to ``minimum`` at ``total``."""
    warm = round(total * warmup_ratio) if warmup_ratio else 0
    if warm and step <= warm:
        frac = 1.0 if warm == 1 else (step - 1) / (warm - 1)
    else:
        t = min(max((step - warm) / max(total - warm, 1), 0.0), 1.0)
        frac = 0.5 * (1.0 + math.cos(math.pi * t))
    return minimum + (base - minimum) * frac


def _block_forward(model: Qwen3LM, batch: PackedTrainBatch, cache):
    lc, q = batch.clean_ids.shape[1], batch.draft_ids.shape[1]
    return model(batch.draft_ids, batch.positions, mask=rows_to_dense(batch.rows, lc + q), cache=cache,
                 store_kv=False, output_hidden_states=True)


def block_accept_lengths(pred: torch.Tensor, batch: PackedTrainBatch) -> torch.Tensor:
    """``1 + leading matches`` of every placed block (``[blocks]``)."""
    K = batch.block_size
    B, Q = pred.shape
    ok = (pred.eq(batch.target_ids) & batch.active).view(B, Q // K, K)[..., 1:]
    acc = ok.long().cumprod(-1).sum(-1) + 1
    return acc[batch.block_keep]


def recovery_losses(student: Qwen3LM, teacher: Qwen3LM, retained_original: Sequence[int], batch: PackedTrainBatch,
                    prompt_lens: torch.Tensor) -> Dict[str, torch.Tensor]:
    """The four recovery terms (differentiable through the student) and the
    student's and teacher's block accept lengths."""
    K = batch.block_size
    act = batch.active
    w = torch.exp(-(batch.offsets.float() - 1).clamp_min(0) / position_decay(K)) * act.float()
    wa = w[act]
    with torch.no_grad():
        th, ths = _block_forward(teacher, batch, clean_prefill(teacher, batch))
        tl_full = teacher.logits(th)
        tlog = tl_full[act]
        scache = clean_prefill(student, batch)       # clean keys/values: no gradient, as in the reference
    sh, shs = _block_forward(student, batch, scache)
    sl_full = student.logits(sh)
    slog = sl_full[act]
    tgt = batch.target_ids[act]
    ce = masked_mean(target_ce(slog, tgt), wa, distributed=True)
    kl = masked_mean(corrected_kl(slog, tlog, tgt), wa, distributed=True)
    L = len(shs) - 1
    if len(retained_original) != L:
        raise ValueError("retained-layer mapping does not match the student's depth")
    s_b = torch.stack([shs[j + 1][act] for j in range(L)], 0)
    t_b = torch.stack([ths[int(r) + 1][act] for r in retained_original], 0)
    hm = boundary_hidden_mse(s_b, t_b)
    hidden = masked_mean(hm, wa[None].expand_as(hm), distributed=True)
    # next-token loss over the response of the clean sequence
    lg = student.logits(student(batch.clean_ids))[:, :-1]
    n = batch.clean_ids.shape[1] - 1
    pos = torch.arange(n, device=lg.device)[None]
    arw = ((pos >= prompt_lens.to(lg.device)[:, None] - 1) & (pos < batch.clean_lens.to(lg.device)[:, None] - 1))
    ar = masked_mean(target_ce(lg.reshape(-1, lg.shape[-1]), batch.clean_ids[:, 1:].reshape(-1)),
                     arw.reshape(-1).float(), distributed=True)
    with torch.no_grad():
        s_acc = block_accept_lengths(sl_full.argmax(-1), batch).float().mean()
        t_acc = block_accept_lengths(tl_full.argmax(-1), batch).float().mean()
    return {"autoregressive_loss": ar, "cross_entropy": ce, "kl": kl, "hidden": hidden,
            "student_accept_length": s_acc, "teacher_accept_length": t_acc}


def make_student(parent: Qwen3LM, removed_compact: int) -> Qwen3LM:
    """An in-memory pruned copy of ``parent`` with embeddings and LM head frozen."""
    import copy
    from .prune import drop_layers_inplace
    s = copy.deepcopy(parent)
    drop_layers_inplace(s, [removed_compact])
    for p in s.parameters():
        p.requires_grad_(True)
    freeze_io(s)
    s.train()
    return s


def freeze_io(model: Qwen3LM) -> None:
    model.model.embed_tokens.weight.requires_grad_(False)
    if not model.cfg.tie_word_embeddings:
        model.lm_head.weight.requires_grad_(False)


# ------------------------------------------------------------ the stage
class WindowData:
    """This rank's examples of a recovery data window: virtual positions
    ``cursor_start + rank, + world, ...`` below ``cursor_end``, each read
    from the row the seeded permutation maps it to, skipped when the row does
    not encode (length limits, no assistant turn) or its response is shorter
    than ``min_response``.  ``path == "synthetic"`` serves seeded random
    token rows instead of a file."""

    def __init__(self, path: str, window: dict, rank: int, seed: int, *, tokenizer_dir: Optional[str] = None,
                 max_prompt: int = 4096, max_seq: int = 8192, min_response: int = 16, vocab: int = 1000):
        from ..train.data import JsonlIndex, RowLimits
        self.path, self.window, self.rank, self.seed = path, window, rank, seed
        self.limits = RowLimits(max_prompt_len=max_prompt, max_seq_len=max_seq)
        self.min_response, self.vocab = min_response, vocab
        self.tokenizer_dir, self._tok = tokenizer_dir, None
        self.index = None if path == "synthetic" else JsonlIndex(path)
        if self.index is not None and len(self.index) != window["dataset_rows"]:
            raise RuntimeError(f"dataset changed: expected {window['dataset_rows']} rows, found {len(self.index)}")

    def _encode(self, row: dict) -> Optional[Example]:
        from ..train.data import encode_row
        if "prompt_ids" not in row and self._tok is None:
            from transformers import AutoTokenizer
            self._tok = AutoTokenizer.from_pretrained(self.tokenizer_dir)
        return encode_row(row, self._tok, self.limits)

    def __iter__(self):
        from .common import permuted_row
        w = self.window
        for pos in range(w["cursor_start"] + self.rank, w["cursor_end"], w["world_size"]):
            if self.index is None:
                rng = random.Random(f"{self.seed}:{pos}")
                n_p, n_r = rng.randint(8, 32), rng.randint(self.min_response, 3 * self.min_response)
                ex = Example([rng.randrange(2, self.vocab) for _ in range(n_p)],
                             [rng.randrange(2, self.vocab) for _ in range(n_r)])
            else:
                ex = self._encode(self.index.row(permuted_row(pos, w["dataset_rows"], self.seed)))
            if ex is not None and len(ex.response_ids) >= self.min_response:
                yield pos, ex


def _next_together(it, device):
    """The next example on every rank, or an error on every rank -- decided
    before any collective of the step (``train_recovery.py:157-190``)."""
    item, err = None, None
    try:
        item = next(it)
    except StopIteration:
        err = "candidate window exhausted after filtering; raise --candidate-multiplier or check row lengths"
    except Exception as exc:           # a malformed row must not strand the other ranks
        err = f"{type(exc).__name__}: {exc}"
    errs = [err]
    if dist.is_initialized():
        ok = torch.tensor([int(err is None)], dtype=torch.int32, device=device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if int(ok.item()):
            return item
        errs = [None] * dist.get_world_size()
        dist.all_gather_object(errs, err)
    if any(e is not None for e in errs):
        detail = "; ".join(f"rank {r}: {e}" for r, e in enumerate(errs) if e is not None)
        raise RuntimeError(f"recovery data ran out before the step budget ({detail})")
    return item


def _dist_mean(x: torch.Tensor) -> float:
    x = x.detach().float().reshape(1).clone()
    if dist.is_initialized():
        dist.all_reduce(x)
        x /= dist.get_world_size()
    return float(x.item())


def _copy_support(src: Path, dst: Path) -> None:
    """Tokenizer and other side files of the student checkpoint."""
    skip = {"config.json", "model.safetensors.index.json", "layer_prune.json", "recovery_info.json"}
    for f in src.iterdir():
        if f.is_file() and f.suffix != ".safetensors" and f.name not in skip:
            shutil.copy2(f, dst / f.name)


def run_recovery(a, rank: int = 0, world: int = 1, device: Optional[torch.device] = None) -> dict:
    """The recovery stage; ``a`` carries the reference's flags (see
    ``python -m d3d_b200.pruning train --help``)."""
    from ..checkpoint import load_model, save_model
    from ..train.optim import ShardedAdamW
    from ..train.trainer import _opt_step
    from ..utils.io import write_json
    from .common import checkpoint_depth, resolve_mask_id, window_bounds
    device = device or torch.device("cpu")
    student_path = Path(a.student).resolve()
    out = Path(a.output_dir).resolve()
    if out.exists():
        raise FileExistsError(f"Refusing to overwrite {out}")
    positive = (a.max_steps, a.gradient_accumulation_steps, a.learning_rate, a.min_lr, a.save_steps, a.log_steps)
    if any(v <= 0 for v in positive):
        raise ValueError("step counts and learning rates must be positive")
    if a.data_cursor < 0 or not 0 <= a.warmup_ratio < 1 or a.candidate_multiplier < 1 or a.min_lr > a.learning_rate:
        raise ValueError("invalid data cursor, warm-up ratio, candidate multiplier or minimum learning rate")
    if a.optimizer == "adamw8bit" and a.fsdp_cpu_offload:
        raise ValueError("adamw8bit does not support CPU offload")
    if a.optimizer == "adamw8bit" and getattr(a, "fsdp", False):
        raise ValueError("8-bit optimizer moments are not kept for sharded decoder layers; use --optimizer adamw")
    meta = json.loads((student_path / "layer_prune.json").read_text())
    K = int(meta["block_size"])
    depth = int(meta["child_depth"])
    retained = [int(i) for i in meta["retained_original_layers"]]
    teacher_path = Path(meta["teacher_checkpoint"]).resolve()
    mask_id = resolve_mask_id(student_path)
    resolve_mask_id(teacher_path, mask_id)
    if checkpoint_depth(student_path) != depth or len(retained) != depth:
        raise ValueError("student config and layer-pruning metadata disagree")
    anchors = a.anchors_per_example or 2048 // K
    if anchors <= 0 or anchors * K > 2048:
        raise ValueError("anchors-per-example exceeds the 2048-token draft budget")
    rows = 0
    if str(a.dataset) != "synthetic":
        from ..train.data import JsonlIndex
        rows = len(JsonlIndex(str(a.dataset)))
    window = window_bounds(a.data_cursor, a.max_steps, a.gradient_accumulation_steps, world, a.candidate_multiplier,
                           rows or 1 << 30)
    window["seed"] = a.seed
    torch.manual_seed(a.seed + rank)
    # bf16 mixed precision on a GPU, as the reference's Accelerate run: a bf16
    # frozen teacher, fp32 student parameters and master weights, bf16 matmuls
    cuda = device.type == "cuda"
    teacher = load_model(teacher_path, device=device, mask_token_id=mask_id,
                         dtype=torch.bfloat16 if cuda else torch.float32).eval()
    for p in teacher.parameters():
        p.requires_grad_(False)
    student = load_model(student_path, device=device, mask_token_id=mask_id)
    student.train()
    freeze_io(student)
    z3 = None
    if getattr(a, "fsdp", False):
        from ..parallel.zero3 import Zero3Layers
        z3 = Zero3Layers(student.model.layers, lr=a.learning_rate, weight_decay=a.weight_decay)
    opt = ShardedAdamW(student.parameters(), lr=a.learning_rate, weight_decay=a.weight_decay,
                       state_bits=8 if a.optimizer == "adamw8bit" else 32, offload=a.fsdp_cpu_offload)
    run_config = {
        "format_version": 1, "method": "progressive_layer_pruning_fixed_budget_recovery", "mask_token_id": mask_id,
        "student": str(student_path), "teacher": str(teacher_path), "child_depth": depth,
        "retained_original_layers": retained, "block_size": K,
        "loss_weights": {"autoregressive": LAMBDA_AR, "cross_entropy": LAMBDA_CE, "kl": LAMBDA_KL, "hidden": LAMBDA_H},
        "frozen_modules": ["model.embed_tokens", "lm_head"], "max_steps": a.max_steps,
        "gradient_accumulation_steps": a.gradient_accumulation_steps, "world_size": world,
        "learning_rate": a.learning_rate, "min_lr": a.min_lr, "warmup_ratio": a.warmup_ratio,
        "optimizer": a.optimizer, "data_window": window, "dataset": str(a.dataset), "seed": a.seed,
        "sharded_layers": z3 is not None, "cpu_offload": bool(a.fsdp_cpu_offload)}
    if rank == 0:
        out.mkdir(parents=True)
        write_json(str(out / "run_config.json"), run_config)
    if dist.is_initialized():
        dist.barrier()
    data = iter(WindowData(str(a.dataset), window, rank, a.seed, tokenizer_dir=str(student_path),
                           max_prompt=a.max_prompt_tokens, max_seq=a.max_sequence_tokens, min_response=K,
                           vocab=min(student.cfg.vocab_size, 151643)))
    metrics_path = out / "training_metrics.jsonl"
    started, t_step = time.time(), time.perf_counter()
    step, micro, last = 0, 0, None

    def save(step_no: int) -> Path:
        extra = z3.full_state("model.layers.") if z3 is not None else None     # collective
        dst = out / f"step-{step_no}"
        if rank == 0:
            if dst.exists():
                raise FileExistsError(f"Refusing to overwrite {dst}")
            tmp = Path(tempfile.mkdtemp(prefix=f".{dst.name}.", dir=out))
            try:
                save_model(student, tmp / "m", extra=extra)
                for f in (tmp / "m").iterdir():
                    os.replace(f, tmp / f.name)
                (tmp / "m").rmdir()
                _copy_support(student_path, tmp)
                shutil.copy2(student_path / "layer_prune.json", tmp / "layer_prune.json")
                write_json(str(tmp / "recovery_info.json"), {**run_config, "optimizer_step": step_no,
                                                             "checkpoint": str(dst)})
                os.replace(tmp, dst)
            except BaseException:
                shutil.rmtree(tmp, ignore_errors=True)
                raise
        if dist.is_initialized():
            dist.barrier()
        return dst

    while step < a.max_steps:
        pos, ex = _next_together(data, device)
        batch = build_packed_block_batch([ex], block_size=K, mask_token_id=mask_id, max_anchors=anchors,
                                         rng=random.Random(f"d3d-prune-{a.seed}-{pos}"), full_blocks=True)
        if batch is None:
            continue
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=cuda):
            terms = recovery_losses(student, teacher, retained, batch.to(device),
                                    torch.tensor([len(ex.prompt_ids)]))
        loss = (LAMBDA_AR * terms["autoregressive_loss"] + LAMBDA_CE * terms["cross_entropy"]
                + LAMBDA_KL * terms["kl"] + LAMBDA_H * terms["hidden"])
        (loss / a.gradient_accumulation_steps).backward()
        micro += 1
        if micro % a.gradient_accumulation_steps:
            continue
        step += 1
        lr = learning_rate(step, a.max_steps, a.learning_rate, a.min_lr, a.warmup_ratio)
        gnorm = _opt_step(opt, z3, a.gradient_clip, lr)
        opt.zero_grad()
        rec = {"optimizer_step": step, "loss": _dist_mean(loss)}
        for k in ("autoregressive_loss", "cross_entropy", "kl", "hidden", "student_accept_length",
                  "teacher_accept_length"):
            rec[k] = _dist_mean(terms[k])
        rec.update(learning_rate=lr, gradient_norm=float(gnorm), step_seconds=time.perf_counter() - t_step,
                   elapsed_seconds=time.time() - started, virtual_position=int(pos))
        if rank == 0:
            with metrics_path.open("a") as f:
                f.write(json.dumps(rec) + "\n")
            if step % a.log_steps == 0:
                print(json.dumps(rec), flush=True)
        if step % a.save_steps == 0 or step == a.max_steps:
            last = save(step)
        t_step = time.perf_counter()
    summary = {**run_config, "completed_steps": step, "next_data_cursor": window["cursor_end"],
               "final_checkpoint": str(last), "elapsed_seconds": time.time() - started}
    if rank == 0:
        write_json(str(out / "training_summary.json"), summary)
    if z3 is not None:
        z3.close()
    return summary
