"""Recovery objectives (reference: ``pruning/losses.py``).

* ``corrected_kl``: KL from a teacher distribution that is moved toward the
  target token just enough for the target to lead the best other token by
  ``margin`` (``pruning/losses.py:59-118``);
* ``target_ce``: cross-entropy of the target tokens;
* ``boundary_hidden_mse``: RMS-normalised hidden-state MSE at the layer
  boundary where the pruned student should reproduce the teacher's output of
  the deleted layer (``pruning/losses.py:121-165``);
* ``masked_mean`` with an optional distributed normaliser.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F


def masked_mean(values: torch.Tensor, weights: torch.Tensor, distributed: bool = False) -> torch.Tensor:
    num = (values * weights).sum()
    den = weights.sum().detach()
    if distributed and dist.is_initialized():
        den = den.clone()
        dist.all_reduce(den)
        return num * dist.get_world_size() / den.clamp_min(1e-8)
    return num / den.clamp_min(1e-8)


def corrected_kl(student_logits, teacher_logits, targets, temperature: float = 1.0, margin: float = 0.01):
    s = F.log_softmax(student_logits.float() / temperature, -1)
    tp = F.softmax(teacher_logits.detach().float() / temperature, -1)
    tgt_p = tp.gather(-1, targets[:, None])[:, 0]
    top2 = torch.topk(tp, 2, -1)
    other = torch.where(top2.indices[:, 0].eq(targets), top2.values[:, 1], top2.values[:, 0])
    deficit = other - tgt_p
    corr = ((deficit + margin) / (1.0 + deficit).clamp_min(1e-8)).clamp(0.0, 1.0)
    q = (tp * (1.0 - corr[:, None])).scatter_add(-1, targets[:, None], corr[:, None])
    return (q * (q.clamp_min(1e-30).log() - s)).sum(-1) * temperature ** 2


def target_ce(logits, targets):
    return F.cross_entropy(logits.float(), targets.long(), reduction="none")


def boundary_hidden_mse(student, teacher, eps: float = 1e-6):
    a = student.float() * torch.rsqrt(student.float().square().mean(-1, keepdim=True) + eps)
    b = teacher.float() * torch.rsqrt(teacher.float().square().mean(-1, keepdim=True) + eps)
    return (a - b).square().mean(-1)
