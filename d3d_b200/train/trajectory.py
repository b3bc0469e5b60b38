"""Hidden-trajectory distillation (optional, off by default).

Teacher (8B) and student (1.7B) hidden widths differ, so the two models'
hidden states are not compared directly: within each packed block the
cosine-similarity matrix of the rows' hidden states (a width-free "shape" of
the block's trajectory) is matched, SmoothL1 over the off-diagonal pairs of
the block's valid rows.  Only blocks where the teacher drafts better than the
student (or both draft the whole block) contribute.  Reference:
``train/trajectory.py:16-294`` (selection, relation matrices, per-block
mean, distributed normalisation).

Shapes: ``[B, NB, K, ...]`` -- sequences x blocks x block rows.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F


def block_accept_lengths(pred: torch.Tensor, target: torch.Tensor, valid: torch.Tensor) -> torch.Tensor:
    """Leading run of correct predictions per block: ``pred``, ``target``,
    ``valid`` are [B, NB, L] (L = supervised rows of a block)."""
    ok = (pred == target) & valid
    return ok.long().cumprod(-1).sum(-1)


def selection_mask(teacher_acc: torch.Tensor, student_acc: torch.Tensor, active_len: torch.Tensor,
                   keep: torch.Tensor) -> torch.Tensor:
    """Blocks the teacher drafts further than the student, or both fully."""
    both_full = (teacher_acc == active_len) & (student_acc == active_len)
    return ((teacher_acc > student_acc) | both_full) & keep.bool()


def relation(h: torch.Tensor) -> torch.Tensor:
    """Cosine-similarity matrix of every block's rows: [B, NB, K, D] -> [B, NB, K, K]."""
    u = F.normalize(h.float(), dim=-1)
    return u @ u.transpose(-1, -2)


def shuffle_among_equal_length(rt: torch.Tensor, selected: torch.Tensor, active_len: torch.Tensor,
                               gen: torch.Generator) -> torch.Tensor:
    """Teacher relation matrices permuted among the selected blocks that have
    the same number of valid rows (the reference's negative control: the
    targets keep their shape statistics but lose their pairing)."""
    k = rt.shape[-1]
    flat = rt.reshape(-1, k, k)
    sel = selected.reshape(-1).bool()
    ln = active_len.reshape(-1)
    out = flat.clone()
    for length in torch.unique(ln[sel]).tolist():
        idx = torch.nonzero(sel & (ln == length), as_tuple=True)[0]
        perm = torch.randperm(len(idx), generator=gen).to(idx.device)
        out[idx] = flat[idx[perm]]
    return out.view_as(rt)


def relational_loss(student_h: torch.Tensor, teacher_h: torch.Tensor, valid: torch.Tensor,
                    selected: torch.Tensor, shuffle: Optional[torch.Generator] = None):
    """Sum over selected blocks of the mean SmoothL1 between the student's and
    the (detached) teacher's relation matrices over off-diagonal valid pairs.
    Returns ``(loss_sum, selected_count)``; divide by the global count.
    ``shuffle``: permute the teacher targets among selected blocks of equal
    active length first (:func:`shuffle_among_equal_length`)."""
    rs = relation(student_h)
    rt = relation(teacher_h.detach())
    if shuffle is not None:
        rt = shuffle_among_equal_length(rt, selected, valid.sum(-1), shuffle)
    k = rs.shape[-1]
    pair = valid.unsqueeze(-1) & valid.unsqueeze(-2) & ~torch.eye(k, dtype=torch.bool, device=rs.device)
    per_pair = F.smooth_l1_loss(rs, rt, reduction="none") * pair
    per_block = per_pair.sum((-1, -2)) / pair.sum((-1, -2)).clamp_min(1)
    sel = selected.bool() & (pair.sum((-1, -2)) > 0)
    return (per_block * sel).sum(), sel.sum()


def distributed_block_mean(local_sum: torch.Tensor, global_count: float, world: int) -> torch.Tensor:
    """Scale a rank's block-loss sum so that data-parallel gradient averaging
    over ``world`` ranks yields the mean over all ranks' selected blocks."""
    if global_count <= 0:
        return local_sum * 0.0
    return local_sum * (float(world) / float(global_count))


def by_block(x: torch.Tensor, block_size: int) -> torch.Tensor:
    """[B, NB*K, ...] -> [B, NB, K, ...]."""
    b, q = x.shape[:2]
    return x.reshape(b, q // block_size, block_size, *x.shape[2:])
