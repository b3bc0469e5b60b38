"""Distillation objectives (reference: ``train/losses.py``,
``train/objective_kernels.py``).

* Objective names and aliases, position-decayed weights
  ``exp(-(offset-1)/gamma)`` over block offsets.
* Per-token CE / forward KL / reverse KL in PyTorch (the oracle).
* :func:`lmhead_distill_loss`: the LM-head projection fused with forward-KL
  (teacher logits from the frozen target's hidden states and LM head) plus
  CE, over vocabulary chunks, never materialising ``[N, V]`` logits.  On
  CUDA the chunk logits come from the tcgen05 GEMM and the reductions /
  gradients from ``kl_ce_stats`` / ``kl_ce_grad``; the backward recomputes
  the chunk logits.  On CPU the same chunked algorithm runs in PyTorch.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

OBJECTIVE_ALIASES = {"ce": "ce", "hard_ce": "ce", "kl": "forward_kl", "fkl": "forward_kl",
                     "forward_kl": "forward_kl", "forward-kl": "forward_kl", "rkl": "reverse_kl",
                     "reverse_kl": "reverse_kl", "reverse-kl": "reverse_kl", "kl_ce": "kl_ce"}


def normalize_objective(name: str) -> str:
    key = str(name).lower()
    if key not in OBJECTIVE_ALIASES:
        raise ValueError(f"objective must be one of {sorted(OBJECTIVE_ALIASES)}, got {name!r}")
    return OBJECTIVE_ALIASES[key]


def decay_weights(offsets: torch.Tensor, gamma: float = 15.5) -> torch.Tensor:
    return torch.exp(-(offsets.float() - 1).clamp(min=0) / float(gamma))


def forward_kl_per_token(student_logits, teacher_logits):
    with torch.no_grad():
        tl = F.log_softmax(teacher_logits.float(), -1)
        tp = tl.exp()
    return (tp * (tl - F.log_softmax(student_logits.float(), -1))).sum(-1)


def reverse_kl_per_token(student_logits, teacher_logits):
    with torch.no_grad():
        tl = F.log_softmax(teacher_logits.float(), -1)
    sl = F.log_softmax(student_logits.float(), -1)
    return (sl.exp() * (sl - tl)).sum(-1)


def ce_per_token(student_logits, targets):
    return F.cross_entropy(student_logits.float(), targets.long(), reduction="none")


def _nontarget_topk(logits: torch.Tensor, targets: torch.Tensor, k: int):
    """Target logit and the ``k`` largest non-target logits of each row."""
    z = logits.float()
    k = min(int(k), z.shape[-1] - 1)
    zt = z.gather(-1, targets.long()[:, None])[:, 0]
    v, i = torch.topk(z, k + 1, dim=-1)
    v = v.masked_fill(i == targets.long()[:, None], float("-inf"))
    return zt, torch.topk(v, k, dim=-1).values


def hard_negative_ce_per_token(logits, targets, top_k: int = 16, margin: float = 0.0):
    """CE of the target against only its ``top_k`` strongest competitors
    (each shifted by ``margin``): ``log(1 + sum_j exp(z_j + margin - z_y))``
    (reference ``train/objective_kernels.py:102-148``)."""
    zt, neg = _nontarget_topk(logits, targets, top_k)
    terms = torch.cat([torch.zeros_like(zt)[:, None], neg - zt[:, None] + float(margin)], -1)
    return torch.logsumexp(terms, -1)


def target_margin_per_token(logits, targets, top_k: int = 16, margin: float = 1.0, smooth: bool = True,
                            temperature: float = 1.0):
    """Mean penalty of the ``top_k`` strongest competitors that come within
    ``margin`` of the target logit: softplus (smooth) or hinge
    (reference ``train/objective_kernels.py:41-98``)."""
    zt, neg = _nontarget_topk(logits, targets, top_k)
    viol = neg - zt[:, None] + float(margin)
    if smooth:
        pen = F.softplus(viol / float(temperature)) * float(temperature)
    else:
        pen = F.relu(viol)
    return pen.mean(-1)


def ce_aux_per_token(logits, targets, *, ce_weight=1.0, hnce_weight=0.0, hnce_top_k=16, hnce_margin=0.0,
                     margin_weight=0.0, margin_top_k=16, margin_value=1.0, margin_smooth=True):
    """``ce_weight * CE + hnce_weight * hard-negative CE + margin_weight *
    margin`` per token, plus the three terms (reference ``train/losses.py:124-159``)."""
    ce = ce_per_token(logits, targets)
    hn = hard_negative_ce_per_token(logits, targets, hnce_top_k, hnce_margin) if hnce_weight else \
        torch.zeros_like(ce)
    mg = target_margin_per_token(logits, targets, margin_top_k, margin_value, margin_smooth) if margin_weight \
        else torch.zeros_like(ce)
    return ce_weight * ce + hnce_weight * hn + margin_weight * mg, ce, hn, mg


# --------------------------------------------------------------------------
# fused LM-head KL + CE
# --------------------------------------------------------------------------
_ST_N = 8


def _chunk_logits(h: torch.Tensor, w: torch.Tensor, v0: int, c: int, buf: Optional[torch.Tensor]):
    if h.is_cuda:
        from .. import ops
        out = buf[: h.shape[0] * c].view(h.shape[0], c)
        ops.ext().gemm_partial(h, w[v0:v0 + c], out, 1, ops.bt_for(h.shape[0]), None, 0)
        return out
    return h.float() @ w[v0:v0 + c].float().t()


def _stats(hs, ws, ht, wt, tgt, chunk):
    """Per-row [M_t, S_t, A_tt, A_ts, M_s, S_s, z_tgt] over the vocabulary."""
    N, V = hs.shape[0], ws.shape[0]
    st = torch.zeros(N, _ST_N, device=hs.device)
    st[:, 0] = -math.inf
    st[:, 4] = -math.inf
    cuda = hs.is_cuda
    bs = torch.empty(N * chunk, device=hs.device) if cuda else None
    bt = torch.empty(N * chunk, device=hs.device) if (cuda and ht is not None) else None
    for v0 in range(0, V, chunk):
        c = min(chunk, V - v0)
        zs = _chunk_logits(hs, ws, v0, c, bs)
        zt = _chunk_logits(ht, wt, v0, c, bt) if ht is not None else None
        if cuda:
            from .. import ops
            ops.ext().kl_ce_stats(zt, zs, c, v0, tgt, st)
            continue
        if zt is not None:
            mt = zt.max(-1).values
            nm = torch.maximum(st[:, 0], mt)
            fo = torch.where(st[:, 0] == -math.inf, torch.zeros_like(nm), torch.exp(st[:, 0] - nm))
            e = torch.exp(zt - nm[:, None])
            st[:, 1] = st[:, 1] * fo + e.sum(-1)
            st[:, 2] = st[:, 2] * fo + (e * zt).sum(-1)
            st[:, 3] = st[:, 3] * fo + (e * zs).sum(-1)
            st[:, 0] = nm
        ms = zs.max(-1).values
        nm = torch.maximum(st[:, 4], ms)
        fo = torch.where(st[:, 4] == -math.inf, torch.zeros_like(nm), torch.exp(st[:, 4] - nm))
        st[:, 5] = st[:, 5] * fo + torch.exp(zs - nm[:, None]).sum(-1)
        st[:, 4] = nm
        if tgt is not None:
            inr = (tgt >= v0) & (tgt < v0 + c)
            if bool(inr.any()):
                idx = inr.nonzero(as_tuple=True)[0]
                st[idx, 6] = zs[idx, tgt[idx] - v0]
    return st


class _FusedLMHeadLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hs, ws, ht, wt, tgt, w_kl, w_ce, chunk):
        st = _stats(hs, ws, ht, wt, tgt, chunk)
        lse_s = st[:, 4] + torch.log(st[:, 5])
        lse_t = st[:, 0] + torch.log(st[:, 1]) if ht is not None else torch.zeros_like(lse_s)
        kl = (st[:, 2] - st[:, 3]) / st[:, 1] - lse_t + lse_s if ht is not None else torch.zeros_like(lse_s)
        ce = lse_s - st[:, 6]
        loss = torch.zeros((), device=hs.device)
        if w_kl is not None and ht is not None:
            loss = loss + (w_kl * kl).sum()
        if w_ce is not None:
            loss = loss + (w_ce * ce).sum()
        ctx.save_for_backward(hs, ws, ht if ht is not None else torch.empty(0),
                              wt if wt is not None else torch.empty(0),
                              tgt if tgt is not None else torch.empty(0, dtype=torch.long),
                              w_kl if w_kl is not None else torch.empty(0),
                              w_ce if w_ce is not None else torch.empty(0), lse_t, lse_s)
        ctx.chunk = chunk
        ctx.has_t = ht is not None
        ctx.mark_non_differentiable(kl, ce)
        return loss, kl.detach(), ce.detach()

    @staticmethod
    def backward(ctx, g, _gk, _gc):
        hs, ws, ht, wt, tgt, w_kl, w_ce, lse_t, lse_s = ctx.saved_tensors
        has_t = ctx.has_t
        tgt = tgt if tgt.numel() else None
        wkl = (w_kl * g).float().contiguous() if (w_kl.numel() and has_t) else None
        wce = (w_ce * g).float().contiguous() if w_ce.numel() else None
        N, Hs = hs.shape
        V = ws.shape[0]
        chunk = ctx.chunk
        need_w = ctx.needs_input_grad[1]
        dh = torch.zeros(N, Hs, device=hs.device, dtype=torch.float32)
        dw = torch.zeros(V, Hs, device=hs.device, dtype=torch.float32) if need_w else None
        cuda = hs.is_cuda
        if cuda:
            from .. import ops
            E = ops.ext()
            bs = torch.empty(N * chunk, device=hs.device)
            bt = torch.empty(N * chunk, device=hs.device) if has_t else None
            npad = (N + 63) // 64 * 64
            hsT = torch.zeros(Hs, npad, dtype=torch.bfloat16, device=hs.device)
            hsT[:, :N] = hs.t()
            dz = torch.empty(N, chunk, dtype=torch.bfloat16, device=hs.device)
            dzT = torch.zeros(chunk, npad, dtype=torch.bfloat16, device=hs.device)
            dwc = torch.empty(chunk * Hs, device=hs.device)
            # dh = dz @ W contracts over the vocabulary: the tcgen05 GEMM reads
            # W transposed ([Hs, V], made once per backward), each chunk a
            # column window of it
            tc_dh = V % 8 == 0 and chunk % 8 == 0 and Hs % 8 == 0    # 16-byte TMA rows
            wsT = ws.t().contiguous() if tc_dh else None
            dhc = torch.empty(N * Hs, device=hs.device)
        for v0 in range(0, V, chunk):
            c = min(chunk, V - v0)
            zs = _chunk_logits(hs, ws, v0, c, bs if cuda else None)
            zt = _chunk_logits(ht, wt, v0, c, bt if cuda else None) if has_t else None
            if cuda:
                E.kl_ce_grad(zt, zs, c, v0, tgt, lse_t, lse_s, wkl, wce, dz[:, :c], dzT[:c] if need_w else None)
                if tc_dh:
                    E.gemm_partial(dz[:, :c], wsT[:, v0:v0 + c], dhc, 1, ops.bt_for(N), None, 0)
                    dh += dhc.view(N, Hs)
                else:
                    dh += (dz[:, :c] @ ws[v0:v0 + c]).float()
                if need_w:
                    out = dwc[: c * Hs].view(c, Hs)
                    E.gemm_partial(dzT[:c], hsT, out, 1, ops.bt_for(c), None, 0)
                    dw[v0:v0 + c] = out
                continue
            ps = torch.exp(zs - lse_s[:, None])
            gz = torch.zeros_like(zs)
            if wkl is not None:
                gz += wkl[:, None] * (ps - torch.exp(zt - lse_t[:, None]))
            if wce is not None:
                oh = torch.zeros_like(zs)
                if tgt is not None:
                    inr = (tgt >= v0) & (tgt < v0 + c)
                    idx = inr.nonzero(as_tuple=True)[0]
                    oh[idx, tgt[idx] - v0] = 1.0
                gz += wce[:, None] * (ps - oh)
            dh += gz @ ws[v0:v0 + c].float()
            if need_w:
                dw[v0:v0 + c] = gz.t() @ hs.float()
        return (dh.to(hs.dtype), None if dw is None else dw.to(ws.dtype), None, None, None, None, None, None)


def lmhead_distill_loss(h_s: torch.Tensor, w_s: torch.Tensor, h_t: Optional[torch.Tensor],
                        w_t: Optional[torch.Tensor], targets: Optional[torch.Tensor],
                        w_kl: Optional[torch.Tensor], w_ce: Optional[torch.Tensor], chunk: int = 16384
                        ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``sum_n w_kl[n] KL(p_t || p_s)[n] + w_ce[n] CE[n]`` with ``p_s`` from
    ``h_s @ w_s.T`` and ``p_t`` from ``h_t @ w_t.T``.  Returns the weighted sum
    and the per-row KL and CE (detached)."""
    if h_s.is_cuda:
        h_s = h_s.contiguous()
        if h_t is not None:
            h_t = h_t.to(torch.bfloat16).contiguous()
    return _FusedLMHeadLoss.apply(h_s, w_s, h_t, w_t, targets, w_kl, w_ce, int(chunk))
