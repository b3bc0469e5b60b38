"""Sharded AdamW with fp32 master weights (ZeRO-style data parallelism).

The reference trains with Accelerate FSDP2 (bf16 params, fp32 master via
AdamW, ``train/runtime.py:70-114``).  Here every rank computes in bf16 with a
full copy of the drafter (1.7B parameters = 3.4 GB, small next to 180 GB of
HBM), while the fp32 master weights, both Adam moments and the gradients are
sharded across ranks:

1. after backward the bf16/fp32 gradients of all parameters are flattened
   into one buffer (per bucket) and **reduce-scattered** (sum) so each rank
   holds the gradient of its own contiguous shard;
2. the global gradient norm is the all-reduced sum of the shards' squared
   norms (``sumsq`` kernel) → clip coefficient;
3. the fused **AdamW** kernel updates the fp32 master shard, folding the
   1/world mean and the clip coefficient into one gradient scale, and writes
   the updated shard in bf16;
4. the bf16 shards are **all-gathered** back into every rank's compute
   parameters.

On CPU (tests, ``gloo``) steps 2-3 run in PyTorch with the same arithmetic.
"""
from __future__ import annotations

import math
from typing import Iterable, List, Optional

import torch
import torch.distributed as dist


class ShardedAdamW:
    def __init__(self, params: Iterable[torch.nn.Parameter], lr: float = 1e-4, betas=(0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.0, group=None, align: int = 1):
        self.params: List[torch.nn.Parameter] = [p for p in params if p.requires_grad]
        self.lr, self.b1, self.b2, self.eps, self.wd = lr, betas[0], betas[1], eps, weight_decay
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.numel = sum(p.numel() for p in self.params)
        self.shard = math.ceil(self.numel / (self.world * align)) * align
        self.padded = self.shard * self.world
        dev = self.params[0].device
        flat = torch.zeros(self.padded, dtype=torch.float32, device=dev)
        off = 0
        for p in self.params:
            flat[off:off + p.numel()] = p.detach().reshape(-1).float()
            off += p.numel()
        lo = self.rank * self.shard
        self.master = flat[lo:lo + self.shard].clone()
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.step_count = 0
        self.last_grad_norm = 0.0
        self.last_scale = 1.0 / self.world

    def zero_grad(self) -> None:
        for p in self.params:
            p.grad = None

    def _flat_grads(self) -> torch.Tensor:
        dev = self.master.device
        g = torch.zeros(self.padded, dtype=torch.float32, device=dev)
        off = 0
        for p in self.params:
            if p.grad is not None:
                g[off:off + p.numel()] = p.grad.reshape(-1).float()
            off += p.numel()
        return g

    @torch.no_grad()
    def step(self, grad_clip: float = 0.0, lr: Optional[float] = None,
             extra_sumsq: Optional[torch.Tensor] = None) -> float:
        """One AdamW step; returns the global gradient norm.  ``extra_sumsq``
        is this rank's squared norm of gradients updated elsewhere (sharded
        decoder layers): it joins the norm, and the gradient scale applied
        here (1/world times the clip factor) is left in ``last_scale`` for
        that other update."""
        lr = self.lr if lr is None else lr
        self.step_count += 1
        g = self._flat_grads()
        if self.world > 1:
            gs = torch.empty(self.shard, dtype=torch.float32, device=g.device)
            dist.reduce_scatter_tensor(gs, g, op=dist.ReduceOp.SUM, group=self.group)
        else:
            gs = g[: self.shard]
        mean = 1.0 / self.world
        cuda = gs.is_cuda
        if cuda:
            from .. import ops
            sq = torch.zeros(1, device=gs.device)
            ops.ext().sumsq(gs, sq)
        else:
            sq = (gs.double() ** 2).sum().float().reshape(1)
        if extra_sumsq is not None:
            sq = sq + extra_sumsq.to(sq.device)
        if self.world > 1:
            dist.all_reduce(sq, group=self.group)
        norm = math.sqrt(float(sq.item())) * mean
        self.last_grad_norm = norm
        clip = 1.0
        if grad_clip and grad_clip > 0 and norm > grad_clip:
            clip = grad_clip / (norm + 1e-6)
        scale = mean * clip
        self.last_scale = scale
        out = torch.empty(self.shard, dtype=torch.bfloat16, device=gs.device)
        if cuda:
            from .. import ops
            ops.ext().adamw(self.master, gs.contiguous(), self.m, self.v, out, lr, self.b1, self.b2, self.eps,
                            self.wd, self.step_count, scale)
        else:
            gi = gs * scale
            self.m.mul_(self.b1).add_(gi, alpha=1 - self.b1)
            self.v.mul_(self.b2).addcmul_(gi, gi, value=1 - self.b2)
            bc1 = 1 - self.b1 ** self.step_count
            bc2 = 1 - self.b2 ** self.step_count
            self.master.mul_(1 - lr * self.wd)
            self.master.addcdiv_(self.m / bc1, (self.v / bc2).sqrt().add_(self.eps), value=-lr)
            out.copy_(self.master)
        full = torch.empty(self.padded, dtype=torch.bfloat16 if cuda else torch.float32, device=gs.device)
        src = out if cuda else self.master
        if self.world > 1:
            dist.all_gather_into_tensor(full, src, group=self.group)
        else:
            full[: self.shard] = src
        off = 0
        for p in self.params:
            p.data.copy_(full[off:off + p.numel()].view_as(p).to(p.dtype))
            off += p.numel()
        return norm

    # ------------------------------------------------------------ resume
    def state_dict(self) -> dict:
        return {"master": self.master.cpu(), "m": self.m.cpu(), "v": self.v.cpu(), "step": self.step_count,
                "rank": self.rank, "world": self.world, "numel": self.numel}

    def load_state_dict(self, sd: dict) -> None:
        if sd["world"] != self.world or sd["numel"] != self.numel:
            raise ValueError("optimizer shard layout does not match this run")
        self.master.copy_(sd["master"])
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])
        self.step_count = int(sd["step"])


def cosine_lr(step: int, base: float, warmup: int, total: int, min_ratio: float = 0.0) -> float:
    """Linear warm-up then cosine decay (``train/runtime.py:168-187``)."""
    if warmup > 0 and step < warmup:
        return base * (step + 1) / warmup
    if total <= warmup:
        return base
    prog = min(1.0, (step - warmup) / max(1, total - warmup))
    return base * (min_ratio + (1 - min_ratio) * 0.5 * (1 + math.cos(math.pi * prog)))
