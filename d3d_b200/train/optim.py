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


QBLOCK = 256          # elements per quantization block of 8-bit moments


def quantize_signed(x: torch.Tensor):
    """8-bit code of a signed fp32 vector, blockwise: per block of ``QBLOCK``
    the absolute maximum, and per element ``round(127 * sign * sqrt(|x| /
    max))`` -- square-root companding spends the codes on the small values
    that dominate a first moment.  Returns ``(int8 codes, fp32 scales)``."""
    n = x.numel()
    pad = (-n) % QBLOCK
    xb = torch.nn.functional.pad(x.float(), (0, pad)).view(-1, QBLOCK)
    scale = xb.abs().amax(1).clamp_min(1e-30)
    code = torch.round(127.0 * torch.sign(xb) * torch.sqrt(xb.abs() / scale[:, None]))
    return code.to(torch.int8).view(-1)[:n], scale


def dequantize_signed(code: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    n = code.numel()
    pad = (-n) % QBLOCK
    c = torch.nn.functional.pad(code.float(), (0, pad)).view(-1, QBLOCK) / 127.0
    return (torch.sign(c) * c.square() * scale[:, None]).view(-1)[:n]


def quantize_positive(x: torch.Tensor):
    """8-bit code of a non-negative fp32 vector (a second moment), blockwise:
    per block its maximum, and per element ``round(255 * (x / max) ** (1/4))``
    -- fourth-root companding keeps small second moments away from zero,
    where a plain linear code would round them to 0 and blow up the update."""
    n = x.numel()
    pad = (-n) % QBLOCK
    xb = torch.nn.functional.pad(x.float(), (0, pad)).view(-1, QBLOCK)
    scale = xb.amax(1).clamp_min(1e-30)
    code = torch.round(255.0 * torch.sqrt(torch.sqrt((xb / scale[:, None]).clamp(0, 1))))
    return code.to(torch.uint8).view(-1)[:n], scale


def dequantize_positive(code: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    n = code.numel()
    pad = (-n) % QBLOCK
    c = torch.nn.functional.pad(code.float(), (0, pad)).view(-1, QBLOCK) / 255.0
    return (c.square().square() * scale[:, None]).view(-1)[:n]


class ShardedAdamW:
    """``state_bits=8`` keeps both Adam moments as blockwise-quantized 8-bit
    codes (2 bytes per parameter instead of 8; the update itself runs in
    fp32 on the dequantized shard).  ``offload=True`` keeps the fp32 master
    shard and the moments in host memory and runs the update on the CPU
    (the gradient shard goes down, the updated weights come back up)."""

    def __init__(self, params: Iterable[torch.nn.Parameter], lr: float = 1e-4, betas=(0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.0, group=None, align: int = 1,
                 state_bits: int = 32, offload: bool = False):
        if state_bits not in (8, 32):
            raise ValueError("state_bits must be 8 or 32")
        if state_bits == 8 and offload:
            raise ValueError("8-bit moments do not combine with host offload")
        self.state_bits, self.offload = state_bits, bool(offload)
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
        if self.offload:
            self.master = self.master.cpu().pin_memory() if dev.type == "cuda" else self.master.cpu()
        if self.state_bits == 8:
            self.m = quantize_signed(torch.zeros(self.shard, device=dev))
            self.v = quantize_positive(torch.zeros(self.shard, device=dev))
        else:
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
        if cuda and self.state_bits == 32 and not self.offload:
            from .. import ops
            ops.ext().adamw(self.master, gs.contiguous(), self.m, self.v, out, lr, self.b1, self.b2, self.eps,
                            self.wd, self.step_count, scale)
        else:
            m = dequantize_signed(*self.m) if self.state_bits == 8 else self.m
            v = dequantize_positive(*self.v) if self.state_bits == 8 else self.v
            gi = gs.to(self.master.device, non_blocking=True) * scale
            m.mul_(self.b1).add_(gi, alpha=1 - self.b1)
            v.mul_(self.b2).addcmul_(gi, gi, value=1 - self.b2)
            bc1 = 1 - self.b1 ** self.step_count
            bc2 = 1 - self.b2 ** self.step_count
            self.master.mul_(1 - lr * self.wd)
            self.master.addcdiv_(m / bc1, (v / bc2).sqrt().add_(self.eps), value=-lr)
            if self.state_bits == 8:
                self.m, self.v = quantize_signed(m), quantize_positive(v)
            out.copy_(self.master, non_blocking=True)
        full = torch.empty(self.padded, dtype=torch.bfloat16 if cuda else torch.float32, device=gs.device)
        src = out if cuda else self.master.to(gs.device)
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
        cpu = (lambda t: tuple(x.cpu() for x in t)) if self.state_bits == 8 else (lambda t: t.cpu())
        return {"master": self.master.cpu(), "m": cpu(self.m), "v": cpu(self.v), "step": self.step_count,
                "rank": self.rank, "world": self.world, "numel": self.numel, "state_bits": self.state_bits}

    def load_state_dict(self, sd: dict) -> None:
        if sd["world"] != self.world or sd["numel"] != self.numel:
            raise ValueError("optimizer shard layout does not match this run")
        if int(sd.get("state_bits", 32)) != self.state_bits:
            raise ValueError("optimizer state precision does not match this run")
        self.master.copy_(sd["master"])
        if self.state_bits == 8:
            dev = self.m[0].device
            self.m = tuple(x.to(dev) for x in sd["m"])
            self.v = tuple(x.to(dev) for x in sd["v"])
        else:
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
