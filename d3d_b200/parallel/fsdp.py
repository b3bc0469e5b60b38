"""Sharded AdamW whose collectives are fused into its kernels (NVLink peer
memory instead of NCCL).

Same arithmetic and state layout as :class:`~d3d_b200.train.optim.ShardedAdamW`
(fp32 master weights and moments sharded over ranks, bf16 compute copies
everywhere), but the step is

1. copy this rank's gradients into its IPC-mapped fp32 gradient buffer and
   publish "gradients of step e ready" (system-scope release flag on every
   rank);
2. ``fsdp_reduce``: after bounded waits on every rank's flag, sum this
   rank's shard over all ranks' gradient buffers (peer loads, rank order) and
   its squared norm -- the reduce-scatter;
3. the global norm is one scalar all-reduce (clipping);
4. ``fsdp_update``: AdamW on the shard, bf16 cast, and peer stores of the
   new shard into every rank's parameter buffer -- the all-gather -- with the
   kernel's last CTA publishing "shard of step e written";
5. a bounded wait for every rank's shard, then the parameters are refreshed
   from the local bf16 buffer.

The reference trains with FSDP2 through Accelerate (``train/runtime.py:70-114``).
"""
from __future__ import annotations

import math
from typing import Iterable, List, Optional

import torch
import torch.distributed as dist

from .. import ops
from ..train.optim import ShardedAdamW

_FLAG_BYTES = 2 * 8 * 8   # [phase][source rank] int64, up to 8 ranks


class FusedShardedAdamW(ShardedAdamW):
    def __init__(self, params: Iterable[torch.nn.Parameter], lr: float = 1e-4, betas=(0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.0, group=None):
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, group=group, align=4)
        if self.world > 8:
            raise ValueError("the fused sharded optimizer supports up to 8 ranks")
        dev = self.master.device
        if dev.type != "cuda":
            raise ValueError("the fused sharded optimizer needs CUDA parameters")
        self.device = dev
        E = ops.ext()
        self.ext = E
        gb = (4 * self.padded + 255) // 256 * 256
        pb = (2 * self.padded + 255) // 256 * 256
        self.nbytes = _FLAG_BYTES + gb + pb
        self.base = E.mailbox_alloc(self.nbytes, dev.index)
        mem = E.mailbox_view(self.base, self.nbytes, dev.index)
        self.grad_flat = mem[_FLAG_BYTES:_FLAG_BYTES + 4 * self.padded].view(torch.float32)
        self.param_flat = mem[_FLAG_BYTES + gb:_FLAG_BYTES + gb + 2 * self.padded].view(torch.bfloat16)
        handles: List = [None] * self.world
        dist.all_gather_object(handles, (self.rank, E.ipc_handle(self.base, dev.index)), group=group)
        by_rank = dict(handles)
        bases, self._opened = [], []
        for r in range(self.world):
            if r == self.rank:
                bases.append(self.base)
            else:
                p = E.ipc_open(by_rank[r], dev.index)
                self._opened.append(p)
                bases.append(p)
        self.ptrs = torch.tensor([[b + _FLAG_BYTES for b in bases],
                                  [b + _FLAG_BYTES + gb for b in bases],
                                  bases], dtype=torch.int64)
        self.lo = self.rank * self.shard
        self.gshard = torch.zeros(self.shard, dtype=torch.float32, device=dev)
        self.sq = torch.zeros(1, dtype=torch.float32, device=dev)
        self.ticket = torch.zeros(1, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.closed = False

    @torch.no_grad()
    def step(self, grad_clip: float = 0.0, lr: Optional[float] = None,
             extra_sumsq: Optional[torch.Tensor] = None) -> float:
        lr = self.lr if lr is None else lr
        self.step_count += 1
        e = self.step_count
        E, P = self.ext, self.ptrs
        g = self.grad_flat
        off = 0
        for p in self.params:
            n = p.numel()
            if p.grad is not None:
                g[off:off + n].copy_(p.grad.reshape(-1))
            else:
                g[off:off + n].zero_()
            off += n
        E.fsdp_signal(P, self.rank, self.lo, self.shard, 0, e, self.sq)
        self.sq.zero_()
        E.fsdp_reduce(P, self.rank, self.lo, self.shard, e, self.gshard, self.sq, self.status)
        sq = self.sq.clone()
        if extra_sumsq is not None:
            sq += extra_sumsq
        if self.world > 1:
            dist.all_reduce(sq, group=self.group)
        mean = 1.0 / self.world
        norm = math.sqrt(float(sq.item())) * mean
        self.last_grad_norm = norm
        clip = 1.0
        if grad_clip and grad_clip > 0 and norm > grad_clip:
            clip = grad_clip / (norm + 1e-6)
        self.last_scale = mean * clip
        E.fsdp_update(P, self.rank, self.lo, self.shard, e, self.gshard, self.master, self.m, self.v, lr,
                      self.b1, self.b2, self.eps, self.wd, self.step_count, mean * clip, self.ticket, self.status)
        E.fsdp_wait(P, self.rank, self.lo, self.shard, 1, e, self.status)
        if int(self.status.item()) != 0:
            raise RuntimeError(f"fused optimizer step: a peer did not answer in time (status {int(self.status.item())})")
        off = 0
        for p in self.params:
            n = p.numel()
            p.data.copy_(self.param_flat[off:off + n].view_as(p).to(p.dtype))
            off += n
        return norm

    def close(self) -> None:
        """Unmap the peers, wait for every rank to unmap ours, free."""
        if self.closed:
            return
        self.closed = True
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            self.ext.ipc_close(p, self.device.index)
        if dist.is_initialized():
            dist.barrier(group=self.group)
        self.ext.mailbox_free(self.base, self.device.index)
