"""Fully sharded decoder layers (FSDP / ZeRO-3 style) for drafter training.

The reference wraps every decoder layer with FSDP2 through Accelerate
(``train/runtime.py:90-114``; the recovery teacher with ``fully_shard``,
``pruning/train_recovery.py:99-110``): a layer's parameters exist only as
one shard per rank, and the full weights are gathered just before the layer
runs.  Here, per decoder layer:

* the layer's parameters are flattened (padded so every rank's shard is a
  multiple of 8 elements) and rank ``r`` keeps elements ``[r*n, (r+1)*n)`` in
  a bf16 shard buffer that every peer has mapped over NVLink (CUDA IPC), plus
  the fp32 master shard and AdamW moments;
* **forward**: ``fsdp_gather`` reads every rank's shard of the layer into a
  local full-layer buffer (peer loads: each remote byte crosses NVLink once,
  then the GEMMs read local memory), and the layer runs on views of it
  without keeping them for backward;
* **backward**: the layer's weights are gathered again and its forward is
  recomputed with gradients (activation checkpointing per layer, as FSDP does
  with checkpointing on), and the layer's flat gradient is reduce-scattered
  by peer loads (``fsdp_signal`` / ``fsdp_reduce`` with epoch flags and
  bounded waits) into this rank's fp32 shard gradient;
* **optimizer**: AdamW on the shard (``adamw`` kernel) with the clip scale
  shared with the rest of the model, then a barrier so no rank gathers a
  shard a peer is still writing.

On CPU (tests, ``gloo``) the reduce-scatter is a ``torch.distributed``
collective with the same data layout; ``gloo`` has no one-sided reads, so the
shards are all-gathered once per step right after the update into a local copy
that the forward reads (the same values a per-layer gather would return).
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch
import torch.distributed as dist
from torch import nn
from torch.func import functional_call

_FLAG_BYTES = 256   # [4 phases][8 source ranks] int64 flags: 0 ready, 1 read, 2 updated


class _LayerSpec:
    def __init__(self, names: List[str], shapes: List[torch.Size], numel: int, world: int):
        self.names, self.shapes = names, shapes
        self.numel = numel
        self.shard = math.ceil(numel / (8 * world)) * 8
        self.padded = self.shard * world
        self.offset = 0          # this layer's offset inside the shard buffer


class _ShardedLayerFn(torch.autograd.Function):
    # ``anchor``: an empty tensor that requires grad, so the layer's output
    # takes part in autograd even when its input does not (frozen embeddings):
    # the layer's own weights are gathered inside and are no inputs here
    @staticmethod
    def forward(ctx, z, idx, anchor, x, cos, sin, mask, cache, store_kv):
        params = z.views(idx, z.gather(idx))
        with torch.no_grad():
            y = functional_call(z.mods[idx], params, (x, cos, sin, mask, cache, store_kv))
        ctx.z, ctx.idx, ctx.cache, ctx.store_kv = z, idx, cache, store_kv
        ctx.has_mask = mask is not None
        ctx.save_for_backward(x, cos, sin, mask if mask is not None else torch.empty(0))
        return y

    @staticmethod
    def backward(ctx, gy):
        z, idx = ctx.z, ctx.idx
        if ctx.store_kv:
            raise RuntimeError("sharded layers do not differentiate through KV stores")
        x, cos, sin, mask = ctx.saved_tensors
        mask = mask if ctx.has_mask else None
        full = z.gather(idx)
        leaves = {k: v.detach().requires_grad_(True) for k, v in z.views(idx, full).items()}
        xl = x.detach().requires_grad_(x.requires_grad)
        with torch.enable_grad():
            y = functional_call(z.mods[idx], leaves, (xl, cos, sin, mask, ctx.cache, False))
            torch.autograd.backward(y, gy)
        z.reduce_scatter(idx, leaves)
        return None, None, None, xl.grad if x.requires_grad else None, None, None, None, None, None


class ShardedLayer(nn.Module):
    """Stands in for decoder layer ``idx`` of a :class:`Zero3Layers` group
    (same call signature as the wrapped layer)."""

    def __init__(self, z: "Zero3Layers", idx: int):
        super().__init__()
        self._z = [z]            # not a submodule: its parameters are the group's shards
        self.idx = idx

    def forward(self, x, cos, sin, mask, cache, store_kv):
        self._z[0].mods[self.idx].train(self.training)
        z = self._z[0]
        return _ShardedLayerFn.apply(z, self.idx, z.anchor, x, cos, sin, mask, cache, store_kv)


class Zero3Layers:
    """Shards the decoder layers of ``layers`` (an ``nn.ModuleList``, replaced
    in place by :class:`ShardedLayer` modules) over the ranks of ``group``."""

    def __init__(self, layers: nn.ModuleList, group=None, lr: float = 1e-4, betas=(0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.0):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > 8:
            raise ValueError("sharded layers support up to 8 ranks")
        self.b1, self.b2, self.eps, self.wd, self.lr = betas[0], betas[1], eps, weight_decay, lr
        p0 = next(layers[0].parameters())
        self.device, self.dtype = p0.device, p0.dtype
        self.cuda = self.device.type == "cuda"
        if self.cuda and self.dtype != torch.bfloat16:
            raise ValueError("sharded layers on CUDA compute in bf16")
        self.mods: List[nn.Module] = list(layers)
        self.specs: List[_LayerSpec] = []
        off = 0
        for m in self.mods:
            named = [(n, p) for n, p in m.named_parameters()]
            spec = _LayerSpec([n for n, _ in named], [p.shape for _, p in named], sum(p.numel() for _, p in named),
                              self.world)
            spec.offset = off
            off += spec.shard
            self.specs.append(spec)
        self.total = off
        self.max_padded = max(s.padded for s in self.specs)
        self._alloc_buffers()
        # shards of every layer: bf16 compute copy (peer-visible), fp32 master, moments
        self.master = torch.zeros(self.total, dtype=torch.float32, device=self.device)
        for m, s in zip(self.mods, self.specs):
            flat = torch.zeros(s.padded, dtype=torch.float32, device=self.device)
            o = 0
            for _, p in m.named_parameters():
                flat[o:o + p.numel()] = p.detach().reshape(-1).float()
                o += p.numel()
            mine = flat[self.rank * s.shard:(self.rank + 1) * s.shard]
            self.master[s.offset:s.offset + s.shard] = mine
            self.params[s.offset:s.offset + s.shard] = mine.to(self.dtype)
            for _, p in m.named_parameters():     # the full weights live only while a layer runs
                p.requires_grad_(False)
                p.data = torch.empty(0, dtype=p.dtype, device=p.device)
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.grad = torch.zeros_like(self.master)
        if not self.cuda:
            self._refresh_replica()
        elif self.world > 1:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)      # every rank's shards are written before anyone gathers
        self.step_count = 0
        self.epoch = 0
        self.gathered = torch.empty(self.max_padded, dtype=self.dtype, device=self.device)
        self.anchor = torch.zeros(0, device=self.device, requires_grad=True)
        self._part = torch.empty(max(s.shard for s in self.specs), dtype=torch.float32, device=self.device)
        for i in range(len(layers)):
            layers[i] = ShardedLayer(self, i)

    # ----------------------------------------------------------- buffers
    def _alloc_buffers(self) -> None:
        if not self.cuda:
            self.params = torch.zeros(self.total, dtype=self.dtype, device=self.device)
            self.replica = torch.zeros(sum(s.padded for s in self.specs), dtype=self.dtype, device=self.device)
            return
        from .. import ops
        E = ops.ext()
        self.ext = E
        dev = self.device.index
        sb = (4 * self.max_padded + 255) // 256 * 256
        pb = (2 * self.total + 255) // 256 * 256
        self.nbytes = _FLAG_BYTES + sb + pb
        self.base = E.mailbox_alloc(self.nbytes, dev)
        mem = E.mailbox_view(self.base, self.nbytes, dev)
        mem.zero_()
        self.staging = mem[_FLAG_BYTES:_FLAG_BYTES + 4 * self.max_padded].view(torch.float32)
        self.params = mem[_FLAG_BYTES + sb:_FLAG_BYTES + sb + 2 * self.total].view(torch.bfloat16)
        handles: List = [None] * self.world
        if self.world > 1:
            torch.cuda.synchronize(self.device)
            dist.all_gather_object(handles, (self.rank, E.ipc_handle(self.base, dev)), group=self.group)
        else:
            handles = [(0, None)]
        by_rank = dict(handles)
        bases, self._opened = [], []
        for r in range(self.world):
            if r == self.rank:
                bases.append(self.base)
            else:
                p = E.ipc_open(by_rank[r], dev)
                self._opened.append(p)
                bases.append(p)
        self.ptrs = torch.tensor([[b + _FLAG_BYTES for b in bases], [b + _FLAG_BYTES + sb for b in bases], bases],
                                 dtype=torch.int64)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._sq = torch.zeros(1, dtype=torch.float32, device=self.device)

    # ------------------------------------------------------ gather / scatter
    def gather(self, idx: int) -> torch.Tensor:
        """Every rank's shard of layer ``idx``: the full flat weights (bf16)."""
        s = self.specs[idx]
        full = self.gathered[: s.padded]
        if not self.cuda:
            lo = sum(t.padded for t in self.specs[:idx])
            return self.replica[lo:lo + s.padded]
        self.ext.fsdp_gather(self.ptrs, self.rank, s.offset, s.shard, full)
        return full

    def _refresh_replica(self) -> None:
        every = torch.empty(self.world * self.total, dtype=self.dtype, device=self.device)
        if self.world > 1:
            dist.all_gather_into_tensor(every, self.params, group=self.group)
        else:
            every.copy_(self.params)
        every = every.view(self.world, self.total)
        lo = 0
        for s in self.specs:
            self.replica[lo:lo + s.padded].view(self.world, s.shard).copy_(every[:, s.offset:s.offset + s.shard])
            lo += s.padded

    def views(self, idx: int, full: torch.Tensor) -> Dict[str, torch.Tensor]:
        s = self.specs[idx]
        out, o = {}, 0
        for n, shape in zip(s.names, s.shapes):
            k = math.prod(shape)
            out[n] = full[o:o + k].view(shape)
            o += k
        return out

    def reduce_scatter(self, idx: int, leaves: Dict[str, torch.Tensor]) -> None:
        """Sum layer ``idx``'s gradient over the ranks into this rank's shard."""
        s = self.specs[idx]
        if self.cuda:
            g = self.staging
            if self.epoch > 0:      # every peer has finished reading the previous exchange
                self.ext.fsdp_wait(self.ptrs, self.rank, 0, 0, 1, self.epoch, self.status)
        else:
            g = torch.zeros(s.padded, dtype=torch.float32, device=self.device)
        o = 0
        for n, shape in zip(s.names, s.shapes):
            k = math.prod(shape)
            gr = leaves[n].grad if n in leaves else None
            if gr is None:
                g[o:o + k].zero_()
            else:
                g[o:o + k].copy_(gr.reshape(-1))
            o += k
        g[s.numel:s.padded].zero_()
        dst = self.grad[s.offset:s.offset + s.shard]
        if self.cuda:
            self.epoch += 1
            e, lo = self.epoch, self.rank * s.shard
            part = self._part[: s.shard]
            self.ext.fsdp_signal(self.ptrs, self.rank, lo, s.shard, 0, e, g)
            self.ext.fsdp_reduce(self.ptrs, self.rank, lo, s.shard, e, part, self._sq, self.status)
            self.ext.fsdp_signal(self.ptrs, self.rank, lo, s.shard, 1, e, g)
            dst.add_(part)
        else:
            if self.world > 1:
                dist.all_reduce(g, group=self.group)
            dst.add_(g[self.rank * s.shard:(self.rank + 1) * s.shard])

    def idle_exchanges(self, n: int) -> None:
        """Take part in ``n`` gradient exchanges with a zero gradient -- for a
        rank with nothing to supervise this step, so the other ranks' layer
        exchanges stay matched (every decoder layer has the same shard
        size, so which layer a zero contribution lands on does not matter)."""
        if len({s.shard for s in self.specs}) != 1:
            raise RuntimeError("idle exchanges need layers of one shape")
        zero = {}
        for i in range(n):
            idx = len(self.specs) - 1 - (i % len(self.specs))
            self.reduce_scatter(idx, zero)

    def check(self) -> None:
        if self.cuda and int(self.status.item()) != 0:
            raise RuntimeError(f"sharded-layer exchange: a peer did not answer in time "
                               f"(status {int(self.status.item())})")

    # ------------------------------------------------------------ optimizer
    def zero_grad(self) -> None:
        self.grad.zero_()
        if self.cuda:
            self._sq.zero_()

    def sumsq(self) -> torch.Tensor:
        """Local squared norm of this rank's shard gradients ([1] fp32)."""
        if self.cuda:
            sq = torch.zeros(1, dtype=torch.float32, device=self.device)
            self.ext.sumsq(self.grad, sq)
            return sq
        return (self.grad.double() ** 2).sum().float().reshape(1)

    @torch.no_grad()
    def step(self, scale: float, lr: Optional[float] = None) -> None:
        """AdamW on the shards with gradient scale ``scale`` (mean over ranks
        times the clip factor shared with the rest of the model), then every
        rank's new shards are in place before anyone gathers them again
        (device-side flags on CUDA; the replica refresh on CPU)."""
        lr = self.lr if lr is None else lr
        self.step_count += 1
        if self.cuda:
            self.ext.adamw(self.master, self.grad, self.m, self.v, self.params[: self.total], lr, self.b1, self.b2,
                           self.eps, self.wd, self.step_count, scale)
            if self.world > 1:
                # device-side barrier: "my shards of this step are written" to
                # every rank, and no gather of the next forward starts before
                # every rank's flag has arrived (bounded wait, status on timeout)
                self.ext.fsdp_signal(self.ptrs, self.rank, 0, 0, 2, self.step_count, self.status)
                self.ext.fsdp_wait(self.ptrs, self.rank, 0, 0, 2, self.step_count, self.status)
            self.check()
            return
        else:
            gi = self.grad * scale
            self.m.mul_(self.b1).add_(gi, alpha=1 - self.b1)
            self.v.mul_(self.b2).addcmul_(gi, gi, value=1 - self.b2)
            bc1, bc2 = 1 - self.b1 ** self.step_count, 1 - self.b2 ** self.step_count
            self.master.mul_(1 - lr * self.wd)
            self.master.addcdiv_(self.m / bc1, (self.v / bc2).sqrt().add_(self.eps), value=-lr)
            self.params.copy_(self.master.to(self.dtype))
            self._refresh_replica()

    # ------------------------------------------------------------ checkpoint
    @torch.no_grad()
    def full_state(self, prefix: str) -> Dict[str, torch.Tensor]:
        """fp32 full weights of every layer (gathered master shards), named
        ``{prefix}{layer}.{param}`` -- collective over the group."""
        out = {}
        for i, s in enumerate(self.specs):
            mine = self.master[s.offset:s.offset + s.shard].contiguous()
            full = torch.empty(s.padded, dtype=torch.float32, device=self.device)
            if self.world > 1:
                dist.all_gather_into_tensor(full, mine, group=self.group)
            else:
                full.copy_(mine)
            for n, v in self.views(i, full).items():
                out[f"{prefix}{i}.{n}"] = v.cpu().clone()
        return out

    def state_dict(self) -> dict:
        return {"master": self.master.cpu(), "m": self.m.cpu(), "v": self.v.cpu(), "step": self.step_count,
                "rank": self.rank, "world": self.world, "total": self.total}

    def load_state_dict(self, sd: dict) -> None:
        if sd["world"] != self.world or sd["total"] != self.total:
            raise ValueError("sharded-layer state does not match this run")
        self.master.copy_(sd["master"])
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])
        self.params.copy_(self.master.to(self.dtype))
        self.step_count = int(sd["step"])
        if not self.cuda:
            self._refresh_replica()
        elif self.world > 1:
            dist.barrier(group=self.group)      # every rank's shards are loaded before anyone gathers

    def close(self) -> None:
        if not self.cuda or getattr(self, "_closed", False):
            return
        self._closed = True
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            self.ext.ipc_close(p, self.device.index)
        if self.world > 1:
            dist.barrier(group=self.group)
        self.ext.mailbox_free(self.base, self.device.index)
