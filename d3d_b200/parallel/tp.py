"""Tensor parallelism for the target (one process per GPU).

Megatron-style split of a Qwen3 decoder over ``tp`` ranks:

* column-parallel ``qkv`` (each rank owns ``Hq/tp`` query heads and
  ``Hkv/tp`` kv heads, and the KV cache of those heads) and ``gate_up``
  (``I/tp`` rows of gate and of up);
* row-parallel ``o`` and ``down``: each rank multiplies its slice of the
  inner dimension and the ranks' fp32 partials are summed by the consumer
  kernel (``add_rmsnorm_tp``), which reads the peers' exchange regions over
  NVLink after bounded acquire-waits on their flags -- the all-reduce of the
  row-parallel output fused into the residual add + RMSNorm;
* vocab-parallel LM head: each rank takes the top-k of its ``V/tp`` rows and
  ``topk_merge_tp`` merges the ranks' candidates.

The residual stream, norms and embedding are replicated.  The reference has
no working tensor parallelism at all (its vendored TP layers run at
tp_size=1, ``serving/vendor/ssd/layers/linear.py:68-199``).

:class:`TPGroup` owns this rank's exchange region (flags, two partial
buffers, the LM-head candidate slot), maps every peer's region through CUDA
IPC and keeps the device epoch counter the kernels use as flag values.
"""
from __future__ import annotations

from typing import List

import torch
import torch.distributed as dist

from .. import ops
from ..config import ModelConfig

FLAG_BYTES_PER_X = 8  # one int64 per (exchange, source rank)


def local_config(cfg: ModelConfig, tp: int) -> ModelConfig:
    """The per-rank shapes of a ``tp``-way split (hidden size unchanged)."""
    if tp == 1:
        return cfg
    for name, v in (("num_attention_heads", cfg.num_attention_heads),
                    ("num_key_value_heads", cfg.num_key_value_heads),
                    ("vocab_size", cfg.vocab_size)):
        if v % tp:
            raise ValueError(f"{name}={v} is not divisible by tp={tp}")
    if cfg.intermediate_size % (64 * tp):
        raise ValueError(f"intermediate_size={cfg.intermediate_size} must be a multiple of 64*tp")
    return cfg.replace(num_attention_heads=cfg.num_attention_heads // tp,
                       num_key_value_heads=cfg.num_key_value_heads // tp,
                       intermediate_size=cfg.intermediate_size // tp,
                       vocab_size=cfg.vocab_size // tp)


class TPGroup:
    """Exchange state of one rank.  Collective over ``group`` (all ranks of
    the tensor-parallel group construct it together)."""

    def __init__(self, rank: int, size: int, device, group=None, num_layers: int = 64,
                 part_bytes: int = 64 << 20, cand_bytes: int = 1 << 20):
        if size > 8:
            raise ValueError("tp size above 8")
        self.rank, self.size = int(rank), int(size)
        self.device = torch.device(device)
        self.group = group
        self.n_x = 2 * num_layers + 1                         # exchanges per forward
        self.flag_bytes = (self.n_x * self.size * FLAG_BYTES_PER_X + 255) // 256 * 256
        self.part_bytes = (part_bytes + 255) // 256 * 256
        self.cand_off = self.flag_bytes + 2 * self.part_bytes
        # armed-verify decision record (rank 0 writes it into every other rank)
        self.dec_off = self.cand_off + (cand_bytes + 255) // 256 * 256
        self.nbytes = self.dec_off + 256
        E = ops.ext()
        self.ext = E
        self.base = E.mailbox_alloc(self.nbytes, self.device.index)     # zero-filled
        self.mem = E.mailbox_view(self.base, self.nbytes, self.device.index)
        self.epoch = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.ticket = torch.zeros(1, dtype=torch.int32, device=self.device)   # last-CTA counter of the GEMMs
        handles: List = [None] * dist.get_world_size(group)
        dist.all_gather_object(handles, (self.rank, E.ipc_handle(self.base, self.device.index)), group=group)
        by_rank = {r: h for r, h in handles}
        self.peer_bases = []
        self._opened = []
        for r in range(self.size):
            if r == self.rank:
                self.peer_bases.append(self.base)
            else:
                p = E.ipc_open(by_rank[r], self.device.index)
                self._opened.append(p)
                self.peer_bases.append(p)
        # [2, tp]: flag arrays, exchange regions (partials start after the flags)
        self.ptrs = torch.tensor([[b for b in self.peer_bases],
                                  [b for b in self.peer_bases]], dtype=torch.int64)
        self.closed = False
        # measurement only (D3D_TP_LOCAL=1): skip every cross-rank step (local
        # partials, no flags) to time what the exchanges cost; results are wrong
        import os
        self.local_only = os.environ.get("D3D_TP_LOCAL") == "1"
        # exchange mode (measured on two B200s, 32B forward: pull 10.3 ms,
        # pull_cta 11.3 ms, push 11.4 ms at M=1):
        #   "pull"     each rank's GEMM keeps its partials, a one-thread kernel
        #              raises the flags, consumers read the peers' partials;
        #   "pull_cta" the same, flags raised by the GEMM's last CTA;
        #   "push"     GEMM epilogues store into every rank's buffer, last CTA flags.
        self.mode = os.environ.get("D3D_TP_MODE", "pull")
        if self.mode not in ("pull", "pull_cta", "push"):
            raise ValueError("D3D_TP_MODE must be pull, pull_cta or push")
        self.pull = self.mode != "push"

    # --------------------------------------------------------------- layout
    def part_offset(self, parity: int) -> int:
        return self.flag_bytes + (parity & 1) * self.part_bytes

    def part_view(self, parity: int, n_floats: int) -> torch.Tensor:
        """This rank's partial buffer ``parity`` as an fp32 tensor."""
        if 4 * n_floats > self.part_bytes:
            raise ValueError(f"partials of {4 * n_floats} bytes exceed the {self.part_bytes}-byte buffer")
        off = self.part_offset(parity)
        return self.mem[off:off + 4 * n_floats].view(torch.float32)

    def decision_records(self) -> torch.Tensor:
        """Where this rank's armed-verify decisions go (int64 addresses): on
        rank 0 every other rank's record, elsewhere this rank's own."""
        if self.rank == 0:
            return torch.tensor([b + self.dec_off for b in self.peer_bases[1:]], dtype=torch.int64)
        return torch.tensor([self.base + self.dec_off], dtype=torch.int64)

    def cand_view(self) -> torch.Tensor:
        return self.mem[self.cand_off:]

    # -------------------------------------------------------------- kernels
    def bump(self) -> None:
        self.ext.tp_epoch_bump(self.epoch)

    def signal(self, x: int) -> None:
        if self.local_only:
            return
        self.ext.tp_signal(self.ptrs, self.rank, self.epoch, x)

    def gemm(self, x_act, w, x: int, splits: int, bt: int) -> None:
        """Row-parallel GEMM of exchange ``x``: partials pushed to every rank
        (buffer parity ``x & 1``), flags raised by the GEMM's last CTA."""
        if 4 * splits * self.size * x_act.shape[0] * w.n > self.part_bytes:
            raise ValueError("row-parallel partials exceed the exchange buffer")
        if self.local_only:
            self.ext.gemm_partial(x_act, w.data, self.part_view(x, splits * x_act.shape[0] * w.n), splits, bt,
                                  self.status, w.n)
            return
        if self.mode == "pull":
            n = splits * x_act.shape[0] * w.n           # this rank's slots [rank][split] of buffer x & 1
            off = self.part_offset(x) + 4 * self.rank * n
            self.ext.gemm_partial(x_act, w.data, self.mem[off:off + 4 * n].view(torch.float32), splits, bt,
                                  self.status, w.n)
            self.signal(x)
            return
        self.ext.gemm_partial_tp(x_act, w.data, self.ptrs, self.rank, self.epoch, self.ticket, x,
                                 self.part_offset(x), splits, bt, self.status, w.n, self.pull)

    def add_rmsnorm(self, x: int, parity: int, nsplit: int, residual, w, out, eps: float) -> None:
        if self.local_only:
            self.ext.add_rmsnorm(self.part_view(parity, nsplit * residual.numel()), nsplit, residual, w, out, eps)
            return
        self.ext.add_rmsnorm_tp(self.ptrs, self.rank, self.epoch, x, self.part_offset(parity), nsplit,
                                residual, w, out, eps, self.status, self.pull)

    def merge_topk(self, x: int, M: int, k: int, ov, oi) -> None:
        if self.local_only:
            return
        self.ext.topk_merge_tp(self.ptrs, self.rank, self.epoch, x, self.cand_off, M, k, ov, oi, self.status)

    def close(self) -> None:
        """Unmap the peers, wait until every peer unmapped ours, free."""
        if self.closed:
            return
        self.closed = True
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            self.ext.ipc_close(p, self.device.index)
        if dist.is_initialized():
            dist.barrier(group=self.group)
        self.ext.mailbox_free(self.base, self.device.index)


# ----------------------------------------------------------------- weights
def shard_weights(w, tp: int, rank: int):
    """The ``rank``-th of ``tp`` shards of :class:`~d3d_b200.models.fast.FastWeights`."""
    from ..models.fast import FastWeights, LayerWeights
    if tp == 1:
        return w
    cfg = w.cfg
    lc = local_config(cfg, tp)
    d = cfg.head_dim
    hq, hkv, I = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size
    qs, ks = hq * d, hkv * d
    qa, qb = rank * lc.num_attention_heads * d, (rank + 1) * lc.num_attention_heads * d
    ka, kb = rank * lc.num_key_value_heads * d, (rank + 1) * lc.num_key_value_heads * d
    ia, ib = rank * lc.intermediate_size, (rank + 1) * lc.intermediate_size
    order = ops.gate_up_order(I).to(w.embed.device)
    layers = []
    for L in w.layers:
        qkv = L.qkv.unpack()
        q, k, v = qkv[:qs], qkv[qs:qs + ks], qkv[qs + ks:]
        qkv_l = torch.cat([q[qa:qb], k[ka:kb], v[ka:kb]], 0).contiguous()
        o = L.o.unpack()[:, qa:qb].contiguous()
        gu = torch.empty(2 * I, cfg.hidden_size, dtype=torch.bfloat16, device=w.embed.device)
        gu[order] = L.gate_up.unpack()                       # back to [gate; up]
        gate_l, up_l = gu[:I][ia:ib].contiguous(), gu[I:][ia:ib].contiguous()
        down = L.down.unpack()[:, ia:ib].contiguous()
        layers.append(LayerWeights(qkv=ops.pack_weight(qkv_l), o=ops.pack_weight(o),
                                   gate_up=ops.pack_gate_up(gate_l, up_l), down=ops.pack_weight(down),
                                   in_norm=L.in_norm, post_norm=L.post_norm, q_norm=L.q_norm, k_norm=L.k_norm))
    va, vb = rank * lc.vocab_size, (rank + 1) * lc.vocab_size
    lm = ops.pack_weight(w.lm_head.unpack()[va:vb].contiguous())
    out = FastWeights(lc, w.embed, layers, w.final_norm, lm, w.cond_proj)
    out.tp = (tp, rank, cfg)
    return out


def random_shard(cfg: ModelConfig, tp: int, rank: int, seed: int = 0, device="cuda"):
    """Seeded random weights of one shard, drawn directly at shard size (a
    32B-class target never exists whole on one GPU)."""
    from ..models.fast import FastWeights
    if cfg.tie_word_embeddings and tp > 1:
        raise ValueError("tensor parallelism expects an untied LM head")
    lc = local_config(cfg, tp)
    w = FastWeights.random(lc, seed=seed * 1009 + rank, device=device)
    if tp > 1:
        # the embedding is replicated: the same full-vocabulary draw on every rank
        w.embed = FastWeights.seeded_randn((cfg.vocab_size, cfg.hidden_size), seed * 7919 + 17,
                                           cfg.initializer_range, device)
    w.tp = (tp, rank, cfg)
    return w
