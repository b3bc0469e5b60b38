"""The Qwen3 / D3D forward on the sm_100a kernels (inference fast path).
Reference counterparts: the paged runner ``serving/backend.py:44-136`` and
the vendored Qwen3 ``serving/vendor/ssd/models/qwen3.py:14-325``.

Weights are held in bf16 in fused layouts (``qkv = [q; k; v]`` and
``gate_up = [gate; up]`` rows), the KV cache is paged
(``[slots, Hkv, D]`` per layer, slot = page * page_size + offset), and one
layer is nine launches::

    gemm(qkv) -> qkv_rope_kv (QK-norm, RoPE, KV write) -> attention
    -> gemm(o) -> add_rmsnorm -> gemm(gate_up) -> swiglu -> gemm(down)
    -> add_rmsnorm (next layer's input norm, or the final norm)

Every GEMM writes fp32 split-K partials with a split factor that depends on
the weight shape only (``ops.splitk_for``); decode-sized forwards use a fixed
attention key chunk.  Together these make a token's logits bit-identical
whether it is decoded alone (AR) or verified inside a block, so greedy
speculative decoding reproduces AR decoding token for token.

Inputs of a forward live in :class:`StepBuffers` (static device tensors) so
the whole forward can be captured once per shape in a CUDA graph and
replayed.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from .. import ops
from ..config import ModelConfig
from .qwen3 import Qwen3LM


# --------------------------------------------------------------------------
# weights
# --------------------------------------------------------------------------
@dataclass
class LayerWeights:
    qkv: torch.Tensor
    o: torch.Tensor
    gate_up: torch.Tensor
    down: torch.Tensor
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor


class FastWeights:
    def __init__(self, cfg: ModelConfig, embed, layers: List[LayerWeights], final_norm, lm_head,
                 cond_proj=None):
        self.cfg = cfg
        self.embed = embed
        self.layers = layers
        self.final_norm = final_norm
        self.lm_head = lm_head
        self.cond_proj = cond_proj
        # True once the input / post-attention RMSNorm weights are folded into
        # the qkv / gate|up weights (column scale); see fold_norms
        self.folded = False

    @torch.no_grad()
    def fold_norms(self) -> "FastWeights":
        """Fold each layer's RMSNorm weights into the GEMM that consumes the
        normalised activations (in place, idempotent):
        ``rmsnorm(x) * g @ W^T = r(x) * (x @ (W diag(g))^T)``, so the fused
        forward feeds the residual stream itself to the qkv and gate|up GEMMs
        and applies the per-row scale ``r`` in their reduce kernels.  Layers
        whose norm weights are all ones (random init) need no repacking."""
        if self.folded:
            return self
        for L in self.layers:
            for attr, g in (("qkv", L.in_norm), ("gate_up", L.post_norm)):
                if bool((g == 1).all()):
                    continue
                w = getattr(L, attr)
                full = w.unpack().float() * g.float()[None, :]
                setattr(L, attr, ops.pack_weight(full.to(torch.bfloat16)))   # row order kept (interleaved)
        self.folded = True
        return self

    @classmethod
    @torch.no_grad()
    def from_module(cls, m: Qwen3LM, device="cuda") -> "FastWeights":
        bf = lambda t: t.detach().to(device=device, dtype=torch.bfloat16).contiguous()
        pk = lambda t: ops.pack_weight(bf(t))
        layers = []
        for L in m.model.layers:
            a = L.self_attn
            layers.append(LayerWeights(
                qkv=pk(torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0)),
                o=pk(a.o_proj.weight),
                gate_up=ops.pack_gate_up(bf(L.mlp.gate_proj.weight), bf(L.mlp.up_proj.weight)),
                down=pk(L.mlp.down_proj.weight),
                in_norm=bf(L.input_layernorm.weight), post_norm=bf(L.post_attention_layernorm.weight),
                q_norm=bf(a.q_norm.weight), k_norm=bf(a.k_norm.weight)))
        embed = bf(m.model.embed_tokens.weight)
        lm = pk(embed if m.cfg.tie_word_embeddings else m.lm_head.weight)
        cp = pk(m.cond_proj.weight) if getattr(m, "cond_proj", None) is not None else None
        return cls(m.cfg, embed, layers, bf(m.model.norm.weight), lm, cp)

    @classmethod
    @torch.no_grad()
    def from_state(cls, cfg: ModelConfig, state: Dict[str, torch.Tensor], device="cuda") -> "FastWeights":
        """Kernel layouts from a Hugging-Face-named state dict whose tensors
        already have ``cfg``'s (possibly per-rank) shapes -- e.g. one rank's
        slices from ``checkpoint.load_tp_shard`` with a ``parallel.tp.local_config``."""
        bf = lambda t: t.to(device=device, dtype=torch.bfloat16).contiguous()
        pk = lambda t: ops.pack_weight(bf(t))
        layers = []
        for n in range(cfg.num_hidden_layers):
            p = f"model.layers.{n}."
            g = lambda k: state[p + k]
            layers.append(LayerWeights(
                qkv=pk(torch.cat([g("self_attn.q_proj.weight"), g("self_attn.k_proj.weight"),
                                  g("self_attn.v_proj.weight")], 0)),
                o=pk(g("self_attn.o_proj.weight")),
                gate_up=ops.pack_gate_up(bf(g("mlp.gate_proj.weight")), bf(g("mlp.up_proj.weight"))),
                down=pk(g("mlp.down_proj.weight")),
                in_norm=bf(g("input_layernorm.weight")), post_norm=bf(g("post_attention_layernorm.weight")),
                q_norm=bf(g("self_attn.q_norm.weight")), k_norm=bf(g("self_attn.k_norm.weight"))))
        embed = bf(state["model.embed_tokens.weight"])
        lm = pk(state["lm_head.weight"]) if "lm_head.weight" in state else ops.pack_weight(embed)
        cp = pk(state["cond_proj.weight"]) if "cond_proj.weight" in state else None
        return cls(cfg, embed, layers, bf(state["model.norm.weight"]), lm, cp)

    @staticmethod
    @torch.no_grad()
    def seeded_randn(shape, key: int, std: float, device="cuda") -> torch.Tensor:
        """bf16 N(0, std) tensor drawn on the device from generator seed ``key``
        (in chunks, so the fp32 temporary stays small)."""
        gen = torch.Generator(device=device)
        gen.manual_seed(int(key))
        t = torch.empty(*shape, dtype=torch.bfloat16, device=device)
        flat = t.view(-1)
        step = 1 << 26
        for i in range(0, flat.numel(), step):
            n = min(step, flat.numel() - i)
            flat[i:i + n] = (torch.randn(n, generator=gen, device=device) * std).to(torch.bfloat16)
        return t

    @classmethod
    @torch.no_grad()
    def random(cls, cfg: ModelConfig, seed: int = 0, device="cuda",
               std: Optional[float] = None) -> "FastWeights":
        """Seeded N(0, std) init drawn on the device (no host copy of the model)."""
        std = cfg.initializer_range if std is None else std
        counter = [0]

        def rnd(*shape):
            counter[0] += 1
            return cls.seeded_randn(shape, int(seed) * 1_000_003 + counter[0], std, device)

        ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=device)
        prnd = lambda *shape: ops.pack_weight(rnd(*shape))
        h, i, d = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
        layers = [LayerWeights(qkv=prnd(cfg.q_size + 2 * cfg.kv_size, h), o=prnd(h, cfg.q_size),
                               gate_up=ops.pack_gate_up(*rnd(2 * i, h).chunk(2)), down=prnd(h, i),
                               in_norm=ones(h),
                               post_norm=ones(h), q_norm=ones(d), k_norm=ones(d))
                  for _ in range(cfg.num_hidden_layers)]
        embed = rnd(cfg.vocab_size, h)
        lm = ops.pack_weight(embed) if cfg.tie_word_embeddings else prnd(cfg.vocab_size, h)
        cp = prnd(h, cfg.cond_hidden_size) if cfg.cond_hidden_size else None
        return cls(cfg, embed, layers, ones(h), lm, cp)

    @torch.no_grad()
    def to_module(self, device=None, dtype=torch.bfloat16) -> Qwen3LM:
        """The PyTorch module holding these weights (unpacked; the gate|up
        rows put back in order; folded norm scales divided out again), e.g.
        as the oracle that the kernel path is validated against."""
        cfg = self.cfg
        dev = device if device is not None else self.embed.device
        m = Qwen3LM(cfg).to(device=dev, dtype=dtype)
        cast = lambda t: t.to(device=dev, dtype=dtype)
        q, kv = cfg.q_size, cfg.kv_size
        order = ops.gate_up_order(cfg.intermediate_size).to(self.embed.device)
        for L, dst in zip(self.layers, m.model.layers):
            qkv = L.qkv.unpack().float()
            gu = L.gate_up.unpack().float()
            if self.folded:
                qkv = qkv / L.in_norm.float()[None, :]
                gu = gu / L.post_norm.float()[None, :]
            rows = torch.empty_like(gu)
            rows[order] = gu
            a = dst.self_attn
            a.q_proj.weight.copy_(cast(qkv[:q]))
            a.k_proj.weight.copy_(cast(qkv[q:q + kv]))
            a.v_proj.weight.copy_(cast(qkv[q + kv:]))
            a.o_proj.weight.copy_(cast(L.o.unpack()))
            a.q_norm.weight.copy_(cast(L.q_norm))
            a.k_norm.weight.copy_(cast(L.k_norm))
            dst.mlp.gate_proj.weight.copy_(cast(rows[:cfg.intermediate_size]))
            dst.mlp.up_proj.weight.copy_(cast(rows[cfg.intermediate_size:]))
            dst.mlp.down_proj.weight.copy_(cast(L.down.unpack()))
            dst.input_layernorm.weight.copy_(cast(L.in_norm))
            dst.post_attention_layernorm.weight.copy_(cast(L.post_norm))
        m.model.embed_tokens.weight.copy_(cast(self.embed))
        m.model.norm.weight.copy_(cast(self.final_norm))
        if not cfg.tie_word_embeddings:
            m.lm_head.weight.copy_(cast(self.lm_head.unpack()))
        if self.cond_proj is not None and getattr(m, "cond_proj", None) is not None:
            m.cond_proj.weight.copy_(cast(self.cond_proj.unpack()))
        return m.eval()

    def drop_layers(self, idx) -> "FastWeights":
        keep = [L for j, L in enumerate(self.layers) if j not in set(idx)]
        cfg = self.cfg.replace(num_hidden_layers=len(keep))
        return FastWeights(cfg, self.embed, keep, self.final_norm, self.lm_head, self.cond_proj)

    def nbytes(self) -> int:
        """Bytes of weights one forward streams (embedding rows excluded)."""
        n = self.final_norm.numel() + self.lm_head.numel()
        for L in self.layers:
            n += sum(t.numel() for t in (L.qkv, L.o, L.gate_up, L.down, L.in_norm, L.post_norm,
                                         L.q_norm, L.k_norm))
        return 2 * n


# --------------------------------------------------------------------------
# paged KV
# --------------------------------------------------------------------------
class PagedKV:
    """Per-layer paged K/V storage plus a page allocator and block tables."""

    def __init__(self, cfg: ModelConfig, num_pages: int, page_size: int, max_seqs: int,
                 max_pages_per_seq: int, device="cuda"):
        self.cfg = cfg
        self.page_size = page_size
        self.num_pages = num_pages
        slots = num_pages * page_size
        shape = (slots, cfg.num_key_value_heads, cfg.head_dim)
        self.k = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(cfg.num_hidden_layers)]
        self.v = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(cfg.num_hidden_layers)]
        self.free: List[int] = list(range(num_pages - 1, -1, -1))
        self.tables: Dict[int, List[int]] = {}
        self.max_pages_per_seq = max_pages_per_seq
        self.max_seqs = max_seqs
        self.block_table = torch.zeros(max_seqs, max_pages_per_seq, dtype=torch.int32, device=device)
        self.device = device
        self.scratch: List[int] = []    # pages held outside any sequence (placeholder KV stores)

    def scratch_slot(self) -> int:
        """A KV slot of a page no sequence ever owns: where the KV stores of a
        forward run on placeholder inputs go."""
        if not self.scratch:
            if not self.free:
                raise RuntimeError("out of KV pages for the scratch page")
            self.scratch.append(self.free.pop())
        return self.scratch[0] * self.page_size

    def reserve(self, sid: int, row: int, length: int) -> None:
        """Make sequence ``sid`` (block-table row ``row``) cover ``length`` slots."""
        t = self.tables.setdefault(sid, [])
        need = math.ceil(length / self.page_size) - len(t)
        if need > 0:
            if need > len(self.free):
                raise RuntimeError(f"out of KV pages: need {need}, free {len(self.free)}")
            if len(t) + need > self.max_pages_per_seq:
                raise RuntimeError("sequence exceeds max_pages_per_seq")
            new = [self.free.pop() for _ in range(need)]
            t.extend(new)
            self.block_table[row, : len(t)] = torch.tensor(t, dtype=torch.int32).to(self.device,
                                                                                   non_blocking=True)

    def trim(self, sid: int, row: int, length: int) -> None:
        t = self.tables.get(sid, [])
        keep = math.ceil(length / self.page_size)
        while len(t) > keep:
            self.free.append(t.pop())

    def release(self, sid: int) -> None:
        for p in self.tables.pop(sid, []):
            self.free.append(p)

    def slots(self, sid: int, start: int, n: int):
        """Physical KV slots of logical positions start..start+n-1 (numpy int64)."""
        t = np.asarray(self.tables[sid], dtype=np.int64)
        ps = self.page_size
        lp = np.arange(start, start + n, dtype=np.int64)
        return t[lp // ps] * ps + lp % ps

    @property
    def leaked(self) -> int:
        return self.num_pages - len(self.free) - sum(len(t) for t in self.tables.values()) - len(self.scratch)


# --------------------------------------------------------------------------
# step buffers + runner
# --------------------------------------------------------------------------
class StepBuffers:
    """Static device inputs/outputs of one forward shape (B sequences x Q tokens)."""

    def __init__(self, cfg: ModelConfig, B: int, Q: int, topk: int, n_chunks: int,
                 splits: Dict[str, int], device="cuda", with_hidden_copy: bool = False, fused_norm: bool = False):
        T = B * Q
        self.B, self.Q, self.T, self.topk, self.n_chunks = B, Q, T, topk, n_chunks
        dev = device
        h, d = cfg.hidden_size, cfg.head_dim
        # All integer step inputs live in one byte buffer (and a pinned host
        # twin), so a forward needs a single host->device copy.
        segs = [("ids", T, torch.int64), ("pos", T, torch.int64), ("slots", T, torch.int64),
                ("seq_rows", B, torch.int64), ("rows", 3 * T, torch.int32), ("kv_end", B, torch.int32),
                ("cond_rows", T, torch.uint8)]
        offs, off = {}, 0
        for name, n, dt in segs:
            offs[name] = off
            off += (n * torch.tensor([], dtype=dt).element_size() + 15) // 16 * 16
        self.in_bytes = off
        self.inbuf = torch.zeros(off, dtype=torch.uint8, device=dev)
        self.inbuf_host = torch.zeros(off, dtype=torch.uint8, pin_memory=str(dev).startswith("cuda"))
        views = {}
        for name, n, dt in segs:
            nb = n * torch.tensor([], dtype=dt).element_size()
            views[name] = (self.inbuf[offs[name]:offs[name] + nb].view(dt),
                           self.inbuf_host[offs[name]:offs[name] + nb].view(dt).numpy())
        self.ids, self.h_ids = views["ids"]
        self.pos, self.h_pos = views["pos"]
        self.slots, self.h_slots = views["slots"]
        self.seq_rows, self.h_seq_rows = views["seq_rows"]        # block-table rows
        rows, self.h_rows = views["rows"]
        self.rows = rows.view(T, 3)
        self.h_rows = self.h_rows.reshape(T, 3)
        self.kv_end, self.h_kv_end = views["kv_end"]
        self.cond_rows, self.h_cond_rows = views["cond_rows"]
        self.bt_view = None    # [B, max_pages] gathered per step from the KV block table
        self.cond = torch.zeros(B, cfg.cond_hidden_size or 8, dtype=torch.bfloat16, device=dev)
        self.cond_h = torch.zeros(B, h, dtype=torch.bfloat16, device=dev)
        self.x = torch.zeros(T, h, dtype=torch.bfloat16, device=dev)       # residual stream
        self.xn = torch.zeros(T, h, dtype=torch.bfloat16, device=dev)      # normed
        self.q = torch.zeros(T, cfg.num_attention_heads, d, dtype=torch.bfloat16, device=dev)
        self.attn = torch.zeros(T, cfg.q_size, dtype=torch.bfloat16, device=dev)
        self.h = torch.zeros(T, cfg.intermediate_size, dtype=torch.bfloat16, device=dev)
        width = dict(qkv=cfg.q_size + 2 * cfg.kv_size, o=h, gate_up=2 * cfg.intermediate_size, down=h)
        pl = {g: (v if isinstance(v, tuple) else (0, v, False)) for g, v in splits.items() if g in width}
        # fp32 split-K partials for the GEMMs that reduce partials; direct ones write bf16
        nmax = max([pl[g][1] * width[g] for g in width if fused_norm or not pl[g][2]] + [1])
        self.part = torch.zeros(nmax * T, dtype=torch.float32, device=dev)
        # fused norms: per-tile row sums of squares of the residual stream after
        # attention (ss_post) and after the MLP / embedding (ss_in), and the
        # split-K tickets of the GEMMs that reduce into the residual
        ht = math.ceil(h / 128)
        self.ss_in = torch.zeros(ht * T if fused_norm else 1, dtype=torch.float32, device=dev)
        self.ss_post = torch.zeros(ht * T if fused_norm else 1, dtype=torch.float32, device=dev)
        self.ticket = torch.zeros(ht * math.ceil(T / 16) if fused_norm else 1, dtype=torch.int32, device=dev)
        self.qkv = torch.zeros(T if pl["qkv"][2] else 1, width["qkv"], dtype=torch.bfloat16, device=dev)
        self.att_o = torch.zeros(n_chunks * T * cfg.num_attention_heads * d if n_chunks > 1 else 1,
                                 dtype=torch.float32, device=dev)
        self.att_ml = torch.zeros(n_chunks * T * cfg.num_attention_heads * 2 if n_chunks > 1 else 1,
                                  dtype=torch.float32, device=dev)
        kt = 1 if topk <= 1 else (2 if topk <= 2 else 4)
        self.kt = kt
        ntiles = math.ceil(cfg.vocab_size / 128)
        self.ntiles = ntiles
        self.tv = torch.zeros(T * ntiles * kt, dtype=torch.float32, device=dev)
        self.ti = torch.zeros(T * ntiles * kt, dtype=torch.int32, device=dev)
        # topk < 0: the LM head writes fp32 logits of every row (full-vocabulary
        # sampling) instead of the fused top-k
        self.logits = torch.zeros(T, cfg.vocab_size, dtype=torch.float32, device=dev) if topk < 0 else None
        self.top_v = torch.zeros(T, max(topk, 1), dtype=torch.float32, device=dev)
        self.top_i = torch.zeros(T, max(topk, 1), dtype=torch.int64, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)


class FastRunner:
    """Runs forwards of one model on the kernels; captures CUDA graphs per shape."""

    def __init__(self, weights: FastWeights, kv: PagedKV, *, decode_chunk: Optional[int] = None,
                 max_context: int = 4096, batch_invariant: bool = True, device="cuda", tp=None):
        self.w = weights
        self.cfg = weights.cfg          # per-rank shapes under tensor parallelism
        self.kv = kv
        self.device = device
        self.tp = tp                    # d3d_b200.parallel.tp.TPGroup or None
        # Key chunk per attention CTA (a fixed absolute split of the keys, so a
        # row's attention does not depend on the batch it is computed in).
        # D3D_TARGET_CHUNK / D3D_DRAFT_CHUNK override (0 = one chunk over the
        # whole context, no combine pass); the target's chunk must be the same
        # for every forward of a runner (AR and verify), which it is.
        env = os.environ.get("D3D_TARGET_CHUNK" if batch_invariant else "D3D_DRAFT_CHUNK")
        if decode_chunk is None and env is not None:
            decode_chunk = int(env) if int(env) > 0 else -1
        # measured best on B200 (in-graph forward, ~1000-token contexts): 128 keys
        # per CTA for the target's verify / AR forwards, 512 for the drafter's
        # packed forward
        self.decode_chunk = decode_chunk or (128 if batch_invariant else 512)
        self.max_context = max_context
        self.batch_invariant = batch_invariant
        # D3D_FUSE_NORM=1: residual + RMSNorm fused into the target's o / down
        # GEMMs and its qkv / SwiGLU reduce kernels.  Measured on B200 (36-layer
        # 8B forward, CUDA graph): 3557 vs 3632 us at M=1 but 4105 vs 3842 us at
        # M=16 -- the in-kernel tickets and split reduction lengthen each GEMM's
        # tail by more than the launch they save -- so the separate kernels are
        # the default (AR and verify must share one path for token identity).
        self.fused_norm = tp is None and batch_invariant and os.environ.get("D3D_FUSE_NORM", "0") == "1"
        if self.fused_norm:
            weights.fold_norms()
        elif weights.folded:
            raise ValueError("weights with folded norms need the fused-norm forward")
        c = self.cfg
        self.inv_freq = (1.0 / (c.rope_theta ** (torch.arange(0, c.head_dim, 2, dtype=torch.float32)
                                                 / c.head_dim))).to(device)
        self.scale = 1.0 / math.sqrt(c.head_dim)
        self._bufs: Dict[Tuple, StepBuffers] = {}
        self._graphs: Dict[Tuple, torch.cuda.CUDAGraph] = {}
        self.tuned: Dict[int, Dict[str, object]] = {}

    # ------------------------------------------------------------- policies
    GEMMS = ("qkv", "o", "gate_up", "down")
    FIN_MAX_T = int(os.environ.get("D3D_FIN_MAX_T", "64"))

    def _shapes(self) -> Dict[str, Tuple[int, int]]:
        c = self.cfg
        return dict(qkv=(c.q_size + 2 * c.kv_size, c.hidden_size), o=(c.hidden_size, c.q_size),
                    gate_up=(2 * c.intermediate_size, c.hidden_size),
                    down=(c.hidden_size, c.intermediate_size))

    def plan(self, T: int, tune: bool = False) -> Dict[str, Tuple[int, int, bool]]:
        """(token tile, split-K, direct) per GEMM of a T-token forward, plus the
        LM head's token tile under ``"lm_bt"``.

        Batch-invariant runners (the target) take the split from the weight
        shape alone for decode-sized T, so a token's reduction order does not
        depend on how many tokens share the forward, and always reduce fp32
        partials.  Other runners (the drafter) measure their plan on the
        device when decode buffers for a new T are made (``tune``;
        :meth:`_autotune`, off with D3D_AUTOTUNE=0), else use the
        wave-filling heuristic (prefill).
        ``direct`` GEMMs write bf16 themselves (residual add / SwiGLU in the
        epilogue; same rounding as reducing one partial)."""
        bt = ops.bt_for(T)
        shapes = self._shapes()
        if self.batch_invariant:
            if T > 256:
                pl = {g: (bt, 1, False) for g in self.GEMMS}
            else:
                pl = {g: (bt, min(16, ops.splitk_for(n, k, mtiles=1, bt=16)), False)
                      for g, (n, k) in shapes.items()}
            pl["lm_bt"] = bt
            return pl
        if tune and T not in self.tuned and 64 <= T <= 2048 and os.environ.get("D3D_AUTOTUNE", "1") != "0" \
                and torch.cuda.is_available() and not torch.cuda.is_current_stream_capturing():
            self.tuned[T] = self._autotune(T)
        if T in self.tuned:
            return dict(self.tuned[T])
        if T > 2048:
            pl = {g: (bt, 1, False) for g in self.GEMMS}
        else:
            mt = math.ceil(T / bt)
            pl = {g: (bt, ops.splitk_for(n, k, mtiles=mt, bt=bt, m=T), False) for g, (n, k) in shapes.items()}
        pl["lm_bt"] = bt
        return pl

    @torch.no_grad()
    def _autotune(self, T: int, reps: int = 6) -> Dict[str, object]:
        """Time candidate (token tile, split-K, direct) configurations of each
        GEMM at T tokens on this device and keep the fastest.  Weights cycle
        over the model's layers so every timed launch streams from HBM; a
        partial-reducing configuration is timed together with a split-K
        reduction of its partials (``residual_split_reduce``, standing in for
        the consumer kernel), so it pays its partials' round trip where they
        really live -- L2 for small token counts, HBM otherwise, when
        ``D3D_AUTOTUNE_CONSUMER=1``; by default a fixed 6 TB/s charge."""
        E = ops.ext()
        dev = self.device
        L = self.w.layers
        shapes = self._shapes()
        maxk = max(k for _, k in shapes.values())
        maxn = max(n for n, _ in shapes.values())
        x = (torch.randn(T, maxk, device=dev) * 0.1).to(torch.bfloat16)
        part = torch.empty(16 * T * maxn, device=dev)
        yb = torch.zeros(T, maxn, dtype=torch.bfloat16, device=dev)
        st = torch.zeros(1, dtype=torch.int32, device=dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

        def timed(fn):
            fn(0)
            fn(1)
            e0.record()
            for i in range(reps):
                fn(i + 2)
            e1.record()
            e1.synchronize()
            return e0.elapsed_time(e1) / reps * 1e-3

        base = ops.bt_for(T)
        bts = sorted({b for b in (base, ops.bt_for((T + 1) // 2), ops.bt_for((T + 2) // 3), 96, 64, 48, 32)
                      if b <= max(base, 16)}, reverse=True)
        plan: Dict[str, object] = {}
        # measured: timing a real reduction picks nearly the same plans as the
        # fixed charge, at 3238 vs 3201 us per drafter forward, so it is opt-in
        consumer = os.environ.get("D3D_AUTOTUNE_CONSUMER", "0") == "1"
        for g, (n, k) in shapes.items():
            w = lambda i: getattr(L[i % len(L)], g)
            xk = x[:, :k]
            kb = math.ceil(k / 64)
            best = None
            xr = torch.zeros(T, n, dtype=torch.bfloat16, device=dev)
            ss = torch.zeros(math.ceil(n / 128) * T, device=dev)
            # a direct (bf16-output) GEMM's consumer still reads its T x n
            # outputs: charge it one single-split pass over the same size
            t_read = timed(lambda i: E.residual_split_reduce(part, 1, xr, ss)) if consumer else 0.0
            for bt in bts:
                for s in range(1, 17):
                    if s > 1 and kb // s < 4:
                        break
                    if consumer:
                        def fn(i, bt=bt, s=s):
                            E.gemm_partial(xk, w(i).data, part, s, bt, st, n)
                            E.residual_split_reduce(part, s, xr, ss)
                        t = timed(fn)
                    else:
                        t = timed(lambda i: E.gemm_partial(xk, w(i).data, part, s, bt, st, n))
                        t += s * T * n * 4 / 6e12
                    if best is None or t < best[0]:
                        best = (t, bt, s, False)
                if g == "gate_up":
                    h = yb[:, : n // 2]
                    t = timed(lambda i: E.gemm_swiglu(xk, w(i).data, h, bt, st, n)) + t_read / 2
                else:
                    t = timed(lambda i: E.gemm_bf16(xk, w(i).data, yb[:, :n], None, bt, st, n)) + t_read
                if t < best[0]:
                    best = (t, bt, 1, True)
            plan[g] = best[1:]
        if self.w.lm_head is not None:
            lm = self.w.lm_head
            nt = math.ceil(lm.n / 128)
            tv = torch.empty(T * nt * 2, device=dev)
            ti = torch.empty(T * nt * 2, dtype=torch.int32, device=dev)
            xh = x[:, : self.cfg.hidden_size]
            best = None
            for bt in sorted({b for b in (base, ops.bt_for((T + 1) // 2), ops.bt_for((T + 2) // 3), 96, 64, 48)
                              if b <= base}):
                t = timed(lambda i: E.gemm_topk(xh, lm.data, tv, ti, 2, bt, st, lm.n))
                if best is None or t < best[0]:
                    best = (t, bt)
            plan["lm_bt"] = best[1]
        else:
            plan["lm_bt"] = base
        torch.cuda.synchronize()
        if int(st.item()) != 0:
            raise RuntimeError(f"GEMM autotune: kernel reported error {int(st.item())}")
        return plan

    def splits(self, T: int) -> Dict[str, int]:
        return {g: v[1] for g, v in self.plan(T).items() if g in self.GEMMS}

    def buffers(self, B: int, Q: int, topk: int, prefill: bool = False) -> StepBuffers:
        key = (B, Q, topk, prefill)
        b = self._bufs.get(key)
        if b is None:
            T = B * Q
            chunk = self.chunk_for(prefill)
            nch = max(1, math.ceil(self.max_context / chunk))
            b = StepBuffers(self.cfg, B, Q, topk, nch, self.plan(T, tune=not prefill), self.device,
                            fused_norm=self.fused_norm)
            b.bt_view = torch.zeros(B, self.kv.max_pages_per_seq, dtype=torch.int32, device=self.device)
            b.chunk = chunk
            self._bufs[key] = b
        return b

    def _layers_fused(self, b: StepBuffers, E, hq: int, hkv: int, d: int, B: int, Q: int, pl, eps: float) -> int:
        """The decoder layers with the residual add and RMSNorm fused into the
        GEMMs (weights from :meth:`FastWeights.fold_norms`): the o / down
        GEMMs reduce their split-K partials into the residual stream ``x``
        inside the kernel and leave per-tile row sums of squares; the qkv /
        SwiGLU reduce kernels apply the RMSNorm row scale.  The last layer's
        down projection ends in the final add + RMSNorm (``xn``, the hidden
        state the LM head and the handoffs read).  Returns the launch count."""
        w, H = self.w, self.cfg.hidden_size
        n = 0
        last = len(w.layers) - 1
        # decode-sized forwards reduce the o / down splits inside the GEMM (the
        # last unit of a tile does it, no extra launch); larger ones with the
        # stand-alone kernel, whose results are bit-identical
        fin = b.T <= self.FIN_MAX_T
        for li, L in enumerate(w.layers):
            gbt, s, direct = pl["qkv"]
            if direct:
                E.gemm_bf16(b.x, L.qkv.data, b.qkv, None, gbt, b.status, L.qkv.n)
                E.qkv_rope_kv(None, b.qkv, 1, L.q_norm, L.k_norm, self.inv_freq, b.pos, b.slots,
                              b.q, self.kv.k[li], self.kv.v[li], hq, hkv, d, eps, b.status, b.ss_in, H)
            else:
                E.gemm_partial(b.x, L.qkv.data, b.part, s, gbt, b.status, L.qkv.n)
                E.qkv_rope_kv(b.part, None, s, L.q_norm, L.k_norm, self.inv_freq, b.pos, b.slots,
                              b.q, self.kv.k[li], self.kv.v[li], hq, hkv, d, eps, b.status, b.ss_in, H)
            E.attention(b.q, self.kv.k[li], self.kv.v[li], b.bt_view, b.rows, b.kv_end, B, Q, hq, hkv,
                        self.kv.page_size, self.scale, b.chunk, b.n_chunks,
                        b.att_o if b.n_chunks > 1 else None, b.att_ml if b.n_chunks > 1 else None,
                        b.attn, self.batch_invariant, b.status)
            gbt, s, _ = pl["o"]
            if fin:
                E.gemm_partial_fin(b.attn, L.o.data, b.part, s, gbt, b.status, L.o.n, b.x, b.ss_post, b.ticket)
            else:
                E.gemm_partial(b.attn, L.o.data, b.part, s, gbt, b.status, L.o.n)
                E.residual_split_reduce(b.part, s, b.x, b.ss_post)
            gbt, s, _ = pl["gate_up"]
            E.gemm_partial(b.x, L.gate_up.data, b.part, s, gbt, b.status, L.gate_up.n)
            E.swiglu_rowscale(b.part, s, b.h, b.ss_post, H, eps)
            gbt, s, _ = pl["down"]
            if li < last and fin:
                E.gemm_partial_fin(b.h, L.down.data, b.part, s, gbt, b.status, L.down.n, b.x, b.ss_in, b.ticket)
                n += 8 + (1 if b.n_chunks > 1 else 0)
            elif li < last:
                E.gemm_partial(b.h, L.down.data, b.part, s, gbt, b.status, L.down.n)
                E.residual_split_reduce(b.part, s, b.x, b.ss_in)
                n += 10 + (1 if b.n_chunks > 1 else 0)
            else:
                E.gemm_partial(b.h, L.down.data, b.part, s, gbt, b.status, L.down.n)
                E.add_rmsnorm(b.part, s, b.x, w.final_norm, b.xn, eps)
                n += 9 + (1 if b.n_chunks > 1 else 0)
        return n

    def chunk_for(self, prefill: bool) -> int:
        if prefill or self.decode_chunk < 0:
            return max(64, int(math.ceil(self.max_context / 64) * 64))
        return self.decode_chunk

    # -------------------------------------------------------------- forward
    def forward(self, b: StepBuffers, use_cond: bool = False) -> int:
        """Forward over ``b`` (inputs already in place); writes ``b.top_i``/``b.top_v``
        (top-k over the vocabulary of every row) and ``b.xn`` (final hidden).
        Returns the number of kernels launched."""
        E = ops.ext()
        c, w = self.cfg, self.w
        T, B, Q = b.T, b.B, b.Q
        pl = self.plan(T)
        bt = ops.bt_for(T)
        hq, hkv, d = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        cond = None
        if use_cond and w.cond_proj is not None:
            ops.gemm_bf16(b.cond, w.cond_proj, b.cond_h, None, ops.bt_for(B), b.status)
            cond = b.cond_h
        E.embed(b.ids, w.embed, cond, b.cond_rows if cond is not None else None, Q, b.x, b.status)
        if self.fused_norm:
            E.tile_sumsq(b.x, b.ss_in)
        else:
            E.add_rmsnorm(None, 1, b.x, w.layers[0].in_norm, b.xn, c.rms_norm_eps)
        torch.index_select(self.kv.block_table, 0, b.seq_rows, out=b.bt_view)
        n = 3
        eps = c.rms_norm_eps
        tp = self.tp
        if tp is not None:
            tp.bump()
            n += 1
        if self.fused_norm:
            n += self._layers_fused(b, E, hq, hkv, d, B, Q, pl, eps)
        for li, L in enumerate(w.layers if not self.fused_norm else []):
            gbt, s, direct = pl["qkv"]
            if direct:
                E.gemm_bf16(b.xn, L.qkv.data, b.qkv, None, gbt, b.status, L.qkv.n)
                E.qkv_rope_kv(None, b.qkv, 1, L.q_norm, L.k_norm, self.inv_freq, b.pos, b.slots,
                              b.q, self.kv.k[li], self.kv.v[li], hq, hkv, d, eps, b.status)
            else:
                E.gemm_partial(b.xn, L.qkv.data, b.part, s, gbt, b.status, L.qkv.n)
                E.qkv_rope_kv(b.part, None, s, L.q_norm, L.k_norm, self.inv_freq, b.pos, b.slots,
                              b.q, self.kv.k[li], self.kv.v[li], hq, hkv, d, eps, b.status)
            E.attention(b.q, self.kv.k[li], self.kv.v[li], b.bt_view, b.rows, b.kv_end, B, Q, hq, hkv,
                        self.kv.page_size, self.scale, b.chunk, b.n_chunks,
                        b.att_o if b.n_chunks > 1 else None, b.att_ml if b.n_chunks > 1 else None,
                        b.attn, self.batch_invariant, b.status)
            n += 3 + (1 if b.n_chunks > 1 else 0)
            gbt, s, direct = pl["o"]
            if tp is not None:   # row-parallel: partials exchanged, reduced in the norm
                xo = 2 * li
                tp.gemm(b.attn, L.o, xo, s, gbt)
                tp.add_rmsnorm(xo, xo, s, b.x, L.post_norm, b.xn, eps)
            elif direct:   # residual added in the epilogue, in place
                E.gemm_bf16(b.attn, L.o.data, b.x, b.x, gbt, b.status, L.o.n)
                E.add_rmsnorm(None, 1, b.x, L.post_norm, b.xn, eps)
            else:
                E.gemm_partial(b.attn, L.o.data, b.part, s, gbt, b.status, L.o.n)
                E.add_rmsnorm(b.part, s, b.x, L.post_norm, b.xn, eps)
            gbt, s, direct = pl["gate_up"]
            if direct:
                E.gemm_swiglu(b.xn, L.gate_up.data, b.h, gbt, b.status, L.gate_up.n)
                n += 3
            else:
                E.gemm_partial(b.xn, L.gate_up.data, b.part, s, gbt, b.status, L.gate_up.n)
                E.swiglu(b.part, s, b.h, True)
                n += 4
            nxt = w.layers[li + 1].in_norm if li + 1 < len(w.layers) else w.final_norm
            gbt, s, direct = pl["down"]
            if tp is not None:
                xd = 2 * li + 1
                tp.gemm(b.h, L.down, xd, s, gbt)
                tp.add_rmsnorm(xd, xd, s, b.x, nxt, b.xn, eps)
            elif direct:
                E.gemm_bf16(b.h, L.down.data, b.x, b.x, gbt, b.status, L.down.n)
                E.add_rmsnorm(None, 1, b.x, nxt, b.xn, eps)
            else:
                E.gemm_partial(b.h, L.down.data, b.part, s, gbt, b.status, L.down.n)
                E.add_rmsnorm(b.part, s, b.x, nxt, b.xn, eps)
            n += 2
        if b.topk > 0:
            E.gemm_topk(b.xn, w.lm_head.data, b.tv, b.ti, b.topk, pl["lm_bt"], b.status, w.lm_head.n)
            E.topk_merge(b.tv, b.ti, T, b.ntiles, b.kt, b.topk, b.top_v, b.top_i)
            if tp is not None:   # vocab-parallel: merge the ranks' candidates (global ids)
                xl = 2 * len(w.layers)
                E.tp_publish_topk(b.top_v, b.top_i, tp.rank * c.vocab_size, tp.cand_view())
                tp.signal(xl)
                tp.merge_topk(xl, T, b.topk, b.top_v, b.top_i)
                n += 3
        n += 2 if b.topk > 0 else 0
        if b.topk < 0:
            if tp is not None:
                raise NotImplementedError("full-vocabulary logits with a tensor-parallel LM head")
            E.gemm_partial(b.xn, w.lm_head.data, b.logits, 1, pl["lm_bt"], b.status, w.lm_head.n)
            n += 1
        return n + (1 if cond is not None else 0)
