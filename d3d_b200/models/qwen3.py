"""Qwen3 decoder in plain PyTorch: the target model, the drafter, and the oracle.

One module serves three roles:

* the **target** (a stock Qwen3: GQA attention, per-head QK-RMSNorm, RoPE,
  SwiGLU MLP; reference ``serving/vendor/ssd/models/qwen3.py:14-325``);
* the **block-diffusion drafter** (the same network, fed ``MASK`` tokens and an
  arbitrary boolean attention mask that is bidirectional inside a block and
  reads the causal prefix KV; reference ``models/d3d/modeling_d3d.py:221-644``),
  optionally conditioned on the target's last-layer hidden state;
* the **CPU oracle** for every CUDA kernel and for the fast engine: this path is
  written for clarity, runs in fp32 on the CPU and supports autograd, which the
  training stack uses.

Parameter names are Hugging Face's (``model.layers.N.self_attn.q_proj.weight``
and so on), so released checkpoints load without renaming.  The fast CUDA path
lives in :mod:`d3d_b200.models.fast`; it reads the weights of this module.
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence

import torch
import torch.nn.functional as F
from torch import nn

from ..config import ModelConfig


class RMSNorm(nn.Module):
    """RMSNorm with the Hugging Face Qwen3 rounding order (fp32 statistics,
    scale applied after the cast back to the input dtype)."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dt = x.dtype
        xf = x.float()
        xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return self.weight * xf.to(dt)


def rope_cos_sin(positions: torch.Tensor, head_dim: int, theta: float,
                 dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables for rotate-half RoPE, computed in fp32 ([..., head_dim])."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32,
                                        device=positions.device) / head_dim))
    freqs = positions.to(torch.float32)[..., None] * inv
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


class DenseKVCache:
    """Contiguous per-layer K/V cache with HF ``DynamicCache`` semantics
    (append on store, ``crop`` to roll back).  Shapes ``[B, Hkv, L, D]``."""

    def __init__(self, num_layers: int):
        self.k: List[Optional[torch.Tensor]] = [None] * num_layers
        self.v: List[Optional[torch.Tensor]] = [None] * num_layers

    @property
    def length(self) -> int:
        return 0 if self.k[0] is None else int(self.k[0].shape[2])

    def get(self, layer: int):
        return self.k[layer], self.v[layer]

    def append(self, layer: int, k: torch.Tensor, v: torch.Tensor):
        if self.k[layer] is None:
            self.k[layer], self.v[layer] = k, v
        else:
            self.k[layer] = torch.cat([self.k[layer], k], dim=2)
            self.v[layer] = torch.cat([self.v[layer], v], dim=2)
        return self.k[layer], self.v[layer]

    def crop(self, length: int) -> None:
        length = int(length)
        for i in range(len(self.k)):
            if self.k[i] is not None:
                self.k[i] = self.k[i][:, :, :length]
                self.v[i] = self.v[i][:, :, :length]

    def clone(self) -> "DenseKVCache":
        c = DenseKVCache(len(self.k))
        c.k = [None if t is None else t.clone() for t in self.k]
        c.v = [None if t is None else t.clone() for t in self.v]
        return c


class _TcLinearFn(torch.autograd.Function):
    """``y = x W^T`` and its gradients on the tcgen05 GEMM of
    ``ops/csrc/gemm_tcgen05.cu`` (bf16 operands, fp32 accumulation):

    * forward  ``y[m, n]  = sum_k x[m, k] W[n, k]``          (bf16 out);
    * backward ``dx[m, k] = sum_n dy[m, n] W^T[k, n]``        (bf16 out);
    * backward ``dW[n, k] = sum_m dy^T[n, m] x^T[k, m]``      (fp32 out).

    The kernel contracts over the contiguous dimension of both operands, so
    the backward products read transposed copies (one copy kernel each)."""

    @staticmethod
    def forward(ctx, x2, w):
        from .. import ops
        y = torch.empty(x2.shape[0], w.shape[0], dtype=torch.bfloat16, device=x2.device)
        ops.gemm_bf16(x2, w, y)
        ctx.save_for_backward(x2, w)
        return y

    @staticmethod
    def backward(ctx, gy):
        from .. import ops
        x2, w = ctx.saved_tensors
        gy = gy.to(torch.bfloat16).contiguous()
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty_like(x2)
            ops.gemm_bf16(gy, w.t().contiguous(), dx)
        if ctx.needs_input_grad[1]:
            dw32 = torch.empty(w.shape, dtype=torch.float32, device=w.device)
            ops.gemm_partial(gy.t().contiguous(), x2.t().contiguous(), dw32, 1)
            dw = dw32.to(w.dtype)
        return dx, dw


# tcgen05 linears for bf16 CUDA tensors (D3D_TC_LINEAR=0 uses torch's GEMM)
TC_LINEAR = True


class Linear(nn.Linear):
    """``nn.Linear`` (same parameters and names) whose bf16 CUDA path runs on
    the framework's tcgen05 GEMM, forward and backward; other devices and
    dtypes use ``F.linear``."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        rows = x.numel() // max(1, self.in_features)
        # TMA rows of every operand (forward and both backward products) must be
        # multiples of 16 bytes: in, out features and token count multiples of 8
        if (TC_LINEAR and x.is_cuda and x.dtype == torch.bfloat16 and self.weight.dtype == torch.bfloat16
                and self.bias is None and self.in_features % 8 == 0 and self.out_features % 8 == 0
                and rows > 0 and rows % 8 == 0):
            import os
            if os.environ.get("D3D_TC_LINEAR", "1") != "0":
                x2 = x.reshape(-1, self.in_features).contiguous()
                return _TcLinearFn.apply(x2, self.weight).view(*x.shape[:-1], self.out_features)
        return F.linear(x, self.weight, self.bias)


class Attention(nn.Module):
    impl = "sdpa"   # "sdpa" (torch's fused attention) or "eager" (explicit fp32 softmax)

    def __init__(self, cfg: ModelConfig, layer_idx: int):
        super().__init__()
        self.cfg = cfg
        self.layer_idx = layer_idx
        h, d = cfg.hidden_size, cfg.head_dim
        self.q_proj = Linear(h, cfg.q_size, bias=cfg.attention_bias)
        self.k_proj = Linear(h, cfg.kv_size, bias=cfg.attention_bias)
        self.v_proj = Linear(h, cfg.kv_size, bias=cfg.attention_bias)
        self.o_proj = Linear(cfg.q_size, h, bias=cfg.attention_bias)
        self.q_norm = RMSNorm(d, cfg.rms_norm_eps)
        self.k_norm = RMSNorm(d, cfg.rms_norm_eps)

    def forward(self, x, cos, sin, mask, cache: Optional[DenseKVCache], store_kv: bool):
        b, q, _ = x.shape
        d = self.cfg.head_dim
        qs = self.q_norm(self.q_proj(x).view(b, q, -1, d)).transpose(1, 2)
        ks = self.k_norm(self.k_proj(x).view(b, q, -1, d)).transpose(1, 2)
        vs = self.v_proj(x).view(b, q, -1, d).transpose(1, 2)
        c, s = cos[:, None], sin[:, None]
        qs = qs * c + rotate_half(qs) * s
        ks = ks * c + rotate_half(ks) * s
        if cache is not None:
            if store_kv:
                ks, vs = cache.append(self.layer_idx, ks, vs)
            elif cache.k[self.layer_idx] is not None:
                pk, pv = cache.get(self.layer_idx)
                ks = torch.cat([pk, ks], dim=2)
                vs = torch.cat([pv, vs], dim=2)
        g = self.cfg.gqa_group
        if g > 1:
            ks = ks.repeat_interleave(g, dim=1)
            vs = vs.repeat_interleave(g, dim=1)
        attn_mask = None
        if mask is not None:
            attn_mask = mask[:, None, :, : ks.shape[2]]
        if self.impl == "eager":
            sc = torch.matmul(qs.float(), ks.float().transpose(-1, -2)) / math.sqrt(d)
            if attn_mask is not None:
                sc = (sc.masked_fill(~attn_mask, float("-inf")) if attn_mask.dtype == torch.bool
                      else sc + attn_mask.float())
            out = torch.matmul(torch.softmax(sc, -1), vs.float()).to(vs.dtype)
        else:
            out = F.scaled_dot_product_attention(qs, ks, vs, attn_mask=attn_mask,
                                                 scale=1.0 / math.sqrt(d))
        out = out.transpose(1, 2).reshape(b, q, -1)
        return self.o_proj(out)


class MLP(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.gate_proj = Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.up_proj = Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.down_proj = Linear(cfg.intermediate_size, cfg.hidden_size, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class DecoderLayer(nn.Module):
    def __init__(self, cfg: ModelConfig, layer_idx: int):
        super().__init__()
        self.self_attn = Attention(cfg, layer_idx)
        self.mlp = MLP(cfg)
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)

    def forward(self, x, cos, sin, mask, cache, store_kv):
        x = x + self.self_attn(self.input_layernorm(x), cos, sin, mask, cache, store_kv)
        return x + self.mlp(self.post_attention_layernorm(x))


class Backbone(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList(DecoderLayer(cfg, i) for i in range(cfg.num_hidden_layers))
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)


class Qwen3LM(nn.Module):
    """Qwen3 causal LM / D3D drafter.

    ``forward`` returns the final-norm hidden states ``[B, Q, H]``; call
    :meth:`logits` to project them.  ``mask`` is a boolean ``[B, Q, S]`` tensor
    over keys ``[cache ; new tokens]`` (``True`` = visible); ``None`` means
    causal attention over the cache plus the new tokens.
    """

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        cfg.validate()
        self.cfg = cfg
        self.model = Backbone(cfg)
        if not cfg.tie_word_embeddings:
            self.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)
        if cfg.cond_hidden_size:
            self.cond_proj = nn.Linear(cfg.cond_hidden_size, cfg.hidden_size, bias=False)
        self.gradient_checkpointing = False

    # ------------------------------------------------------------------ init
    def set_attn_implementation(self, name: Optional[str]) -> str:
        """Attention math of this module: ``sdpa`` (default) or ``eager``.
        ``flash_attention_2`` (the Hugging Face name) selects ``sdpa``, whose
        dispatcher picks the fused flash kernel where the mask allows.
        Returns the implementation in effect."""
        impl = {None: "sdpa", "sdpa": "sdpa", "flash_attention_2": "sdpa", "eager": "eager"}.get(name)
        if impl is None:
            raise ValueError(f"unknown attention implementation {name!r} (sdpa, eager, flash_attention_2)")
        for m in self.modules():
            if isinstance(m, Attention):
                m.impl = impl
        return impl

    @torch.no_grad()
    def init_weights(self, seed: int = 0, std: Optional[float] = None) -> "Qwen3LM":
        """Seeded N(0, std) init of every linear/embedding; norms at 1."""
        std = self.cfg.initializer_range if std is None else std
        g = torch.Generator(device="cpu").manual_seed(int(seed))
        for name, p in self.named_parameters():
            if name.endswith("norm.weight") or "layernorm" in name:
                p.fill_(1.0)
            else:
                p.copy_(torch.randn(p.shape, generator=g, dtype=torch.float32) * std)
        return self

    @property
    def lm_weight(self) -> torch.Tensor:
        return self.model.embed_tokens.weight if self.cfg.tie_word_embeddings else self.lm_head.weight

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return F.linear(hidden, self.lm_weight)

    # --------------------------------------------------------------- forward
    def embed(self, input_ids, cond=None, cond_rows=None):
        x = self.model.embed_tokens(input_ids)
        if cond is not None and getattr(self, "cond_proj", None) is not None:
            c = self.cond_proj(cond.to(x.dtype))  # [B, H]
            if cond_rows is None:
                cond_rows = torch.zeros(input_ids.shape, dtype=torch.bool, device=input_ids.device)
                cond_rows[:, 0] = True
            x = x + cond_rows[..., None].to(x.dtype) * c[:, None, :]
        return x

    def forward(self, input_ids: torch.Tensor, positions: Optional[torch.Tensor] = None,
                mask: Optional[torch.Tensor] = None, cache: Optional[DenseKVCache] = None,
                store_kv: bool = False, cond: Optional[torch.Tensor] = None,
                cond_rows: Optional[torch.Tensor] = None,
                output_hidden_states: bool = False,
                layer_skip: Optional[Sequence[int]] = None):
        b, q = input_ids.shape
        past = cache.length if cache is not None else 0
        if positions is None:
            positions = torch.arange(past, past + q, device=input_ids.device)[None].expand(b, q)
        if mask is None:
            qpos = torch.arange(past, past + q, device=input_ids.device)
            kpos = torch.arange(past + q, device=input_ids.device)
            mask = (kpos[None, :] <= qpos[:, None])[None].expand(b, q, past + q)
        x = self.embed(input_ids, cond, cond_rows)
        cos, sin = rope_cos_sin(positions, self.cfg.head_dim, self.cfg.rope_theta, x.dtype)
        hidden_states = [x] if output_hidden_states else None
        skip = set(layer_skip or ())
        for i, layer in enumerate(self.model.layers):
            if i in skip:
                if hidden_states is not None:
                    hidden_states.append(x)
                continue
            if self.gradient_checkpointing and self.training and not store_kv and torch.is_grad_enabled():
                # per-layer recomputation; a clean-prefix cache is only read
                # here, so the recomputed layer sees the same keys and values
                x = torch.utils.checkpoint.checkpoint(layer, x, cos, sin, mask, cache, False,
                                                      use_reentrant=False)
            else:
                x = layer(x, cos, sin, mask, cache, store_kv)
            if hidden_states is not None:
                hidden_states.append(x)
        out = self.model.norm(x)
        if output_hidden_states:
            return out, hidden_states
        return out


def build_model(cfg: ModelConfig, seed: Optional[int] = 0, dtype=torch.float32,
                device="cpu") -> Qwen3LM:
    m = Qwen3LM(cfg)
    if seed is not None:
        m.init_weights(seed)
    return m.to(device=device, dtype=dtype)
