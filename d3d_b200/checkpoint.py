"""Hugging Face-layout safetensors checkpoints (FP32 on disk, bf16 at runtime).

Layout: ``config.json`` plus ``model.safetensors`` or
``model-XXXXX-of-YYYYY.safetensors`` shards with ``model.safetensors.index.json``
— the format of the reference's training saves (``train/runtime.py:224-259``)
and of released D3D checkpoints (``docs/models.md:5-26``).  Loading is strict
like the reference's SSD loader (``serving/vendor/ssd/utils/loader.py:188-262``):
every expected tensor must be present exactly once with the expected shape,
and unexpected tensors are rejected.

Tensor-parallel loading (:func:`load_tp_shard`) slices column-parallel weights
(q/k/v, gate/up) by output rows and row-parallel weights (o, down) by input
columns on load, so a rank never materialises the full matrix on the GPU.
"""
from __future__ import annotations

import json
import os
import tempfile
from pathlib import Path
from typing import Dict, Iterable, Optional

import torch

from .config import ModelConfig
from .models.qwen3 import Qwen3LM

INDEX = "model.safetensors.index.json"


def _st():
    import safetensors.torch as st
    return st


def expected_keys(cfg: ModelConfig) -> Dict[str, tuple]:
    h, i, d = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    k: Dict[str, tuple] = {"model.embed_tokens.weight": (cfg.vocab_size, h), "model.norm.weight": (h,)}
    if not cfg.tie_word_embeddings:
        k["lm_head.weight"] = (cfg.vocab_size, h)
    if cfg.cond_hidden_size:
        k["cond_proj.weight"] = (h, cfg.cond_hidden_size)
    for n in range(cfg.num_hidden_layers):
        p = f"model.layers.{n}."
        k[p + "self_attn.q_proj.weight"] = (cfg.q_size, h)
        k[p + "self_attn.k_proj.weight"] = (cfg.kv_size, h)
        k[p + "self_attn.v_proj.weight"] = (cfg.kv_size, h)
        k[p + "self_attn.o_proj.weight"] = (h, cfg.q_size)
        k[p + "self_attn.q_norm.weight"] = (d,)
        k[p + "self_attn.k_norm.weight"] = (d,)
        k[p + "mlp.gate_proj.weight"] = (i, h)
        k[p + "mlp.up_proj.weight"] = (i, h)
        k[p + "mlp.down_proj.weight"] = (h, i)
        k[p + "input_layernorm.weight"] = (h,)
        k[p + "post_attention_layernorm.weight"] = (h,)
    return k


def _shard_files(path: Path) -> Dict[str, str]:
    """tensor name -> shard file (validated index)."""
    idx = path / INDEX
    if idx.is_file():
        wm = json.loads(idx.read_text())["weight_map"]
        files = set(wm.values())
        for f in files:
            if not (path / f).is_file():
                raise FileNotFoundError(f"missing shard {f} listed in {INDEX}")
        return dict(wm)
    single = path / "model.safetensors"
    if not single.is_file():
        raise FileNotFoundError(f"no safetensors weights in {path}")
    with _st().safe_open(str(single), "pt") as f:
        return {k: "model.safetensors" for k in f.keys()}


def read_state(path: str | Path, keys: Optional[Iterable[str]] = None,
               dtype: Optional[torch.dtype] = None) -> Dict[str, torch.Tensor]:
    path = Path(path)
    wm = _shard_files(path)
    want = set(wm) if keys is None else set(keys)
    by_file: Dict[str, list] = {}
    for k in want:
        if k not in wm:
            raise KeyError(f"checkpoint {path} is missing tensor {k}")
        by_file.setdefault(wm[k], []).append(k)
    out = {}
    for f, ks in by_file.items():
        with _st().safe_open(str(path / f), "pt") as fh:
            for k in ks:
                t = fh.get_tensor(k)
                out[k] = t.to(dtype) if dtype is not None else t
    return out


def load_model(path: str | Path, device="cpu", dtype=torch.float32, strict: bool = True,
               mask_token_id: Optional[int] = None) -> Qwen3LM:
    cfg = ModelConfig.from_pretrained(path, mask_token_id=mask_token_id)
    exp = expected_keys(cfg)
    wm = _shard_files(Path(path))
    if strict:
        missing = sorted(set(exp) - set(wm))
        extra = sorted(set(wm) - set(exp) - ({"lm_head.weight"} if cfg.tie_word_embeddings else set()))
        if missing:
            raise ValueError(f"checkpoint {path} is missing {len(missing)} tensors, e.g. {missing[:3]}")
        if extra:
            raise ValueError(f"checkpoint {path} has unexpected tensors, e.g. {extra[:3]}")
    state = read_state(path, exp.keys())
    for k, shape in exp.items():
        if tuple(state[k].shape) != tuple(shape):
            raise ValueError(f"{k}: shape {tuple(state[k].shape)} != expected {shape}")
    m = Qwen3LM(cfg)
    m.load_state_dict(state, strict=True)
    return m.to(device=device, dtype=dtype)


def save_model(model: Qwen3LM, path: str | Path, max_shard_bytes: int = 4 << 30,
               dtype=torch.float32, extra: Optional[Dict[str, torch.Tensor]] = None) -> None:
    """Atomic save: write into a temp dir next to ``path`` and rename.
    ``extra``: tensors the module does not hold itself (the gathered weights
    of sharded decoder layers), stored under their own names."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = Path(tempfile.mkdtemp(prefix=path.name + ".tmp", dir=str(path.parent)))
    state = {k: v.detach().to("cpu", dtype).contiguous() for k, v in model.state_dict().items()}
    for k, v in (extra or {}).items():
        state[k] = v.detach().to("cpu", dtype).contiguous()
    if model.cfg.tie_word_embeddings:
        state.pop("lm_head.weight", None)
    write_state(state, tmp, max_shard_bytes)
    model.cfg.save(tmp)
    if path.exists():
        old = path.with_name(path.name + ".old")
        os.replace(path, old)
        os.replace(tmp, path)
        import shutil
        shutil.rmtree(old, ignore_errors=True)
    else:
        os.replace(tmp, path)


def write_state(state: Dict[str, torch.Tensor], path: Path, max_shard_bytes: int = 4 << 30) -> None:
    st = _st()
    shards, cur, size = [], {}, 0
    for k in sorted(state):
        n = state[k].numel() * state[k].element_size()
        if cur and size + n > max_shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = state[k]
        size += n
    if cur:
        shards.append(cur)
    if len(shards) == 1:
        st.save_file(shards[0], str(path / "model.safetensors"), metadata={"format": "pt"})
        return
    wm = {}
    for i, sh in enumerate(shards):
        name = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        st.save_file(sh, str(path / name), metadata={"format": "pt"})
        wm.update({k: name for k in sh})
    total = sum(t.numel() * t.element_size() for t in state.values())
    (path / INDEX).write_text(json.dumps({"metadata": {"total_size": total}, "weight_map": wm}, indent=2))


def load_tp_shard(path: str | Path, rank: int, world: int, device="cuda",
                  dtype=torch.bfloat16) -> Dict[str, torch.Tensor]:
    """The rank's slice of every tensor for Megatron-style tensor parallelism.

    Column-parallel (split output rows): q/k/v, gate/up, and the LM head
    (vocab-parallel).  Row-parallel (split input columns): o, down.  Norms
    and embeddings are replicated.  Slices are read straight from the
    safetensors files (only this rank's part of a split tensor is read), one
    tensor at a time, so host memory stays at one tensor."""
    cfg = ModelConfig.from_pretrained(path)
    if cfg.num_key_value_heads % world or cfg.num_attention_heads % world:
        raise ValueError("heads must divide the tensor-parallel world size")
    path = Path(path)
    wm = _shard_files(path)
    want = set(expected_keys(cfg))
    if cfg.tie_word_embeddings:
        want.discard("lm_head.weight")
    by_file: Dict[str, list] = {}
    for k in want:
        if k not in wm:
            raise KeyError(f"checkpoint {path} is missing tensor {k}")
        by_file.setdefault(wm[k], []).append(k)
    out = {}
    for f, ks in by_file.items():
        with _st().safe_open(str(path / f), "pt") as fh:
            for k in sorted(ks):
                sl = fh.get_slice(k)
                shape = sl.get_shape()
                if any(n in k for n in ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj")) or k == "lm_head.weight":
                    step = shape[0] // world
                    t = sl[rank * step:(rank + 1) * step]
                elif "o_proj" in k or "down_proj" in k:
                    step = shape[1] // world
                    t = sl[:, rank * step:(rank + 1) * step]
                else:
                    t = sl[:]
                out[k] = t.to(device=device, dtype=dtype).contiguous()
    if cfg.tie_word_embeddings:
        v = cfg.vocab_size // world
        out["lm_head.weight"] = out["model.embed_tokens.weight"][rank * v:(rank + 1) * v].contiguous()
    return out
