"""Model configuration for the Qwen3 target and the block-diffusion drafter.

The on-disk format is the Hugging Face ``config.json`` of a Qwen3 checkpoint.
A drafter checkpoint is a Qwen3 checkpoint whose config also carries
``d3d_draft: true`` and ``mask_token_id`` and still names
``architectures: ["Qwen3ForCausalLM"]`` (reference:
``models/d3d/configuration_d3d.py:211-215``; mask-id validation
``models/token_ids.py:8-18``).  Reading and writing this file keeps released
checkpoints loadable unchanged.

Two optional fields are additions of this framework:

* ``block_size``: the diffusion block length the drafter was trained for.
* ``cond_hidden_size``: when set, the drafter owns a ``cond_proj`` linear map
  from the target's last-layer hidden state (of that width) into its own
  embedding width, added to the embedding of the anchor slot of every block.
  It is absent (``None``) for released checkpoints, which are token-only.
"""
from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Optional

DEFAULT_MASK_TOKEN_ID = 151669
QWEN3_EOS_IDS = (151643, 151645)


@dataclass
class ModelConfig:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    max_position_embeddings: int = 40960
    tie_word_embeddings: bool = False
    attention_bias: bool = False
    initializer_range: float = 0.02
    # drafter fields
    d3d_draft: bool = False
    mask_token_id: Optional[int] = None
    block_size: Optional[int] = None
    cond_hidden_size: Optional[int] = None
    # fields carried through unchanged when a checkpoint is rewritten
    extra: dict = field(default_factory=dict, repr=False, compare=False)

    # ------------------------------------------------------------------ derived
    @property
    def q_size(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def gqa_group(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads

    def num_parameters(self) -> int:
        h, i, v = self.hidden_size, self.intermediate_size, self.vocab_size
        per_layer = (
            h * (self.q_size + 2 * self.kv_size)
            + self.q_size * h
            + 3 * h * i
            + 2 * h
            + 2 * self.head_dim
        )
        n = v * h + self.num_hidden_layers * per_layer + h
        if not self.tie_word_embeddings:
            n += v * h
        if self.cond_hidden_size:
            n += self.cond_hidden_size * h
        return n

    def validate(self) -> "ModelConfig":
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("num_attention_heads must be a multiple of num_key_value_heads")
        if self.d3d_draft:
            mid = self.mask_token_id
            if mid is None:
                raise ValueError("a drafter config needs mask_token_id")
            if not 0 <= int(mid) < self.vocab_size:
                raise ValueError(
                    f"mask token ID {mid} is outside checkpoint vocabulary {self.vocab_size}")
        return self

    # ------------------------------------------------------------- HF json io
    _HF_KEYS = (
        "vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
        "num_attention_heads", "num_key_value_heads", "head_dim", "rms_norm_eps",
        "rope_theta", "max_position_embeddings", "tie_word_embeddings",
        "attention_bias", "initializer_range",
    )

    @classmethod
    def from_hf_dict(cls, d: dict, mask_token_id: Optional[int] = None) -> "ModelConfig":
        kw: dict[str, Any] = {}
        for k in cls._HF_KEYS:
            if k in d and d[k] is not None:
                kw[k] = d[k]
        if "head_dim" not in kw:
            kw["head_dim"] = d["hidden_size"] // d["num_attention_heads"]
        rope = d.get("rope_parameters") or {}
        if "rope_theta" not in kw and "rope_theta" in rope:
            kw["rope_theta"] = rope["rope_theta"]
        draft = bool(d.get("d3d_draft", False))
        saved_mid = d.get("mask_token_id")
        if saved_mid is not None and mask_token_id is not None and int(saved_mid) != int(mask_token_id):
            raise ValueError("--mask-token-id conflicts with the checkpoint's mask_token_id")
        mid = mask_token_id if mask_token_id is not None else saved_mid
        if draft and mid is None:
            mid = DEFAULT_MASK_TOKEN_ID
        known = set(cls._HF_KEYS) | {"d3d_draft", "mask_token_id", "block_size",
                                     "cond_hidden_size", "architectures", "model_type"}
        extra = {k: v for k, v in d.items() if k not in known}
        return cls(
            d3d_draft=draft,
            mask_token_id=None if mid is None else int(mid),
            block_size=d.get("block_size"),
            cond_hidden_size=d.get("cond_hidden_size"),
            extra=extra,
            **kw,
        ).validate()

    def to_hf_dict(self) -> dict:
        d = dict(self.extra)
        for k in self._HF_KEYS:
            d[k] = getattr(self, k)
        d["architectures"] = ["Qwen3ForCausalLM"]
        d["model_type"] = "qwen3"
        d.setdefault("hidden_act", "silu")
        d.setdefault("torch_dtype", "float32")
        if self.d3d_draft:
            d["d3d_draft"] = True
            d["mask_token_id"] = self.mask_token_id
            if self.block_size is not None:
                d["block_size"] = self.block_size
            if self.cond_hidden_size is not None:
                d["cond_hidden_size"] = self.cond_hidden_size
        return d

    @classmethod
    def from_pretrained(cls, path: str | Path, mask_token_id: Optional[int] = None) -> "ModelConfig":
        p = Path(path) / "config.json"
        if not p.is_file():
            raise FileNotFoundError(f"Missing config.json in checkpoint: {path}")
        return cls.from_hf_dict(json.loads(p.read_text()), mask_token_id=mask_token_id)

    def save(self, path: str | Path) -> None:
        Path(path).mkdir(parents=True, exist_ok=True)
        (Path(path) / "config.json").write_text(json.dumps(self.to_hf_dict(), indent=2, sort_keys=True))

    def replace(self, **kw) -> "ModelConfig":
        return dataclasses.replace(self, **kw)


# ---------------------------------------------------------------- presets
def qwen3_8b() -> ModelConfig:
    return ModelConfig(vocab_size=151936, hidden_size=4096, intermediate_size=12288,
                       num_hidden_layers=36, num_attention_heads=32, num_key_value_heads=8,
                       head_dim=128, tie_word_embeddings=False)


def qwen3_32b() -> ModelConfig:
    return ModelConfig(vocab_size=151936, hidden_size=5120, intermediate_size=25600,
                       num_hidden_layers=64, num_attention_heads=64, num_key_value_heads=8,
                       head_dim=128, tie_word_embeddings=False)


def d3d_1p7b(num_layers: int = 28, cond_hidden_size: Optional[int] = None,
             block_size: int = 16) -> ModelConfig:
    return ModelConfig(vocab_size=151936, hidden_size=2048, intermediate_size=6144,
                       num_hidden_layers=num_layers, num_attention_heads=16,
                       num_key_value_heads=8, head_dim=128, tie_word_embeddings=True,
                       d3d_draft=True, mask_token_id=DEFAULT_MASK_TOKEN_ID,
                       block_size=block_size, cond_hidden_size=cond_hidden_size)


def tiny_target() -> ModelConfig:
    return ModelConfig(vocab_size=1024, hidden_size=128, intermediate_size=384,
                       num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                       head_dim=32, tie_word_embeddings=False, max_position_embeddings=4096)


def tiny_drafter(cond: bool = True) -> ModelConfig:
    return ModelConfig(vocab_size=1024, hidden_size=128, intermediate_size=384,
                       num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                       head_dim=32, tie_word_embeddings=False, max_position_embeddings=4096,
                       d3d_draft=True, mask_token_id=1023, block_size=8,
                       cond_hidden_size=128 if cond else None)


PRESETS = {
    "qwen3-8b": qwen3_8b,
    "qwen3-32b": qwen3_32b,
    "d3d-1.7b": d3d_1p7b,
    "d3d-1.7b-pruned24": lambda: d3d_1p7b(num_layers=24),
    "tiny-target": tiny_target,
    "tiny-drafter": tiny_drafter,
}
