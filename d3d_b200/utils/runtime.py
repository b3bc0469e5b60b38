"""Paths, hardware checks, capacity checks and run metadata
(reference: ``common/runtime.py``)."""
from __future__ import annotations

import hashlib
import importlib.metadata
import json
import math
import platform
import subprocess
from pathlib import Path
from typing import Dict, Iterable, Optional, Sequence

from ..engine.layout import paged_draft_branch_tokens


def resolve_model_path(model: str) -> str:
    """A local checkpoint directory (no network downloads in this build)."""
    p = Path(model).expanduser()
    if not p.is_dir():
        raise FileNotFoundError(f"Model directory does not exist: {model}")
    if not (p / "config.json").is_file():
        raise FileNotFoundError(f"Missing config.json in checkpoint: {p}")
    return str(p.resolve())


def check_hardware(devices: Sequence[str] = ("cuda:0",), distinct: bool = False) -> None:
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is unavailable")
    if distinct and len(set(devices)) != len(devices):
        raise ValueError("target and draft must use distinct CUDA devices in this mode")
    for name in devices:
        d = torch.device(name)
        if d.type != "cuda" or d.index is None or d.index >= torch.cuda.device_count():
            raise ValueError(f"Unavailable CUDA device: {name}")
        if torch.cuda.get_device_capability(d) < (10, 0):
            raise RuntimeError(f"{name} is not an sm_100 (Blackwell) device")


def required_pages(prompt_lens: Iterable[int], max_new_tokens: int, concurrency: int, page_size: int,
                   extra: int) -> int:
    need = max(prompt_lens) + int(max_new_tokens) + int(extra)
    return int(concurrency) * math.ceil(need / int(page_size))


def check_paged_capacity(prompt_lens: Sequence[int], max_new_tokens: int, concurrency: Iterable[int],
                         pages: int, page_size: int, block_size: int = 16, anchor_num: int = 3,
                         context_limit: int = 16384) -> None:
    """Raise if a concurrency level cannot fit its KV (target and draft)."""
    branch = paged_draft_branch_tokens(block_size, max(anchor_num, 1))
    for name, extra in (("target", block_size), ("draft", branch)):
        need = max(prompt_lens) + max_new_tokens + extra
        if need > context_limit:
            raise ValueError(f"{name} context limit {context_limit} is too small: need {need} tokens")
        for c in concurrency:
            req = required_pages(prompt_lens, max_new_tokens, min(c, len(prompt_lens)), page_size, extra)
            if req > pages:
                raise ValueError(f"{name} needs {req} pages at concurrency {c}; configured pages={pages}")


def runtime_metadata(models: Optional[Dict[str, str]] = None) -> dict:
    import torch
    versions = {}
    for pkg in ("torch", "transformers", "safetensors", "numpy"):
        try:
            versions[pkg] = importlib.metadata.version(pkg)
        except importlib.metadata.PackageNotFoundError:
            versions[pkg] = None
    root = Path(__file__).resolve().parents[2]
    commit = None
    if (root / ".git").exists():
        r = subprocess.run(["git", "-C", str(root), "rev-parse", "HEAD"], capture_output=True, text=True)
        commit = r.stdout.strip() if r.returncode == 0 else None
    ckpts = {}
    for name, path in (models or {}).items():
        try:
            cfg = json.loads((Path(path) / "config.json").read_text())
            ckpts[name] = {"model_type": cfg.get("model_type"), "d3d_draft": bool(cfg.get("d3d_draft"))}
        except OSError:
            ckpts[name] = None
    src = sorted((root / "d3d_b200").rglob("*.py")) + sorted((root / "d3d_b200").rglob("*.cu"))
    return {"python": platform.python_version(), "packages": versions, "cuda_build": torch.version.cuda,
            "gpus": [torch.cuda.get_device_name(i) for i in range(torch.cuda.device_count())],
            "source_commit": commit, "checkpoints": ckpts,
            "source_sha256": {str(p.relative_to(root)): hashlib.sha256(p.read_bytes()).hexdigest() for p in src}}


def resolve_dtype(name: str):
    import torch
    table = {"bf16": torch.bfloat16, "bfloat16": torch.bfloat16, "fp16": torch.float16,
             "float16": torch.float16, "fp32": torch.float32, "float32": torch.float32}
    if name not in table:
        raise ValueError(f"Unsupported dtype {name!r}")
    return table[name]
