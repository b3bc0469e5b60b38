"""Physical layer deletion (reference: ``pruning/prune.py:74-178``).

Rewrites a checkpoint without one decoder layer: tensors
``model.layers.N.*`` are renamed to their new compact index, the config's
``num_hidden_layers`` is decremented, and ``layer_prune.json`` records the
provenance (parent, removed layer, original indices of retained layers).
The output is built in a temporary directory and renamed into place; an
existing output is never overwritten.
"""
from __future__ import annotations

import json
import os
import re
import shutil
import tempfile
from pathlib import Path
from typing import Dict, Optional, Sequence

import torch

from ..checkpoint import read_state, write_state
from ..config import ModelConfig

_LAYER = re.compile(r"^model\.layers\.(\d+)\.(.+)$")


def renamed_key(name: str, old_to_new: Dict[int, int]) -> Optional[str]:
    m = _LAYER.match(name)
    if m is None:
        return name
    old = int(m.group(1))
    if old not in old_to_new:
        return None
    return f"model.layers.{old_to_new[old]}.{m.group(2)}"


def prune_checkpoint(parent: str | Path, output: str | Path, removed: int,
                     retained_original: Optional[Sequence[int]] = None) -> Path:
    parent, output = Path(parent), Path(output)
    if output.exists():
        raise FileExistsError(f"Refusing to overwrite {output}")
    cfg = ModelConfig.from_pretrained(parent)
    depth = cfg.num_hidden_layers
    if not 0 <= removed < depth:
        raise ValueError(f"removed layer {removed} outside [0, {depth})")
    keep = [i for i in range(depth) if i != removed]
    old_to_new = {old: new for new, old in enumerate(keep)}
    prov_path = parent / "layer_prune.json"
    parent_orig = (json.loads(prov_path.read_text())["retained_original_layers"]
                   if prov_path.exists() else list(range(depth)))
    retained_original = list(retained_original) if retained_original is not None else \
        [parent_orig[i] for i in keep]
    if len(retained_original) != depth - 1:
        raise ValueError("retained original-layer mapping has the wrong length")
    output.parent.mkdir(parents=True, exist_ok=True)
    tmp = Path(tempfile.mkdtemp(prefix=f".{output.name}.building.", dir=output.parent))
    try:
        state = read_state(parent)
        new_state = {}
        for k, v in state.items():
            nk = renamed_key(k, old_to_new)
            if nk is not None:
                new_state[nk] = v
        write_state(new_state, tmp)
        for f in parent.iterdir():
            if f.suffix in (".json", ".txt", ".model", ".py") and f.name not in (
                    "config.json", "model.safetensors.index.json", "layer_prune.json"):
                shutil.copy2(f, tmp / f.name)
        cfg.replace(num_hidden_layers=depth - 1).save(tmp)
        (tmp / "layer_prune.json").write_text(json.dumps({
            "parent_checkpoint": str(parent), "parent_depth": depth, "child_depth": depth - 1,
            "removed_compact_layer": removed, "removed_original_layer": parent_orig[removed],
            "retained_original_layers": retained_original}, indent=2))
        os.replace(tmp, output)
    except BaseException:
        shutil.rmtree(tmp, ignore_errors=True)
        raise
    return output


def prune_from_selection(selection: str | Path, output: str | Path) -> Path:
    sel = json.loads(Path(selection).read_text())
    parent = Path(sel["parent_checkpoint"])
    if ModelConfig.from_pretrained(parent).num_hidden_layers != int(sel["parent_depth"]):
        raise ValueError("The selected parent no longer has the recorded depth")
    return prune_checkpoint(parent, output, int(sel["removed_compact_layer"]),
                            sel.get("child_retained_original_layers"))


def drop_layers_inplace(model, compact_indices: Sequence[int]) -> None:
    """Delete decoder layers from an in-memory module (indices are compact)."""
    drop = set(int(i) for i in compact_indices)
    kept = [l for i, l in enumerate(model.model.layers) if i not in drop]
    model.model.layers = torch.nn.ModuleList(kept)
    for i, l in enumerate(kept):
        l.self_attn.layer_idx = i
    model.cfg = model.cfg.replace(num_hidden_layers=len(kept))
    for l in kept:
        l.self_attn.cfg = model.cfg
