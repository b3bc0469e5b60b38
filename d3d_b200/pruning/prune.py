"""Physical layer deletion (reference: ``pruning/prune.py:74-178``).

Rewrites a checkpoint without one decoder layer: tensors
``model.layers.N.*`` are renamed to their new compact index, the config's
``num_hidden_layers`` is decremented, and ``layer_prune.json`` records the
provenance (original teacher and depth, parent, removed layer, original
indices of retained layers; the reference's ``layer_prune.json`` fields, so
checkpoints pruned by either implementation feed the other's later stages).
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


# files of a parent that describe the parent itself, not the child
_NOT_COPIED = {"config.json", "model.safetensors.index.json", "layer_prune.json", "recovery_info.json",
               "layer_schedule.json", "checkpoint_validation.json"}


def prune_checkpoint(parent: str | Path, output: str | Path, removed: int,
                     retained_original: Optional[Sequence[int]] = None, *, block_size: int = 16,
                     mask_token_id: Optional[int] = None, selection_file: Optional[str] = None) -> Path:
    """Write ``parent`` without compact layer ``removed`` to ``output`` and
    record the provenance the later stages read: the original teacher and
    depth, the parent and child depths, the removed layer in parent and
    original numbering, the retained layers in both numberings, the block
    size and the parameter count."""
    from .common import provenance
    parent, output = Path(parent).resolve(), Path(output).resolve()
    if output.exists():
        raise FileExistsError(f"Refusing to overwrite {output}")
    cfg = ModelConfig.from_pretrained(parent, mask_token_id=mask_token_id)
    depth = cfg.num_hidden_layers
    if not 0 <= removed < depth:
        raise ValueError(f"removed layer {removed} outside [0, {depth})")
    teacher, original_depth, parent_orig = provenance(parent)
    keep = [i for i in range(depth) if i != removed]
    old_to_new = {old: new for new, old in enumerate(keep)}
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
            if (f.is_file() and f.name not in _NOT_COPIED and f.suffix != ".safetensors"
                    and not f.name.startswith(("compact_model_", "progressive_checkpoint_", "recovery_checkpoint_"))):
                shutil.copy2(f, tmp / f.name)
        child = cfg.replace(num_hidden_layers=depth - 1)
        if "max_window_layers" in child.extra:
            child.extra["max_window_layers"] = min(int(child.extra["max_window_layers"]), depth - 1)
        child.save(tmp)
        (tmp / "layer_prune.json").write_text(json.dumps({
            "format_version": 1, "method": "progressive_single_layer_pruning",
            "parent_checkpoint": str(parent), "teacher_checkpoint": str(teacher), "original_depth": original_depth,
            "parent_depth": depth, "child_depth": depth - 1, "removed_parent_layer": removed,
            "removed_original_layer": parent_orig[removed], "retained_parent_layers": keep,
            "retained_original_layers": retained_original, "block_size": int(block_size),
            "selection_file": selection_file, "parameters": int(sum(v.numel() for v in new_state.values()))},
            indent=2, sort_keys=True))
        os.replace(tmp, output)
    except BaseException:
        shutil.rmtree(tmp, ignore_errors=True)
        raise
    return output


def prune_from_selection(selection: str | Path, output: str | Path) -> Path:
    """Carry out a ``selection.json`` (``pruning/prune.py:114-178``)."""
    selection = Path(selection).resolve()
    sel = json.loads(selection.read_text())
    parent = Path(sel["parent_checkpoint"])
    depth = int(sel["parent_depth"])
    removed = int(sel["removed_compact_layer"])
    if ModelConfig.from_pretrained(parent).num_hidden_layers != depth:
        raise ValueError("The selected parent no longer has the recorded depth")
    if int(sel.get("child_depth", depth - 1)) != depth - 1 or not 0 <= removed < depth:
        raise ValueError("selection.json does not describe one valid layer removal")
    return prune_checkpoint(parent, output, removed, sel.get("child_retained_original_layers"),
                            block_size=int(sel.get("block_size", 16)), mask_token_id=sel.get("mask_token_id"),
                            selection_file=str(selection))


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
