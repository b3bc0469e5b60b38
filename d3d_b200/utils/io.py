"""Atomic JSON output and output-tag sanitising (reference: ``common/io.py``)."""
from __future__ import annotations

import json
import os
import re
from pathlib import Path
from typing import Any, Optional


def safe_tag(path_or_name: str) -> str:
    tag = Path(str(path_or_name)).name or str(path_or_name).strip().replace("/", "_")
    return re.sub(r"[^A-Za-z0-9_.-]+", "_", tag) or "model"


def safe_custom_tag(tag: Optional[str], fallback: str) -> str:
    if tag:
        return re.sub(r"[^A-Za-z0-9_.-]+", "_", str(tag).strip()) or fallback
    return fallback


def write_json(path: Optional[str], payload: Any) -> None:
    """Write ``payload`` to ``path`` atomically (temp file + rename)."""
    if not path:
        return
    out = Path(path)
    out.parent.mkdir(parents=True, exist_ok=True)
    tmp = out.with_name(f".{out.name}.{os.getpid()}.tmp")
    tmp.write_text(json.dumps(payload, ensure_ascii=False, indent=2, default=str))
    os.replace(tmp, out)
