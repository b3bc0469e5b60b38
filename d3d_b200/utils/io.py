"""Result files: crash-safe JSON writes and file-name-safe labels.

A run's JSON summary is written next to its final name with
``tempfile.mkstemp`` in the same directory, flushed and fsync'ed, then moved
over the final name with ``os.replace`` -- a reader sees either the previous
file or the complete new one, never a torn write (the reference gets the same
guarantee from ``common/io.py:22-29``).  Labels derived from model paths are
reduced to ``[A-Za-z0-9_.-]`` so they can be embedded in file names.
"""
from __future__ import annotations

import json
import os
import tempfile
from pathlib import Path
from typing import Any, Optional

_KEEP = frozenset("abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789_.-")


def label(text: Optional[str], default: str = "run") -> str:
    """File-name-safe label: the last path component of ``text`` with every
    run of disallowed characters collapsed to one ``_``."""
    s = str(text or "").rstrip("/").split("/")[-1].strip()
    out, prev_bad = [], False
    for ch in s:
        if ch in _KEEP:
            out.append(ch)
            prev_bad = False
        elif not prev_bad:
            out.append("_")
            prev_bad = True
    res = "".join(out).strip("_")
    return res or default


def write_json(path: Optional[str], payload: Any) -> Optional[Path]:
    """Atomically replace ``path`` with ``payload`` as indented JSON.  ``None``
    or an empty path is a no-op (the CLIs' output flags are optional)."""
    if not path:
        return None
    dst = Path(path)
    dst.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(dir=dst.parent, prefix=dst.name, suffix=".partial")
    try:
        with os.fdopen(fd, "w", encoding="utf-8") as f:
            json.dump(payload, f, indent=2, ensure_ascii=False, default=str)
            f.write("\n")
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, dst)
    except BaseException:
        if os.path.exists(tmp):
            os.unlink(tmp)
        raise
    return dst
