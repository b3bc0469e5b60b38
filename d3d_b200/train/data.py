"""Training data: a byte-offset index over a JSONL file, rank-strided rows,
chat-template prompt/response splitting, and a background prefetcher that
packs the next step's blocks on the host while the GPU runs the current one.

The reference reads the same kind of file through an offset-indexed
``Dataset`` in DataLoader workers (``train/dataset.py:71-113,157-231,
277-313``).  Here the index is built in one vectorised pass over a
memory-mapped file (newline positions via numpy), rows are parsed only when
a step asks for them, and packing runs on one host thread ahead of the
device; nothing reads the whole file into Python objects.

Accepted row formats (one JSON object per line):

* ``{"prompt_ids": [...], "response_ids": [...]}`` -- already tokenized;
* ``{"messages" | "conversations": [{"role"|"from", "content"|"value"}, ...]}``
  -- rendered with the tokenizer's chat template (thinking off unless asked)
  and split at the last assistant turn (its tokens are supervised);
* ``{"prompt": str, "response": str}`` -- plain text, encoded without
  special tokens.

Rows with ``status`` other than ``success``, without a prompt, with fewer
than two response tokens, or longer than the prompt / sequence limits are
skipped (and counted), as the reference skips them.
"""
from __future__ import annotations

import json
import queue
import random
import threading
from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional, Sequence

import numpy as np

from .blocks import Example

_ROLE = {"human": "user", "user": "user", "gpt": "assistant", "assistant": "assistant", "system": "system"}


class JsonlIndex:
    """Byte ranges of the non-blank lines of a JSONL file that belong to
    ``rank`` (global row ``i`` goes to rank ``i % world``), capped at
    ``max_rows`` global rows (0 = all)."""

    def __init__(self, path: str, rank: int = 0, world: int = 1, max_rows: int = 0):
        self.path = str(path)
        buf = np.memmap(self.path, dtype=np.uint8, mode="r")
        n = buf.shape[0]
        ends = np.flatnonzero(buf == 0x0A)
        if n and (len(ends) == 0 or ends[-1] != n - 1):
            ends = np.append(ends, n)                      # last line without a newline
        starts = np.concatenate([[0], ends[:-1] + 1]) if len(ends) else np.zeros(0, np.int64)
        # blank lines: nothing but whitespace between start and end
        keep = ends > starts
        if keep.any():
            lens = (ends - starts)[keep]
            small = lens <= 4
            if small.any():     # lines of <= 4 bytes are checked for content explicitly
                idx = np.flatnonzero(keep)[small]
                for i in idx:
                    if not bytes(buf[starts[i]:ends[i]]).strip():
                        keep[i] = False
        starts, ends = starts[keep].astype(np.int64), ends[keep].astype(np.int64)
        if max_rows:
            starts, ends = starts[:max_rows], ends[:max_rows]
        self.total_rows = len(starts)
        self.rows = np.arange(rank, self.total_rows, max(1, world), dtype=np.int64)
        self.starts, self.ends = starts[self.rows], ends[self.rows]
        self._buf = buf

    def __len__(self) -> int:
        return len(self.rows)

    def raw(self, i: int) -> bytes:
        return bytes(self._buf[self.starts[i]:self.ends[i]])

    def row(self, i: int) -> Dict[str, Any]:
        return json.loads(self.raw(i))

    def global_row(self, i: int) -> int:
        return int(self.rows[i])


def normalize_messages(msgs: Sequence[Dict[str, Any]]) -> List[Dict[str, str]]:
    out = []
    for m in msgs:
        role = _ROLE.get(str(m.get("role", m.get("from", ""))), str(m.get("role", m.get("from", ""))))
        out.append({"role": role, "content": str(m.get("content", m.get("value", "")) or "")})
    return out


@dataclass
class RowLimits:
    max_prompt_len: int = 4096
    max_seq_len: int = 8192
    thinking: bool = False


def encode_row(row: Dict[str, Any], tokenizer=None, limits: RowLimits = RowLimits()) -> Optional[Example]:
    """One JSONL row -> ``Example`` (prompt ids, response ids), or ``None``
    when the row is to be skipped."""
    if row.get("status") not in (None, "success"):
        return None
    if "prompt_ids" in row:
        prompt, resp = [int(t) for t in row["prompt_ids"]], [int(t) for t in row["response_ids"]]
    elif "messages" in row or "conversations" in row:
        if tokenizer is None:
            raise ValueError("chat rows need --tokenizer")
        from ..utils.text import split_chat
        msgs = normalize_messages(row.get("messages") or row.get("conversations") or [])
        last = max((i for i, m in enumerate(msgs) if m["role"] == "assistant"), default=None)
        if last is None or last == 0:
            return None
        prompt, resp = split_chat(tokenizer, msgs[: last + 1])
    elif "prompt" in row:
        if tokenizer is None:
            raise ValueError("text rows need --tokenizer")
        prompt = list(tokenizer.encode(row["prompt"], add_special_tokens=False))
        resp = list(tokenizer.encode(row.get("response", ""), add_special_tokens=False))
    else:
        return None
    if not prompt or len(resp) < 2:
        return None
    if len(prompt) > limits.max_prompt_len or len(prompt) + len(resp) > limits.max_seq_len:
        return None
    return Example(prompt, resp)


class IndexedExamples:
    """Rank-local examples of a JSONL file, parsed on demand.  ``take(cursor,
    n)`` returns the next ``n`` valid examples at or after local position
    ``cursor`` (wrapping around) and the cursor after them; skipped rows are
    counted in ``skipped``."""

    def __init__(self, path: str, rank: int, world: int, tokenizer=None, limits: RowLimits = RowLimits(),
                 max_rows: int = 0):
        self.index = JsonlIndex(path, rank, world, max_rows)
        if len(self.index) == 0:
            raise ValueError(f"{path}: no rows for rank {rank} of {world}")
        self.tokenizer, self.limits = tokenizer, limits
        self.skipped = 0

    def __len__(self) -> int:
        return len(self.index)

    def take(self, cursor: int, n: int):
        out, tries, N = [], 0, len(self.index)
        while len(out) < n and tries < N:
            ex = encode_row(self.index.row(cursor % N), self.tokenizer, self.limits)
            cursor += 1
            tries += 1
            if ex is None:
                self.skipped += 1
            else:
                out.append(ex)
        return out, cursor


class Prefetcher:
    """Runs ``make(step)`` for steps ``start..stop-1`` on one host thread,
    ``depth`` steps ahead of the consumer, so tokenization and block packing
    overlap the device work of the current step.  Exceptions in the producer
    are re-raised in the consumer."""

    _END = object()

    def __init__(self, make: Callable[[int], Any], start: int, stop: int, depth: int = 2):
        self.q: "queue.Queue" = queue.Queue(maxsize=max(1, depth))
        self._stop = threading.Event()

        def run():
            try:
                for s in range(start, stop):
                    if self._stop.is_set():
                        return
                    self.q.put((s, make(s)))
                self.q.put((None, self._END))
            except BaseException as e:  # surfaced by get()
                self.q.put((None, e))

        self.t = threading.Thread(target=run, daemon=True, name="d3d-prefetch")
        self.t.start()

    def get(self):
        s, item = self.q.get()
        if item is self._END:
            raise StopIteration
        if isinstance(item, BaseException):
            raise item
        return s, item

    def close(self):
        self._stop.set()
        try:
            while True:
                self.q.get_nowait()
        except queue.Empty:
            pass


def worker_rng(seed: int, rank: int, step: int) -> random.Random:
    """Per-(rank, step) anchor RNG: the packing of a step does not depend on
    how far ahead the prefetcher ran."""
    return random.Random((seed * 1_000_003 + rank) * 1_000_033 + step)
