"""Acceptance-controlled drafting (an addition: the reference has no such mode).

Random-init drafters accept almost nothing, so throughput would measure only
the worst case.  In controlled mode the drafter still runs every forward it
would run, but each proposed block is replaced, after the forward, by the
target's own greedy continuation (precomputed by an AR pass) corrupted at a
seeded per-position rate.  The same injection is applied to the reference
framework in ``bench.py --impl reference`` so both frameworks see identical
acceptance.

Rules (all functions of the absolute sequence position ``p`` only, so every
block or branch that covers ``p`` sees the same decision):

* ``keep(p)`` = ``hash(seed, stream, p) >= rate``; the draft token at ``p`` is
  the oracle token if kept, else ``corrupt(oracle[p])`` (never equal to it).
* The draft's top-(A+1) list at ``p`` is ``[draft, alt_1, ...]`` where
  ``alt_1`` is the oracle token when the draft was corrupted (so an anchor
  branch can be reused) and other alternatives are further corruptions.

With per-position keep probability ``1-r`` and block size K the expected
commit length per verify is ``1 + sum_{i=1}^{K-1} (1-r)^i``;
:func:`rate_for_mean_accept` inverts it.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence

import torch

_M = (1 << 61) - 1


def splitmix64(x: int) -> int:
    """splitmix64's output function, written out from its published definition."""
    x = (x + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
    return x ^ (x >> 31)


_mix = splitmix64


def uniform(seed: int, stream: int, pos: int) -> float:
    return (_mix(_mix(_mix(seed) ^ stream) ^ pos) >> 11) / float(1 << 53)


def expected_commit(rate: float, block_size: int) -> float:
    keep = 1.0 - rate
    return 1.0 + sum(keep ** i for i in range(1, block_size))


def rate_for_mean_accept(mean: float, block_size: int) -> float:
    """Corruption rate whose expected commit length equals ``mean``."""
    if mean >= block_size:
        return 0.0
    if mean <= 1.0:
        return 1.0
    lo, hi = 0.0, 1.0
    for _ in range(80):
        mid = 0.5 * (lo + hi)
        if expected_commit(mid, block_size) > mean:
            lo = mid
        else:
            hi = mid
    return 0.5 * (lo + hi)


@dataclass
class ControlledAcceptance:
    """Per-request oracle + corruption schedule."""
    oracle: Sequence[int]           # full token sequence: prompt + target greedy continuation
    rate: float
    vocab_size: int
    seed: int = 0
    stream: int = 0                 # request index
    exclude: Sequence[int] = ()     # tokens never produced by corruption (e.g. MASK, EOS)

    def __post_init__(self):
        # draft_at and the alternatives row are pure functions of the position
        # (and, for the anchor row, of the anchor token): memoised, since the
        # same positions are rewritten by every branch that covers them
        self._draft_cache = {}
        self._row_cache = {}

    def keep(self, pos: int) -> bool:
        return uniform(self.seed, self.stream, pos) >= self.rate

    def _corrupt(self, tok: int, pos: int, salt: int) -> int:
        v = self.vocab_size
        bad = set(int(t) for t in self.exclude) | {int(tok)}
        h = _mix(_mix(self.seed ^ 0x5BD1E995) ^ (self.stream * 1315423911) ^ (pos << 8) ^ salt)
        c = int(h % v)
        while c in bad:
            c = (c + 1) % v
        return c

    def oracle_at(self, pos: int) -> Optional[int]:
        return int(self.oracle[pos]) if 0 <= pos < len(self.oracle) else None

    def draft_at(self, pos: int) -> int:
        v = self._draft_cache.get(pos)
        if v is None:
            o = self.oracle_at(pos)
            if o is None:
                v = self._corrupt(0, pos, 7)
            else:
                v = o if self.keep(pos) else self._corrupt(o, pos, 1)
            self._draft_cache[pos] = v
        return v

    def _alts(self, pos: int, first: int, anchor_row: bool, w: int):
        key = (pos, first, anchor_row, w)
        row = self._row_cache.get(key)
        if row is None:
            o = self.oracle_at(pos)
            alts = []
            if not anchor_row and o is not None and o != first:
                alts.append(o)
            salt = 11
            while len(alts) < w - 1:
                c = self._corrupt(first, pos, salt)
                salt += 1
                if c not in alts and (o is None or c != o or anchor_row):
                    alts.append(c)
            row = [first] + alts[: w - 1]
            self._row_cache[key] = row
        return row

    def override(self, block: torch.Tensor, top: Optional[torch.Tensor], anchor_pos: int):
        """Rewrite drafts 1..K-1 of ``block`` (anchor at ``anchor_pos``) and its
        top-token table in place."""
        k = int(block.shape[0])
        vals = [self.draft_at(anchor_pos + i) for i in range(1, k)]
        block[1:] = torch.tensor(vals, dtype=block.dtype, device=block.device)
        if top is not None:
            w = int(top.shape[-1])
            first0 = int(block[0])
            rows = [self._alts(anchor_pos, first0, True, w)]
            rows += [self._alts(anchor_pos + i, vals[i - 1], False, w) for i in range(1, k)]
            top.copy_(torch.tensor(rows, dtype=top.dtype, device=top.device))
        return block, top
