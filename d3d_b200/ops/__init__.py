"""sm_100a kernels of d3d_b200 and their Python entry points.

``ext()`` returns the compiled extension (``d3d_b200/ops/_build/d3d_b200_C.so``).
On a machine with a CUDA device the extension is mandatory: a missing or
broken build raises instead of silently falling back to PyTorch.

Split-K policy (:func:`splitk_for`) depends only on the weight shape, never on
the number of tokens, so every output element is reduced in the same order
whether a token is decoded alone or verified inside a block.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import build as _build

_EXT = None


def ext():
    global _EXT
    if _EXT is None:
        try:
            _EXT = _build.load()
        except Exception as e:  # pragma: no cover - exercised only when the build is broken
            raise RuntimeError(f"d3d_b200 CUDA extension unavailable: {e}") from e
    return _EXT


def available() -> bool:
    if not torch.cuda.is_available():
        return False
    ext()
    return True


# ----------------------------------------------------------------- policies
NUM_SMS = 148


def splitk_for(n: int, k: int, sms: int = NUM_SMS) -> int:
    """Split-K factor from the weight shape alone (batch invariance)."""
    tiles = math.ceil(n / 128)
    kb = math.ceil(k / 64)
    if tiles >= sms:
        return 1
    best, best_eff = 1, 0.0
    for s in range(1, min(16, kb) + 1):
        ctas = tiles * s
        waves = math.ceil(ctas / sms)
        eff = ctas / (waves * sms)
        # prefer fewer splits when efficiency is within 5%
        if eff > best_eff + 0.05:
            best, best_eff = s, eff
    return best


def bt_for(m: int) -> int:
    """Token tile (MMA N) for m tokens: one tile up to 256, padded to 16."""
    if m <= 256:
        return max(16, ((m + 15) // 16) * 16)
    tiles = math.ceil(m / 256)
    per = math.ceil(m / tiles)
    return ((per + 15) // 16) * 16


# ------------------------------------------------------------ thin wrappers
def gemm_partial(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, splits: int,
                 bt: Optional[int] = None, status: Optional[torch.Tensor] = None) -> torch.Tensor:
    ext().gemm_partial(x, w, out, int(splits), int(bt or bt_for(x.shape[0])), status)
    return out


def gemm_bf16(x, w, out, residual=None, bt=None, status=None):
    ext().gemm_bf16(x, w, out, residual, int(bt or bt_for(x.shape[0])), status)
    return out


def gemm_topk(x, w, k: int, bt=None, status=None, bufs=None):
    """Top-k (value, index) of ``x @ w.T`` per row without storing logits."""
    m, n = x.shape[0], w.shape[0]
    kt = 1 if k <= 1 else (2 if k <= 2 else 4)
    ntiles = math.ceil(n / 128)
    if bufs is None:
        tv = torch.empty(m * ntiles * kt, dtype=torch.float32, device=x.device)
        ti = torch.empty(m * ntiles * kt, dtype=torch.int32, device=x.device)
        ov = torch.empty(m, k, dtype=torch.float32, device=x.device)
        oi = torch.empty(m, k, dtype=torch.int64, device=x.device)
    else:
        tv, ti, ov, oi = bufs
    e = ext()
    e.gemm_topk(x, w, tv, ti, int(k), int(bt or bt_for(m)), status)
    e.topk_merge(tv, ti, m, ntiles, kt, int(k), ov, oi)
    return ov, oi


def linear_ref(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """fp32 reference of the GEMM."""
    return x.float() @ w.float().t()
