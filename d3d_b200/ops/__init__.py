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
_EXT_OVERRIDE = None   # instrumentation hook (benchmarks.ablate): stands in for the extension


def ext():
    global _EXT
    if _EXT_OVERRIDE is not None:
        return _EXT_OVERRIDE
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


def ctas_per_sm(bt: int) -> int:
    """Co-resident GEMM CTAs per SM for token tile ``bt`` (mirrors the kernel's
    shared-memory policy: 2 when >= 4 pipeline stages fit in ~110 KB)."""
    stage = 128 * 64 * 2 + bt * 64 * 2
    return 2 if (110 * 1024) // stage >= 4 else 1


def splitk_for(n: int, k: int, sms: int = NUM_SMS, mtiles: int = 1, bt: int = 16, m: int = 0) -> int:
    """Split-K factor that fills whole waves of CTA slots (SMs x co-resident
    CTAs).  For the target it is called with ``mtiles=1, bt=16`` whatever the
    token count, so it depends on the weight shape alone (batch invariance).
    With ``m`` tokens given, the fp32 partials (splits * m * n * 4 bytes) are
    kept no larger than the bf16 weight (n * k * 2 bytes)."""
    sms = sms * ctas_per_sm(bt)
    tiles = math.ceil(n / 128) * mtiles
    kb = math.ceil(k / 64)
    cap = max(1, k // (2 * m)) if m > 0 else 16
    best, best_eff = 1, 0.0
    for s in range(1, min(16, kb, cap) + 1):
        if kb // s < 4:          # keep at least 4 K blocks (256) per CTA
            break
        ctas = tiles * s
        waves = math.ceil(ctas / sms)
        eff = ctas / (waves * sms)
        # prefer fewer splits when efficiency is within 5%
        if eff > best_eff + 0.05:
            best, best_eff = s, eff
    return best


def bt_for(m: int) -> int:
    """Token tile for m tokens: up to 256 in one MMA (multiple of 16), up to
    512 as two MMAs (multiple of 32), so each weight tile is read once for
    up to 512 tokens."""
    if m <= 256:
        return max(16, ((m + 15) // 16) * 16)
    if m <= 512:
        return ((m + 31) // 32) * 32
    tiles = math.ceil(m / 512)
    per = math.ceil(m / tiles)
    return ((per + 31) // 32) * 32


class PackedWeight:
    """A [N, K] bf16 weight stored as contiguous 128 x 64 tiles
    (``[ceil(N/128)][ceil(K/64)][128][64]``, zero padded).  Each GEMM pipeline
    stage then reads one contiguous 16 KB block from HBM instead of 128 rows
    of 128 bytes that are K*2 bytes apart."""

    def __init__(self, data: torch.Tensor, n: int, k: int):
        self.data, self.n, self.k = data, int(n), int(k)

    @property
    def shape(self):
        return (self.n, self.k)

    def numel(self) -> int:
        return self.n * self.k

    def unpack(self) -> torch.Tensor:
        nt, kt = math.ceil(self.n / 128), math.ceil(self.k / 64)
        w = self.data.view(nt, kt, 128, 64).permute(0, 2, 1, 3).reshape(nt * 128, kt * 64)
        return w[: self.n, : self.k]


def pack_weight(w: torch.Tensor) -> PackedWeight:
    n, k = w.shape
    nt, kt = math.ceil(n / 128), math.ceil(k / 64)
    pad = torch.zeros(nt * 128, kt * 64, dtype=torch.bfloat16, device=w.device)
    pad[:n, :k] = w
    data = pad.view(nt, 128, kt, 64).permute(0, 2, 1, 3).contiguous().view(nt * kt * 128, 64)
    return PackedWeight(data, n, k)


def gate_up_order(i: int) -> torch.Tensor:
    """Row order of the interleaved gate|up weight: row ``32w + j`` of tile t
    is gate row ``64t + 16w + j`` (j < 16) or up row ``I + 64t + 16w + j - 16``,
    so the SwiGLU epilogue pairs lanes j and j + 16 of one warp."""
    if i % 64:
        raise ValueError("interleaved gate|up needs intermediate_size % 64 == 0")
    r = torch.arange(2 * i)
    t, w, j = r // 128, (r % 128) // 32, r % 32
    base = 64 * t + 16 * w
    return torch.where(j < 16, base + j, i + base + j - 16)


def pack_gate_up(gate: torch.Tensor, up: torch.Tensor) -> PackedWeight:
    """Pack ``[gate; up]`` ([2I, K]) in the interleaved row order."""
    w = torch.cat([gate, up], 0)
    return pack_weight(w[gate_up_order(gate.shape[0]).to(w.device)])


def _w(w):
    return (w.data, w.n) if isinstance(w, PackedWeight) else (w, 0)


# ------------------------------------------------------------ thin wrappers
def gemm_partial(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, splits: int,
                 bt: Optional[int] = None, status: Optional[torch.Tensor] = None) -> torch.Tensor:
    wd, wn = _w(w)
    ext().gemm_partial(x, wd, out, int(splits), int(bt or bt_for(x.shape[0])), status, wn)
    return out


def gemm_bf16(x, w, out, residual=None, bt=None, status=None):
    wd, wn = _w(w)
    ext().gemm_bf16(x, wd, out, residual, int(bt or bt_for(x.shape[0])), status, wn)
    return out


def gemm_swiglu(x, w: PackedWeight, out, bt=None, status=None):
    """``out = silu(x @ gate.T) * (x @ up.T)`` for an interleaved gate|up
    weight (:func:`pack_gate_up`), in the GEMM epilogue."""
    ext().gemm_swiglu(x, w.data, out, int(bt or bt_for(x.shape[0])), status, w.n)
    return out


def gemm_topk(x, w, k: int, bt=None, status=None, bufs=None):
    """Top-k (value, index) of ``x @ w.T`` per row without storing logits."""
    m, n = x.shape[0], w.shape[0]
    wd, wn = _w(w)
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
    e.gemm_topk(x, wd, tv, ti, int(k), int(bt or bt_for(m)), status, wn)
    e.topk_merge(tv, ti, m, ntiles, kt, int(k), ov, oi)
    return ov, oi


def linear_ref(x: torch.Tensor, w) -> torch.Tensor:
    """fp32 reference of the GEMM."""
    if isinstance(w, PackedWeight):
        w = w.unpack()
    return x.float() @ w.float().t()
