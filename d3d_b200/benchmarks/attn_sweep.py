"""Attention latency against context length and query count (graph-timed).

    python -m d3d_b200.benchmarks.attn_sweep

Separates the fixed cost of one attention launch from the per-key-tile cost
for the target's decode shapes (32 query heads, 8 kv heads, head_dim 128).
"""
from __future__ import annotations

import json
import math

import torch


def main():
    from d3d_b200 import ops
    from d3d_b200.benchmarks.kernels import timeit
    from d3d_b200.engine.layout import causal_rows
    E = ops.ext()
    hq, hkv, d = 32, 8, 128
    for L in (64, 256, 1016, 4096):
        for q in (1, 16):
            prefix = L - q
            pages = math.ceil(L / 16) + 1
            kc = torch.randn(pages * 16, hkv, d, device="cuda").to(torch.bfloat16)
            vc = torch.randn_like(kc)
            bt = torch.arange(pages, dtype=torch.int32, device="cuda")[None]
            qq = torch.randn(q, hq, d, device="cuda").to(torch.bfloat16)
            rows = causal_rows(prefix, q).cuda()
            kv_end = torch.tensor([L], dtype=torch.int32, device="cuda")
            nch = math.ceil(L / 64)
            po = torch.empty(nch * q * hq * d, device="cuda")
            pm = torch.empty(nch * q * hq * 2, device="cuda")
            out = torch.empty_like(qq)
            us = timeit(lambda i: E.attention(qq, kc, vc, bt, rows, kv_end, 1, q, hq, hkv, 16, 1 / math.sqrt(d),
                                              64, nch, po, pm, out), 50)
            print(json.dumps(dict(L=L, q=q, us=round(us, 2))))


if __name__ == "__main__":
    main()
