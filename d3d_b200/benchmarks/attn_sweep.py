"""Attention latency against context length, query count, key chunk and
path (graph-timed).

    python -m d3d_b200.benchmarks.attn_sweep

Part 1: the target's decode shapes (32 query heads, 8 kv heads, head_dim
128) on the default path -- separates the fixed cost of a launch from the
per-key-tile cost.  Part 2: the target verify block and the drafter's packed
all-outcome forward at several key-chunk sizes on the split-KV path (the
chunk is a free choice for the drafter; for the target any fixed chunk keeps
verify and AR bit-identical).
"""
from __future__ import annotations

import json
import math

import torch


def _case(E, timeit, hq, hkv, L, q, rows, chunk, invariant):
    d = 128
    pages = math.ceil(L / 16) + 1
    kc = torch.randn(pages * 16, hkv, d, device="cuda").to(torch.bfloat16)
    vc = torch.randn_like(kc)
    bt = torch.arange(pages, dtype=torch.int32, device="cuda")[None]
    qq = torch.randn(q, hq, d, device="cuda").to(torch.bfloat16)
    kv_end = torch.tensor([L], dtype=torch.int32, device="cuda")
    nch = math.ceil(L / chunk)
    po = torch.empty(nch * q * hq * d, device="cuda")
    pm = torch.empty(nch * q * hq * 2, device="cuda")
    out = torch.empty_like(qq)
    return timeit(lambda i: E.attention(qq, kc, vc, bt, rows, kv_end, 1, q, hq, hkv, 16, 1 / math.sqrt(d),
                                        chunk, nch, po, pm, out, invariant), 50)


def main():
    from d3d_b200 import ops
    from d3d_b200.benchmarks.kernels import timeit
    from d3d_b200.engine.layout import branch_specs, causal_rows, packed_layout
    E = ops.ext()
    for L in (64, 256, 1016, 4096):
        for q in (1, 16):
            rows = causal_rows(L - q, q).cuda()
            us = _case(E, timeit, 32, 8, L, q, rows, 64, True)
            print(json.dumps(dict(part="target", path="default", L=L, q=q, us=round(us, 2))))
    rows = causal_rows(1000, 16).cuda()
    for chunk in (64, 128, 256, 512):
        us = _case(E, timeit, 32, 8, 1016, 16, rows, chunk, False)
        print(json.dumps(dict(part="target verify split", L=1016, q=16, chunk=chunk, us=round(us, 2))))
    blk = torch.randint(0, 1000, (16,))
    lay = packed_layout(blk, branch_specs(blk.tolist(), torch.stack([blk, blk + 1], 1).tolist(), 1), 1000, 16,
                        999, "causal")
    rows = lay.rows.cuda()
    for chunk in (64, 128, 256, 512, 1024):
        us = _case(E, timeit, 16, 8, 1000 + lay.q_len, lay.q_len, rows, chunk, False)
        print(json.dumps(dict(part="drafter packed split", L=1000 + lay.q_len, q=lay.q_len, chunk=chunk,
                              us=round(us, 2))))
    us = _case(E, timeit, 16, 8, 1000 + lay.q_len, lay.q_len, rows, 64, True)
    print(json.dumps(dict(part="drafter packed cluster", L=1000 + lay.q_len, q=lay.q_len, us=round(us, 2))))


if __name__ == "__main__":
    main()
