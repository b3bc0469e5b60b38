"""One eager forward of the target's verify (M=16) or the drafter's packed
all-outcome forward (M=272), after one warm-up forward -- for kernel launch
lists under a profiler.

    python -m d3d_b200.benchmarks.forward_once [--drafter] [--layers N]
"""
from __future__ import annotations

import argparse

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--drafter", action="store_true")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--context", type=int, default=1000)
    a = ap.parse_args()
    from d3d_b200 import config as C
    from d3d_b200.engine.layout import branch_specs, causal_rows, packed_layout
    from d3d_b200.models.fast import FastRunner, FastWeights, PagedKV
    cfg = C.d3d_1p7b() if a.drafter else C.qwen3_8b()
    if a.layers:
        cfg = cfg.replace(num_hidden_layers=a.layers)
    w = FastWeights.random(cfg, seed=0)
    L = a.context
    kv = PagedKV(cfg, num_pages=(L + 1024) // 16 + 8, page_size=16, max_seqs=1, max_pages_per_seq=(L + 1024) // 16 + 8)
    kv.reserve(0, 0, L + 900)
    r = FastRunner(w, kv, max_context=L + 900, batch_invariant=not a.drafter)
    if a.drafter:
        blk = torch.randint(0, 1000, (16,))
        lay = packed_layout(blk, branch_specs(blk.tolist(), torch.stack([blk, blk + 1], 1).tolist(), 1),
                            L, 16, 151669, "causal")
        b = r.buffers(1, lay.q_len, 2)
        b.ids.copy_(lay.input_ids)
        b.pos.copy_(lay.positions)
        b.rows.copy_(lay.rows)
        m = lay.q_len
    else:
        m = 16
        b = r.buffers(1, m, 1)
        b.pos.copy_(torch.arange(L, L + m))
        b.rows.copy_(causal_rows(L, m))
    b.kv_end.fill_(L + m)
    b.slots.copy_(torch.arange(L, L + m))
    n = r.forward(b)
    torch.cuda.synchronize()
    with torch.cuda.nvtx.range("fwd"):      # profile with --nvtx --nvtx-include "fwd/"
        n = r.forward(b)
        torch.cuda.synchronize()
    print(f"launches per forward: {n}; status {int(b.status.item())}")


if __name__ == "__main__":
    main()
