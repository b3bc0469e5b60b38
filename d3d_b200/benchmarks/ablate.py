"""Where a captured forward spends its time, measured inside the graph.

    python -m d3d_b200.benchmarks.ablate [--drafter] [--iters 20]

Kernel-level profilers serialise launches and hide programmatic dependent
launch overlap, so they overstate small kernels.  Here the forward is
captured in a CUDA graph once as is and once per kernel family with that
family's launches replaced by no-ops; the difference in replay time is what
the family costs in the real schedule.  (Outputs of ablated forwards are
meaningless; only the timing is used.)
"""
from __future__ import annotations

import argparse
import json

import torch

FAMILIES = {
    "gemm": ("gemm_partial", "gemm_bf16", "gemm_swiglu", "gemm_partial_fin"),
    "lm_head": ("gemm_topk", "topk_merge"),
    "attention": ("attention",),
    "add_rmsnorm": ("add_rmsnorm", "tile_sumsq"),
    "qkv_rope_kv": ("qkv_rope_kv",),
    "swiglu": ("swiglu", "swiglu_rowscale"),
}


class _Proxy:
    def __init__(self, ext, skip):
        self._ext, self._skip = ext, set(skip)

    def __getattr__(self, name):
        if name in self._skip:
            return lambda *a, **k: None
        return getattr(self._ext, name)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--drafter", action="store_true")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--context", type=int, default=1000)
    a = ap.parse_args()
    from d3d_b200 import config as C, ops
    from d3d_b200.engine.layout import branch_specs, causal_rows, packed_layout
    from d3d_b200.models.fast import FastRunner, FastWeights, PagedKV
    cfg = C.d3d_1p7b() if a.drafter else C.qwen3_8b()
    w = FastWeights.random(cfg, seed=0)
    L = a.context
    npg = (L + 1024) // 16 + 8
    kv = PagedKV(cfg, num_pages=npg, page_size=16, max_seqs=1, max_pages_per_seq=npg)
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
    real_ext = ops.ext()
    st = torch.cuda.Stream()

    def graph_time(skip):
        ops._EXT_OVERRIDE = _Proxy(real_ext, skip) if skip else None
        try:
            with torch.cuda.stream(st):
                r.forward(b)
            st.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                r.forward(b)
        finally:
            ops._EXT_OVERRIDE = None
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.iters):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / a.iters * 1e3

    full = graph_time(())
    out = {"model": "drafter M=%d" % m if a.drafter else "target M=16", "forward_us": round(full, 1)}
    for fam, names in FAMILIES.items():
        out[fam + "_us"] = round(full - graph_time(names), 1)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
