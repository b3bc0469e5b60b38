"""Time one tensor-parallel target forward (graph-replayed) per rank.

    python -m torch.distributed.run --nproc-per-node T -m d3d_b200.benchmarks.tp_forward \\
        [--target qwen3-32b] [--context 1000]

Every rank captures the same forward (decode M=1 and verify M=16 over a
``--context``-token KV cache) and replays it; the printed time is the max
over ranks of the mean replay time.  With T=1 it is the unsharded forward.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--target", default="qwen3-32b")
    ap.add_argument("--context", type=int, default=1000)
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args()
    from d3d_b200 import config as C
    from d3d_b200.engine.layout import causal_rows
    from d3d_b200.models.fast import FastRunner, FastWeights, PagedKV
    from d3d_b200.parallel.tp import TPGroup, random_shard
    from d3d_b200.utils.benchutil import dist_max, dist_setup
    rank, world, local = dist_setup()
    dev = torch.device("cuda", local)
    cfg = C.PRESETS[a.target]()
    T = world
    grp = TPGroup(rank, T, dev, num_layers=cfg.num_hidden_layers) if T > 1 else None
    w = random_shard(cfg, T, rank, device=dev) if T > 1 else FastWeights.random(cfg, device=dev)
    L = a.context
    npg = (L + 64) // 16 + 8
    kv = PagedKV(w.cfg, num_pages=npg, page_size=16, max_seqs=1, max_pages_per_seq=npg, device=dev)
    kv.reserve(0, 0, L + 32)
    r = FastRunner(w, kv, max_context=L + 32, batch_invariant=True, device=dev, tp=grp)
    st = torch.cuda.Stream(device=dev)
    out = {"target": a.target, "tp": T, "context": L}
    for m in (1, 16):
        b = r.buffers(1, m, 1)
        b.pos.copy_(torch.arange(L, L + m))
        b.rows.copy_(causal_rows(L, m))
        b.kv_end.fill_(L + m)
        b.slots.copy_(torch.arange(L, L + m))
        with torch.cuda.stream(st):
            r.forward(b)
        st.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            n = r.forward(b)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        if dist.is_initialized():
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.iters):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = dist_max(e0.elapsed_time(e1) / a.iters * 1e3)
        out[f"forward_M{m}_us"] = round(us, 1)
        out[f"launches_M{m}"] = n
    if grp is not None:
        torch.cuda.synchronize()
        out["exchange_status"] = int(grp.status.item())
        del g
        grp.close()
    if rank == 0:
        print(json.dumps(out), flush=True)
    if dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
