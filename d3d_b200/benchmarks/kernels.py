"""Kernel microbenchmarks at the decode shapes of the headline configuration.

    python -m d3d_b200.benchmarks.kernels [--only gemm,attn,forward] [--iters N]
    python -m d3d_b200.benchmarks.kernels --only forward_eager [--drafter] [--layers N]

``forward_eager`` runs one untimed eager forward after one warm-up forward:
the small, few-launch case that profiler captures of single kernels use.

Times each sm_100a kernel with CUDA events on its launching stream after
warm-up, cycling over enough distinct weight copies that the working set is
larger than the 126 MB L2 (so every timed launch streams its weights from
HBM), and prints achieved bandwidth / FLOP rate against the measured peaks in
``MEASURED_PEAKS.json`` when present.
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def load_peaks():
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    except Exception:
        return PEAKS


def timeit(fn, iters=50, warmup=5, graph=True):
    """Mean device time per call in microseconds.  The ``iters`` calls are
    captured in one CUDA graph and replayed, so host launch overhead is not
    part of the number (back-to-back launches, as inside a decode step)."""
    if not graph:
        for _ in range(warmup):
            fn(0)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(iters):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters * 1e3
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        for _ in range(warmup):
            fn(0)
    st.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(iters):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters * 1e3  # us


def bench_gemm(shapes, iters, peaks, rows):
    from d3d_b200 import ops
    E = ops.ext()
    for name, m, n, k in shapes:
        copies = max(2, math.ceil(3 * 126e6 / (n * k * 2)))
        ws = [ops.pack_weight(torch.randn(n, k, device="cuda").to(torch.bfloat16) * 0.02)
              for _ in range(copies)]
        x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
        bt = ops.bt_for(m)
        s = ops.splitk_for(n, k, mtiles=math.ceil(m / bt), bt=bt) if m <= 2048 else 1
        out = torch.empty(s * m * n, device="cuda")
        us = timeit(lambda i: E.gemm_partial(x, ws[i % copies].data, out, s, bt, None, n), iters)
        byts = n * k * 2 + m * k * 2 + s * m * n * 4
        fl = 2 * m * n * k
        rows.append(dict(kernel="gemm_tcgen05", shape=name, M=m, N=n, K=k, splits=s, bt=bt,
                         us=round(us, 2), GBps=round(byts / us / 1e3, 1),
                         hbm_frac=round(byts / us / 1e3 / peaks["hbm_gbs"], 3),
                         TFLOPs=round(fl / us / 1e6, 1),
                         tensor_frac=round(fl / us / 1e6 / peaks["bf16_tflops"], 3)))
        del ws


DRAFTER_SHAPES = (("qkv", 4096, 2048), ("o", 2048, 2048), ("gate_up", 12288, 2048), ("down", 2048, 6144))


def bench_gemm_sweep(m, iters, peaks, rows, shapes=DRAFTER_SHAPES):
    """Every (token tile, split-K) configuration of the drafter's GEMMs at ``m``
    tokens: fp32 partials for every split count, bf16 output for split 1.
    ``partial_MB`` is what the consuming kernel reads back."""
    from d3d_b200 import ops
    E = ops.ext()
    bts = sorted({ops.bt_for(m), 256, 192, 144, 128, 96, 64, 48, 32, 16}, reverse=True)
    for name, n, k in shapes:
        copies = max(2, math.ceil(3 * 126e6 / (n * k * 2)))
        ws = [ops.pack_weight(torch.randn(n, k, device="cuda").to(torch.bfloat16) * 0.02)
              for _ in range(copies)]
        x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
        kb = math.ceil(k / 64)
        out = torch.empty(16 * m * n, device="cuda")
        yb = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        for bt in bts:
            if bt > 256 and bt % 32:
                continue
            if bt > m and bt != ops.bt_for(m):
                continue
            for s in range(1, 17):
                if kb // s < 4:
                    break
                us = timeit(lambda i: E.gemm_partial(x, ws[i % copies].data, out, s, bt, None, n), iters)
                rows.append(dict(kernel="gemm_sweep", shape=name, M=m, N=n, K=k, bt=bt, splits=s, mode="f32",
                                 ctas=math.ceil(n / 128) * math.ceil(m / bt) * s, us=round(us, 2),
                                 partial_MB=round(s * m * n * 4 / 1e6, 2),
                                 TFLOPs=round(2 * m * n * k / us / 1e6, 1)))
            us = timeit(lambda i: E.gemm_bf16(x, ws[i % copies].data, yb, None, bt, None, n), iters)
            rows.append(dict(kernel="gemm_sweep", shape=name, M=m, N=n, K=k, bt=bt, splits=1, mode="bf16",
                             ctas=math.ceil(n / 128) * math.ceil(m / bt), us=round(us, 2), partial_MB=0,
                             TFLOPs=round(2 * m * n * k / us / 1e6, 1)))
        del ws


def bench_lmhead(iters, peaks, rows, only_m=None, bts=None):
    from d3d_b200 import ops
    E = ops.ext()
    for m, n, k, kk in ((1, 151936, 4096, 1), (16, 151936, 4096, 1), (272, 151936, 2048, 2),
                        (752, 151936, 2048, 4)):
        if only_m is not None and m != only_m:
            continue
        w = ops.pack_weight(torch.randn(n, k, device="cuda").to(torch.bfloat16) * 0.02)
        w2 = ops.pack_weight(torch.randn(n, k, device="cuda").to(torch.bfloat16) * 0.02)
        x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
        ws = [w, w2]
        kt = 1 if kk <= 1 else (2 if kk <= 2 else 4)
        nt = math.ceil(n / 128)
        tv = torch.empty(m * nt * kt, device="cuda")
        ti = torch.empty(m * nt * kt, dtype=torch.int32, device="cuda")
        ov = torch.empty(m, kk, device="cuda")
        oi = torch.empty(m, kk, dtype=torch.int64, device="cuda")

        for bt in (bts or [ops.bt_for(m)]):
            def f(i):
                E.gemm_topk(x, ws[i % 2].data, tv, ti, kk, bt, None, n)
                E.topk_merge(tv, ti, m, nt, kt, kk, ov, oi)
            us = timeit(f, iters)
            byts = n * k * 2
            rows.append(dict(kernel="gemm_topk+merge", shape=f"lm_head top{kk}", M=m, N=n, K=k, bt=bt,
                             us=round(us, 2), GBps=round(byts / us / 1e3, 1),
                             hbm_frac=round(byts / us / 1e3 / peaks["hbm_gbs"], 3),
                             TFLOPs=round(2 * m * n * k / us / 1e6, 1)))


def bench_attn(iters, peaks, rows, only=None, graph=True):
    from d3d_b200 import ops
    from d3d_b200.engine.layout import branch_specs, causal_rows, packed_layout
    E = ops.ext()
    for name, hq, hkv, prefix, q, chunk in (("verify 8B", 32, 8, 1000, 16, 64),
                                           ("ar 8B", 32, 8, 1000, 1, 64),
                                           ("verify 8B c128", 32, 8, 1000, 16, 128),
                                           ("verify 8B c256", 32, 8, 1000, 16, 256),
                                           ("ar 8B c256", 32, 8, 1000, 1, 256),
                                           ("packed 1.7B A1", 16, 8, 1000, 272, 256),
                                           ("packed 1.7B A3", 16, 8, 1000, 752, 256)):
        if only and name != only:
            continue
        d = 128
        L = prefix + q
        pages = math.ceil(L / 16)
        kc = torch.randn(pages * 16, hkv, d, device="cuda").to(torch.bfloat16)
        vc = torch.randn_like(kc)
        bt = torch.arange(pages, dtype=torch.int32, device="cuda")[None]
        qq = torch.randn(q, hq, d, device="cuda").to(torch.bfloat16)
        if name.startswith("packed"):
            A = 1 if name.endswith("A1") else 3
            blk = torch.randint(0, 1000, (16,))
            top = torch.stack([blk + j for j in range(A + 1)], 1)
            lay = packed_layout(blk, branch_specs(blk.tolist(), top.tolist(), A), prefix, 16, 999, "causal")
            rows_t = lay.rows.cuda()
        else:
            rows_t = causal_rows(prefix, q).cuda()
        kv_end = torch.tensor([L], dtype=torch.int32, device="cuda")
        nch = math.ceil(L / chunk)
        po = torch.empty(nch * q * hq * d, device="cuda")
        pm = torch.empty(nch * q * hq * 2, device="cuda")
        out = torch.empty_like(qq)
        us = timeit(lambda i: E.attention(qq, kc, vc, bt, rows_t, kv_end, 1, q, hq, hkv, 16,
                                          1 / math.sqrt(d), chunk, nch, po, pm, out), iters, graph=graph)
        byts = 2 * L * hkv * d * 2
        rows.append(dict(kernel="attention", shape=name, M=q, N=L, K=d, us=round(us, 2),
                         GBps=round(byts / us / 1e3, 1)))


def bench_forward(iters, peaks, rows, layers=36, drafter=False):
    """One full forward, graph-replayed: the target (verify M=16, AR M=1) or
    the drafter's packed all-outcome forward (M=272, one anchor)."""
    from d3d_b200 import config as C
    from d3d_b200.engine.layout import branch_specs, causal_rows, packed_layout
    from d3d_b200.models.fast import FastRunner, FastWeights, PagedKV
    cfg = (C.d3d_1p7b() if drafter else C.qwen3_8b()).replace(num_hidden_layers=layers)
    w = FastWeights.random(cfg, seed=0)
    kv = PagedKV(cfg, num_pages=256, page_size=16, max_seqs=1, max_pages_per_seq=128)
    kv.reserve(0, 0, 1900)
    r = FastRunner(w, kv, max_context=1900, batch_invariant=not drafter)
    shapes = (272,) if drafter else (1, 16)
    for m in shapes:
        b = r.buffers(1, m, 2 if drafter else 1)
        if drafter:
            blk = torch.randint(0, 1000, (16,))
            lay = packed_layout(blk, branch_specs(blk.tolist(), torch.stack([blk, blk + 1], 1).tolist(), 1),
                                1000, 16, 151669, "causal")
            b.ids.copy_(lay.input_ids)
            b.pos.copy_(lay.positions)
            b.rows.copy_(lay.rows)
            b.kv_end.fill_(1000 + m)
        else:
            b.pos.copy_(torch.arange(1000, 1000 + m))
            b.rows.copy_(causal_rows(1000, m))
            b.kv_end.fill_(1000 + m)
        b.slots.copy_(torch.arange(1000, 1000 + m))
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            r.forward(b)
        st.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            n = r.forward(b)
        us = timeit(lambda i: g.replay(), iters, graph=False)
        byts = w.nbytes()
        rows.append(dict(kernel="forward (graph)", shape=f"{'drafter' if drafter else 'Qwen3-8B'} M={m}", M=m, launches=n,
                         us=round(us, 1), GBps=round(byts / us / 1e3, 1),
                         hbm_frac=round(byts / us / 1e3 / peaks["hbm_gbs"], 3),
                         plan={g: v for g, v in r.plan(m).items()}))


def forward_eager(layers, drafter, context=1000):
    """One warm-up forward then one eager forward of the target's verify
    (M=16) or the drafter's packed all-outcome forward (M=272); nothing is
    timed.  Launch ``k`` of kernel family ``f`` in the second forward is
    launch ``layers + k`` of ``f`` overall, which is what ``ncu -s`` skips."""
    from d3d_b200 import config as C
    from d3d_b200.engine.layout import branch_specs, causal_rows, packed_layout
    from d3d_b200.models.fast import FastRunner, FastWeights, PagedKV
    cfg = (C.d3d_1p7b() if drafter else C.qwen3_8b()).replace(num_hidden_layers=layers)
    w = FastWeights.random(cfg, seed=0)
    L = context
    pages = (L + 1024) // 16 + 8
    kv = PagedKV(cfg, num_pages=pages, page_size=16, max_seqs=1, max_pages_per_seq=pages)
    kv.reserve(0, 0, L + 900)
    r = FastRunner(w, kv, max_context=L + 900, batch_invariant=not drafter)
    if drafter:
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
    r.forward(b)
    torch.cuda.synchronize()
    n = r.forward(b)
    torch.cuda.synchronize()
    print(json.dumps(dict(kernel="forward (eager, untimed)", drafter=drafter, layers=layers, M=m,
                          launches=n, status=int(b.status.item()))))


def train_kernels(iters, peaks, rows, n_tok=4096, chunk=16384, hidden=2048, n_params=1_720_000_000 // 8):
    """The training step's own kernels at distillation shapes: online-LSE
    KL+CE statistics and gradient over one vocabulary chunk of fp32 logits
    (``n_tok`` rows), the fused AdamW update and the squared-norm reduction
    over the 1.7B drafter's parameter count / 8 ranks (eager launches)."""
    from d3d_b200 import ops
    E = ops.ext()
    g = torch.Generator(device="cuda").manual_seed(0)
    zs = torch.randn(n_tok, chunk, device="cuda", generator=g)
    zt = torch.randn(n_tok, chunk, device="cuda", generator=g)
    tgt = torch.randint(0, chunk, (n_tok,), device="cuda", generator=g)
    st = torch.zeros(n_tok, 8, device="cuda")
    st[:, 0] = st[:, 4] = -math.inf
    us = timeit(lambda i: E.kl_ce_stats(zt, zs, chunk, 0, tgt, st), iters, graph=False)
    byts = 2 * n_tok * chunk * 4
    rows.append(dict(kernel="kl_ce_stats", shape=f"{n_tok}x{chunk}", us=round(us, 2), GBps=round(byts / us / 1e3, 1),
                     hbm_frac=round(byts / us / 1e3 / peaks["hbm_gbs"], 3)))
    lse = torch.randn(n_tok, device="cuda", generator=g)
    w = torch.rand(n_tok, device="cuda", generator=g)
    dz = torch.empty(n_tok, chunk, dtype=torch.bfloat16, device="cuda")
    us = timeit(lambda i: E.kl_ce_grad(zt, zs, chunk, 0, tgt, lse, lse, w, w, dz, None), iters, graph=False)
    byts = 2 * n_tok * chunk * 4 + n_tok * chunk * 2
    rows.append(dict(kernel="kl_ce_grad", shape=f"{n_tok}x{chunk}", us=round(us, 2), GBps=round(byts / us / 1e3, 1),
                     hbm_frac=round(byts / us / 1e3 / peaks["hbm_gbs"], 3)))
    n = int(n_params)
    p = torch.zeros(n, device="cuda")
    gr = torch.randn(n, device="cuda", generator=g)
    m1, v1 = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    us = timeit(lambda i: E.adamw(p, gr, m1, v1, out, 1e-4, 0.9, 0.95, 1e-8, 0.0, i + 1, 1.0), iters, graph=False)
    byts = n * (4 * 4 + 3 * 4 + 2)
    rows.append(dict(kernel="adamw", shape=f"{n} params", us=round(us, 2), GBps=round(byts / us / 1e3, 1),
                     hbm_frac=round(byts / us / 1e3 / peaks["hbm_gbs"], 3)))
    sq = torch.zeros(1, device="cuda")
    us = timeit(lambda i: E.sumsq(gr, sq), iters, graph=False)
    rows.append(dict(kernel="sumsq", shape=f"{n} floats", us=round(us, 2), GBps=round(n * 4 / us / 1e3, 1),
                     hbm_frac=round(n * 4 / us / 1e3 / peaks["hbm_gbs"], 3)))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="gemm,lmhead,attn,forward")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--json", default=None)
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--lm-m", type=int, default=None)
    ap.add_argument("--lm-bt", default=None, help="lmhead: comma-separated token tiles to time")
    ap.add_argument("--drafter", action="store_true", help="forward: drafter packed M=272")
    ap.add_argument("--sweep-m", type=int, default=272, help="gemm_sweep: token count")
    ap.add_argument("--attn-case", default=None, help="attn: run only this shape (e.g. 'packed 1.7B A1')")
    ap.add_argument("--no-graph", action="store_true", help="eager launches (for profiler captures)")
    ap.add_argument("--adamw-n", type=int, default=1_720_000_000 // 8,
                    help="train_kernels: parameters per rank of the AdamW / squared-norm cases")
    a = ap.parse_args()
    peaks = load_peaks()
    rows = []
    only = set(a.only.split(","))
    if "gemm" in only:
        h, i = 4096, 12288
        shapes = []
        for m in (1, 16, 128):
            shapes += [(f"8B qkv m{m}", m, 6144, h), (f"8B o m{m}", m, h, h),
                       (f"8B gate_up m{m}", m, 2 * i, h), (f"8B down m{m}", m, h, i)]
        for m in (272, 1088):
            shapes += [(f"1.7B qkv m{m}", m, 4096, 2048), (f"1.7B o m{m}", m, 2048, 2048),
                       (f"1.7B gate_up m{m}", m, 12288, 2048), (f"1.7B down m{m}", m, 2048, 6144)]
        shapes += [("square 8192", 8192, 8192, 8192)]
        bench_gemm(shapes, a.iters, peaks, rows)
    if "lmhead" in only:
        bench_lmhead(a.iters, peaks, rows, a.lm_m,
                     [int(b) for b in a.lm_bt.split(",")] if a.lm_bt else None)
    if "attn" in only:
        bench_attn(a.iters, peaks, rows, a.attn_case, not a.no_graph)
    if "gemm_sweep" in only:
        bench_gemm_sweep(a.sweep_m, a.iters, peaks, rows)
    if "train_kernels" in only:
        train_kernels(a.iters, peaks, rows, n_params=a.adamw_n)
    if "forward_eager" in only:
        forward_eager(a.layers, a.drafter)
    if "forward" in only:
        bench_forward(a.iters, peaks, rows, layers=a.layers if not a.drafter else min(a.layers, 28),
                      drafter=a.drafter)
    for r in rows:
        print(json.dumps(r))
    if a.json:
        with open(a.json, "w") as f:
            json.dump(dict(peaks=peaks, rows=rows), f, indent=1)


if __name__ == "__main__":
    main()
