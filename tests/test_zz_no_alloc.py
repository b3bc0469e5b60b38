"""The allocation-free attention entry point, called through its exported C
symbol, must reproduce the allocating entry point on consecutive calls.

Callers that cannot allocate GPU memory (graph capture, plugins of other
runtimes, pre-reserved serving pools) use ``d3d_attention_noalloc``; its
split-KV partials live in a fixed device array inside the library, shared by
every call.  This file is named so pytest collects it last.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

ERR_TOO_LARGE = 1001


@pytest.fixture(scope="module")
def lib():
    from d3d_b200 import ops
    from d3d_b200.ops import build
    ops.ext()                                   # builds / loads the extension
    so = ctypes.CDLL(str(build.so_path()))      # same library, C view
    f = so.d3d_attention_noalloc
    f.restype = ctypes.c_int
    vp, ci = ctypes.c_void_p, ctypes.c_int
    f.argtypes = [vp, vp, vp, vp, ci, vp, vp, ci, ci, ci, ci, ci, ci, ctypes.c_float, ci, ci, vp, vp]
    return f


def _case(B, Q, Hq, Hkv, D, prefix, page, rows_fn, seed):
    g = torch.Generator().manual_seed(seed)
    L = prefix + Q
    npg = math.ceil(L / page)
    total = B * npg + 2
    bt = torch.randperm(total, generator=g)[: B * npg].view(B, npg).int().cuda()
    kc = torch.randn(total * page, Hkv, D, generator=g).to(torch.bfloat16).cuda()
    vc = torch.randn(total * page, Hkv, D, generator=g).to(torch.bfloat16).cuda()
    q = torch.randn(B * Q, Hq, D, generator=g).to(torch.bfloat16).cuda()
    rows = torch.cat([rows_fn(b) for b in range(B)]).int().cuda().contiguous()
    kv_end = torch.full((B,), L, dtype=torch.int32, device="cuda")
    return q, kc, vc, bt, rows, kv_end, L


def _call(f, q, kc, vc, bt, rows, kv_end, B, Q, Hq, Hkv, D, page, chunk, nch, out):
    return f(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), bt.stride(0), rows.data_ptr(),
             kv_end.data_ptr(), B, Q, Hq, Hkv, D, page, 1.0 / math.sqrt(D), chunk, nch, out.data_ptr(),
             torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_allocating_entry_point(lib):
    from d3d_b200 import ops
    from d3d_b200.engine.layout import branch_specs, causal_rows, packed_layout
    E = ops.ext()
    cases = []
    # verify-shaped: GQA 32/8, causal block of 16 over a 900-token prefix, 64-key chunks
    cases.append((2, 16, 32, 8, 128, 900, 16, lambda b: causal_rows(900, 16), 64, 3))
    # drafter packed all-outcome layout, 256-key chunks
    blk = torch.arange(100, 116)
    top = torch.stack([blk, blk + 1], 1)
    lay = packed_layout(blk, branch_specs(blk.tolist(), top.tolist(), 1), 300, 16, 999, "causal")
    cases.append((1, lay.q_len, 16, 8, 128, 300, 16, lambda b: lay.rows, 256, 4))
    # tiny head dim, single chunk (no scratch used)
    cases.append((3, 9, 4, 2, 32, 50, 16, lambda b: causal_rows(50, 9), 4096, 5))
    for (B, Q, Hq, Hkv, D, prefix, page, rows_fn, chunk, seed) in cases:
        q, kc, vc, bt, rows, kv_end, L = _case(B, Q, Hq, Hkv, D, prefix, page, rows_fn, seed)
        nch = math.ceil(L / chunk)
        ref = torch.empty_like(q)
        po = torch.empty(nch * B * Q * Hq * D, device="cuda")
        pm = torch.empty(nch * B * Q * Hq * 2, device="cuda")
        E.attention(q, kc, vc, bt, rows, kv_end, B, Q, Hq, Hkv, page, 1.0 / math.sqrt(D), chunk, nch,
                    po if nch > 1 else None, pm if nch > 1 else None, ref)
        for _ in range(2):      # two calls in a row share (and reuse) the scratch array
            out = torch.full_like(q, float("nan"))
            rc = _call(lib, q, kc, vc, bt, rows, kv_end, B, Q, Hq, Hkv, D, page, chunk, nch, out)
            torch.cuda.synchronize()
            assert rc == 0, rc
            assert torch.allclose(out.float(), ref.float(), atol=2e-2, rtol=0), \
                (out.float() - ref.float()).abs().max().item()


def test_noalloc_rejects_oversized_request(lib):
    from d3d_b200.engine.layout import causal_rows
    B, Q, Hq, Hkv, D, prefix = 1, 256, 32, 8, 128, 16384
    q, kc, vc, bt, rows, kv_end, L = _case(B, Q, Hq, Hkv, D, prefix, 16,
                                           lambda b: causal_rows(prefix, Q), 7)
    out = torch.zeros_like(q)
    nch = math.ceil(L / 64)      # 260 chunks x 256 tokens x 32 heads x 130 floats >> 16 MiB
    rc = _call(lib, q, kc, vc, bt, rows, kv_end, B, Q, Hq, Hkv, D, 16, 64, nch, out)
    torch.cuda.synchronize()
    assert rc == ERR_TOO_LARGE
    assert torch.count_nonzero(out) == 0
