"""The allocation-free attention entry point, called through its exported C
symbol, must reproduce the allocating entry point on consecutive calls.

Some callers of this library cannot allocate GPU memory while they run: code
being recorded into a CUDA graph, plugins of other runtimes whose hooks must
live within memory the host framework already owns, and serving loops that
reserved the device for their own pool.  They call ``d3d_attention_noalloc``,
whose split-KV partials live in a fixed device array inside the library,
shared by every call.  This file is named so pytest collects it last.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

ERR_TOO_LARGE = 1001
ERR_BAD_ARG = 1002


def _bind(so):
    f = so.d3d_attention_noalloc
    f.restype = ctypes.c_int
    vp, ci = ctypes.c_void_p, ctypes.c_int
    f.argtypes = [vp, vp, vp, ctypes.c_longlong, vp, ci, vp, vp, ci, ci, ci, ci, ci, ci, ctypes.c_float, ci, ci,
                  vp, vp]
    return f


@pytest.fixture(scope="module")
def lib():
    from d3d_b200 import ops
    from d3d_b200.ops import build
    ops.ext()                                   # builds / loads the extension
    return _bind(ctypes.CDLL(str(build.so_path())))   # same library, C view


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
    return f(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.size(0), bt.data_ptr(), bt.stride(0), rows.data_ptr(),
             kv_end.data_ptr(), B, Q, Hq, Hkv, D, page, 1.0 / math.sqrt(D), chunk, nch, out.data_ptr(),
             torch.cuda.current_stream().cuda_stream)


def _oracle(q, kc, vc, bt, rows, L, B, Q, Hq, Hkv, D, page):
    """fp32 PyTorch attention with the dense form of the structured rows."""
    from d3d_b200.engine.layout import rows_to_dense
    g, outs = Hq // Hkv, []
    for b in range(B):
        slots = torch.arange(L, device="cuda")
        phys = bt[b][slots // page].long() * page + slots % page
        k = kc[phys].float().transpose(0, 1).repeat_interleave(g, 0)
        v = vc[phys].float().transpose(0, 1).repeat_interleave(g, 0)
        qq = q[b * Q:(b + 1) * Q].float().transpose(0, 1)
        mask = rows_to_dense(rows[b * Q:(b + 1) * Q].long().cpu(), L).cuda()
        s = (qq @ k.transpose(1, 2) / math.sqrt(D)).masked_fill(~mask[None], float("-inf"))
        outs.append((torch.softmax(s, -1) @ v).transpose(0, 1))
    return torch.cat(outs)


def _cases():
    from d3d_b200.engine.layout import branch_specs, causal_rows, packed_layout
    blk = torch.arange(100, 116)
    lay = packed_layout(blk, branch_specs(blk.tolist(), torch.stack([blk, blk + 1], 1).tolist(), 1), 300, 16, 999,
                        "causal")
    return [
        # verify-shaped: GQA 32/8, causal block of 16 over a 900-token prefix, 64-key chunks
        (2, 16, 32, 8, 128, 900, 16, lambda b: causal_rows(900, 16), 64, 3),
        # drafter packed all-outcome layout, 256-key chunks
        (1, lay.q_len, 16, 8, 128, 300, 16, lambda b: lay.rows, 256, 4),
        # tiny head dim, single chunk (no scratch used)
        (3, 9, 4, 2, 32, 50, 16, lambda b: causal_rows(50, 9), 4096, 5),
    ]


def test_noalloc_matches_allocating_entry_point(lib):
    """Bit-identical to the allocating split-KV path (same kernels, partials in
    the library's array instead of caller buffers), on two calls in a row,
    and within the kernel tests' tolerance of the fp32 oracle."""
    from d3d_b200 import ops
    E = ops.ext()
    for (B, Q, Hq, Hkv, D, prefix, page, rows_fn, chunk, seed) in _cases():
        q, kc, vc, bt, rows, kv_end, L = _case(B, Q, Hq, Hkv, D, prefix, page, rows_fn, seed)
        nch = math.ceil(L / chunk)
        ref = torch.empty_like(q)
        po = torch.empty(nch * B * Q * Hq * D, device="cuda")
        pm = torch.empty(nch * B * Q * Hq * 2, device="cuda")
        E.attention(q, kc, vc, bt, rows, kv_end, B, Q, Hq, Hkv, page, 1.0 / math.sqrt(D), chunk, nch,
                    po if nch > 1 else None, pm if nch > 1 else None, ref, force_split=True)
        oracle = _oracle(q, kc, vc, bt, rows, L, B, Q, Hq, Hkv, D, page)
        for _ in range(2):      # two calls in a row share (and reuse) the scratch array
            out = torch.full_like(q, float("nan"))
            rc = _call(lib, q, kc, vc, bt, rows, kv_end, B, Q, Hq, Hkv, D, page, chunk, nch, out)
            torch.cuda.synchronize()
            assert rc == 0, rc
            assert torch.equal(out, ref)
            assert (out.float() - oracle).abs().max().item() < 2e-2


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


def test_noalloc_rejects_bad_shapes(lib):
    """Too many chunks for the combine kernel (even when the partials would
    fit), pages that do not tile a 64-key tile, and chunks that split a page
    are refused before anything is launched."""
    from d3d_b200.engine.layout import causal_rows
    B, Q, Hq, Hkv, D, prefix = 1, 1, 2, 1, 32, 600
    q, kc, vc, bt, rows, kv_end, L = _case(B, Q, Hq, Hkv, D, prefix, 16, lambda b: causal_rows(prefix, Q), 9)
    out = torch.zeros_like(q)
    assert _call(lib, q, kc, vc, bt, rows, kv_end, B, Q, Hq, Hkv, D, 16, 64, 513, out) == ERR_BAD_ARG
    assert _call(lib, q, kc, vc, bt, rows, kv_end, B, Q, Hq, Hkv, D, 48, 192, 4, out) == ERR_BAD_ARG
    assert _call(lib, q, kc, vc, bt, rows, kv_end, B, Q, Hq, Hkv, D, 16, 96, 7, out) == ERR_BAD_ARG
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0
    # 512 chunks is the limit and is accepted
    assert _call(lib, q, kc, vc, bt, rows, kv_end, B, Q, Hq, Hkv, D, 16, 64, 512, out) == 0
    torch.cuda.synchronize()


def test_noalloc_debug_build_matches(lib):
    """The bounds-checked debug library's copy of the entry point (it knows
    the KV slot count from its argument) computes the same result."""
    from d3d_b200.ops import build
    build.load_debug()
    dbg = _bind(ctypes.CDLL(str(build.HERE / "_build_debug" / "d3d_b200_C_debug.so")))
    B, Q, Hq, Hkv, D, prefix, page, rows_fn, chunk, seed = _cases()[0]
    q, kc, vc, bt, rows, kv_end, L = _case(B, Q, Hq, Hkv, D, prefix, page, rows_fn, seed)
    nch = math.ceil(L / chunk)
    outs = []
    for f in (lib, dbg):
        out = torch.full_like(q, float("nan"))
        assert _call(f, q, kc, vc, bt, rows, kv_end, B, Q, Hq, Hkv, D, page, chunk, nch, out) == 0
        torch.cuda.synchronize()
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
