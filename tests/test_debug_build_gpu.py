"""The debug build (device bounds checks on step-input indices) computes
exactly what the normal build computes on valid inputs and raises no
bounds error -- the checks cost nothing in results and do not fire falsely."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_debug_build_matches_normal_build():
    from d3d_b200 import ops
    from d3d_b200.ops import build
    from d3d_b200.engine.layout import causal_rows
    E, D = ops.ext(), build.load_debug()
    g = torch.Generator(device="cuda").manual_seed(7)
    hq, hkv, d, L, q = 8, 2, 128, 300, 16
    pages = math.ceil(L / 16) + 1
    kc = torch.randn(pages * 16, hkv, d, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(pages * 16, hkv, d, device="cuda", generator=g).to(torch.bfloat16)
    bt = torch.randperm(pages, device="cuda").to(torch.int32)[None].contiguous()
    qq = torch.randn(q, hq, d, device="cuda", generator=g).to(torch.bfloat16)
    rows = causal_rows(L - q, q).cuda()
    kv_end = torch.tensor([L], dtype=torch.int32, device="cuda")
    table = torch.randn(1000, 256, device="cuda", generator=g).to(torch.bfloat16)
    ids = torch.randint(0, 1000, (12,), device="cuda", generator=g)
    outs = []
    for mod in (E, D):
        st = torch.zeros(1, dtype=torch.int32, device="cuda")
        out = torch.empty_like(qq)
        # batch-invariant path (cluster kernel): no split-KV partial buffers
        mod.attention(qq, kc, vc, bt, rows, kv_end, 1, q, hq, hkv, 16, 1 / math.sqrt(d), 64, 1, None, None,
                      out, True, st)
        emb = torch.empty(12, 256, dtype=torch.bfloat16, device="cuda")
        mod.embed(ids, table, None, None, 12, emb, st)
        torch.cuda.synchronize()
        outs.append((out.clone(), emb.clone(), int(st.item())))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert outs[0][2] == 0 and outs[1][2] == 0
