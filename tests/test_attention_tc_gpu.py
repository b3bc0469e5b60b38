"""The tcgen05/TMEM attention kernel (``attention_tc.cu``) against an fp32
PyTorch oracle of the same masked attention, for every shape family the
framework runs: target verify and AR decode (GQA 4), prefill, the drafter's
packed all-outcome forward (GQA 2, structured branch rows), block-causal
drafter prefill, 256-key pages, head_dim 64 and GQA 8 -- plus bit-exact batch
invariance (a verify row equals the same row decoded alone)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def E():
    from d3d_b200 import ops
    return ops.ext()


def _case(B, Q, Hq, Hkv, D, prefix, page, rows_fn, seed):
    g = torch.Generator().manual_seed(seed)
    L = prefix + Q
    npg = math.ceil(L / page)
    total = B * npg + 3
    bt = torch.randperm(total, generator=g)[: B * npg].view(B, npg).int().cuda()
    kc = torch.randn(total * page, Hkv, D, generator=g).to(torch.bfloat16).cuda()
    vc = torch.randn(total * page, Hkv, D, generator=g).to(torch.bfloat16).cuda()
    q = torch.randn(B * Q, Hq, D, generator=g).to(torch.bfloat16).cuda()
    rows = torch.cat([rows_fn(b) for b in range(B)]).int().cuda().contiguous()
    kv_end = torch.full((B,), L, dtype=torch.int32, device="cuda")
    return q, kc, vc, bt, rows, kv_end, L


def _oracle(q, kc, vc, bt, rows, L, B, Q, Hq, Hkv, D, page):
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
        p = torch.softmax(s, -1).nan_to_num(0.0)
        outs.append((p @ v).transpose(0, 1))
    return torch.cat(outs)


def _run(E, q, kc, vc, bt, rows, kv_end, B, Q, Hq, Hkv, D, page, chunk, L):
    nch = max(1, math.ceil(L / chunk))
    assert E.attention_uses_tc(Hq, Hkv, D, page, chunk, nch)
    out = torch.full_like(q, float("nan"))
    po = torch.empty(nch * B * Q * Hq * D, device="cuda")
    pm = torch.empty(nch * B * Q * Hq * 2, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    E.attention(q, kc, vc, bt, rows, kv_end, B, Q, Hq, Hkv, page, 1.0 / math.sqrt(D), chunk, nch,
                po if nch > 1 else None, pm if nch > 1 else None, out, True, st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    return out


def _packed_rows(prefix, A, seed):
    from d3d_b200.engine.layout import branch_specs, packed_layout
    g = torch.Generator().manual_seed(seed)
    blk = torch.randint(0, 1000, (16,), generator=g)
    top = torch.randint(0, 1000, (16, A + 1), generator=g)
    lay = packed_layout(blk, branch_specs(blk.tolist(), top.tolist(), A), prefix, 16, 999, "causal")
    return lay.q_len, lay.rows


def _cases():
    from d3d_b200.engine.layout import block_causal_rows, causal_rows
    out = [
        # name, B, Q, Hq, Hkv, D, prefix, page, rows_fn, chunk
        ("verify", 2, 16, 32, 8, 128, 900, 16, lambda b: causal_rows(900, 16), 256),
        ("verify-64", 1, 16, 32, 8, 128, 1000, 16, lambda b: causal_rows(1000, 16), 64),
        ("ar", 3, 1, 32, 8, 128, 700, 16, lambda b: causal_rows(700, 1), 128),
        ("prefill", 1, 300, 32, 8, 128, 0, 16, lambda b: causal_rows(0, 300), 320),
        ("page256", 1, 16, 32, 8, 128, 600, 256, lambda b: causal_rows(600, 16), 256),
        ("d64-gqa8", 2, 16, 64, 8, 64, 333, 16, lambda b: causal_rows(333, 16), 128),
        ("block-causal", 1, 48, 16, 8, 128, 64, 16, lambda b: block_causal_rows(64, 48, 16), 128),
    ]
    for A in (1, 3):
        q_len, rows = _packed_rows(500, A, 11 + A)
        out.append((f"packed-A{A}", 1, q_len, 16, 8, 128, 500, 16, (lambda r: lambda b: r)(rows), 256))
    return out


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c[0])
def test_attention_tc_matches_oracle(E, case):
    name, B, Q, Hq, Hkv, D, prefix, page, rows_fn, chunk = case
    q, kc, vc, bt, rows, kv_end, L = _case(B, Q, Hq, Hkv, D, prefix, page, rows_fn, seed=sum(map(ord, name)))
    out = _run(E, q, kc, vc, bt, rows, kv_end, B, Q, Hq, Hkv, D, page, chunk, L)
    ref = _oracle(q, kc, vc, bt, rows, L, B, Q, Hq, Hkv, D, page)
    assert torch.isfinite(out.float()).all()
    err = (out.float() - ref).abs().max().item()
    assert err < 2e-2, (name, err)


@pytest.mark.parametrize("chunk", [64, 256])
def test_attention_tc_batch_invariance(E, chunk):
    """A verify row equals the same row decoded alone, bit for bit."""
    from d3d_b200.engine.layout import causal_rows
    prefix, Q, D = 900, 16, 128
    q, kc, vc, bt, rows, kv_end, L = _case(1, Q, 32, 8, D, prefix, 16, lambda b: causal_rows(prefix, Q), 5)
    out = _run(E, q, kc, vc, bt, rows, kv_end, 1, Q, 32, 8, D, 16, chunk, L)
    for t in (0, 7, 15):
        end = torch.tensor([prefix + t + 1], dtype=torch.int32, device="cuda")
        o1 = _run(E, q[t:t + 1].contiguous(), kc, vc, bt, rows[t:t + 1].contiguous(), end, 1, 1, 32, 8, D, 16,
                  chunk, prefix + t + 1)
        assert torch.equal(o1[0], out[t])


def test_attention_tc_close_to_mma_sync_path(E):
    """The tensor-core kernel and the mma.sync split-KV kernel agree to bf16
    rounding on the drafter's packed layout."""
    Q, prow = _packed_rows(700, 3, 3)
    q, kc, vc, bt, rows, kv_end, L = _case(1, Q, 16, 8, 128, 700, 16, lambda b: prow, 9)
    tc = _run(E, q, kc, vc, bt, rows, kv_end, 1, Q, 16, 8, 128, 16, 256, L)
    nch = math.ceil(L / 256)
    ref = torch.empty_like(q)
    po = torch.empty(nch * Q * 16 * 128, device="cuda")
    pm = torch.empty(nch * Q * 16 * 2, device="cuda")
    E.attention(q, kc, vc, bt, rows, kv_end, 1, Q, 16, 8, 16, 1 / math.sqrt(128), 256, nch, po, pm, ref,
                force_split=True)
    torch.cuda.synchronize()
    assert (tc.float() - ref.float()).abs().max().item() < 2e-2
