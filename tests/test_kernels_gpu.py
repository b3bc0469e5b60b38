"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def E():
    from d3d_b200 import ops
    return ops.ext()


def _bf(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, generator=g, device="cuda") * scale).to(torch.bfloat16)


@pytest.mark.parametrize("m,n,k,splits,bt", [
    (1, 256, 512, 1, 16), (16, 4096, 4096, 3, 16), (100, 1024, 2048, 2, 112),
    (272, 6144, 2048, 1, 144), (16, 384, 128, 1, 16), (300, 640, 1024, 4, 160),
    (1024, 2048, 1024, 1, 256), (272, 1024, 2048, 2, 288), (1000, 512, 1024, 1, 512)])
def test_gemm_partial(E, m, n, k, splits, bt):
    from d3d_b200 import ops
    x = _bf(m, k, seed=1)
    w = _bf(n, k, scale=0.05, seed=2)
    out = torch.full((splits, m, n), float("nan"), device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.gemm_partial(x, w, out, splits, bt, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = ops.linear_ref(x, w)
    got = out.sum(0)
    err = (got - ref).abs().max().item()
    assert err < 2e-3 * max(1.0, ref.abs().max().item()), err


@pytest.mark.parametrize("m,n,k,splits", [(1, 6144, 4096, 3), (16, 300, 200, 1), (272, 1024, 2048, 4)])
def test_gemm_packed_weight(E, m, n, k, splits):
    """The packed-tile weight layout gives bit-identical partials."""
    from d3d_b200 import ops
    x = _bf(m, k, seed=21)
    w = _bf(n, k, scale=0.05, seed=22)
    pw = ops.pack_weight(w)
    assert torch.equal(pw.unpack(), w)
    o1 = torch.empty(splits, m, n, device="cuda")
    o2 = torch.empty(splits, m, n, device="cuda")
    ops.gemm_partial(x, w, o1, splits)
    ops.gemm_partial(x, pw, o2, splits)
    assert torch.equal(o1, o2)
    ov, oi = ops.gemm_topk(x, pw, 2)
    rv, ri = torch.topk(ops.linear_ref(x, w), 2, dim=-1)
    assert torch.allclose(ov, rv, atol=2e-3, rtol=1e-4)


def test_gemm_bf16_residual(E):
    from d3d_b200 import ops
    x, w, r = _bf(40, 1024, seed=3), _bf(512, 1024, scale=0.05, seed=4), _bf(40, 512, seed=5)
    out = torch.empty(40, 512, dtype=torch.bfloat16, device="cuda")
    ops.gemm_bf16(x, w, out, residual=r, bt=48)
    ref = (ops.linear_ref(x, w).to(torch.bfloat16).float() + r.float())
    assert (out.float() - ref).abs().max().item() < 0.05


@pytest.mark.parametrize("k,m", [(1, 33), (2, 33), (4, 33), (2, 300)])
def test_gemm_topk(E, k, m):
    from d3d_b200 import ops
    x, w = _bf(m, 512, seed=6), _bf(151936 // 8, 512, scale=0.05, seed=7)
    ov, oi = ops.gemm_topk(x, w, k)
    ref = ops.linear_ref(x, w)
    rv, ri = torch.topk(ref, k, dim=-1)
    assert torch.allclose(ov, rv, atol=2e-3, rtol=1e-4)
    # indices must agree wherever the reference has no near-tie
    gaps = (rv[:, :-1] - rv[:, 1:]).abs() if k > 1 else torch.ones(m, 0, device="cuda")
    if k == 1:
        assert (oi[:, 0] == ri[:, 0]).float().mean().item() > 0.97
    else:
        clear = torch.cat([gaps > 1e-2, torch.ones(m, 1, dtype=torch.bool, device="cuda")], 1)
        assert ((oi == ri) | ~clear).all()


@pytest.mark.parametrize("k", [1, 2, 4])
def test_gemm_topk_epilogues_agree(E, k):
    """The column-scan epilogue (token tiles above 32) and the warp-max
    epilogue (tiles of up to 32) give bit-identical candidates, exact ties
    included (duplicated weight rows): the lower row wins."""
    from d3d_b200 import ops
    m = 96
    x = _bf(m, 512, seed=16)
    w = _bf(4096, 512, scale=0.05, seed=17)
    w[1::2] = w[0::2]           # every logit appears twice, in rows 2i and 2i+1
    a = ops.gemm_topk(x, w, k, bt=32)
    b = ops.gemm_topk(x, w, k, bt=96)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    if k >= 2:
        assert (b[1][:, 0] % 2 == 0).all() and (b[1][:, 1] == b[1][:, 0] + 1).all()


def test_gemm_batch_invariance(E):
    """A row's partial sums are bit-identical for any M and token tile."""
    from d3d_b200 import ops
    x = _bf(128, 4096, seed=8)
    w = _bf(4096, 4096, scale=0.02, seed=9)
    s = ops.splitk_for(4096, 4096)
    o1 = torch.empty(s, 1, 4096, device="cuda")
    ops.gemm_partial(x[:1], w, o1, s, 16)
    o16 = torch.empty(s, 16, 4096, device="cuda")
    ops.gemm_partial(x[:16], w, o16, s, 16)
    o128 = torch.empty(s, 128, 4096, device="cuda")
    ops.gemm_partial(x, w, o128, s, 128)
    assert torch.equal(o1[:, 0], o16[:, 0])
    assert torch.equal(o16, o128[:, :16])


def test_add_rmsnorm(E):
    m, n, s = 7, 4096, 3
    part = torch.randn(s, m, n, device="cuda")
    res = _bf(m, n, seed=10)
    w = _bf(n, seed=11)
    out = torch.empty_like(res)
    res0 = res.clone()
    E.add_rmsnorm(part, s, res, w, out, 1e-6)
    y = part.sum(0).to(torch.bfloat16).float()
    x = (res0.float() + y).to(torch.bfloat16)
    assert torch.equal(res, x)
    xf = x.float()
    ref = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16).float() * w.float()
    ref = ref.to(torch.bfloat16).float()     # the kernel rounds its output to bf16 as well
    assert ((out.float() - ref).abs() / ref.abs().clamp_min(1e-2)).max().item() < 2e-2


def test_swiglu(E):
    m, i = 5, 3072
    gen = torch.Generator(device="cuda").manual_seed(41)
    part = torch.randn(2, m, 2 * i, device="cuda", generator=gen)
    h = torch.empty(m, i, dtype=torch.bfloat16, device="cuda")
    E.swiglu(part, 2, h)
    p = part.sum(0).to(torch.bfloat16).float()
    g, u = p[:, :i], p[:, i:]
    # same rounding points as the module: bf16(silu(g)) * bf16(u), rounded once more
    ref = (torch.nn.functional.silu(g).to(torch.bfloat16).float() * u).to(torch.bfloat16).float()
    err = (h.float() - ref).abs() / ref.abs().clamp_min(1e-2)
    assert err.max().item() < 2e-2


@pytest.mark.parametrize("m,i,k,bt", [(1, 384, 128, 16), (16, 6144, 2048, 16), (272, 6144, 2048, 96),
                                       (300, 1024, 512, 288)])
def test_gemm_swiglu_epilogue(E, m, i, k, bt):
    """SwiGLU in the GEMM epilogue (interleaved gate|up weight) equals the
    split-1 partial GEMM followed by the interleaved SwiGLU kernel, and tracks
    the fp32 reference silu(x g^T) * (x u^T)."""
    from d3d_b200 import ops
    x = _bf(m, k, seed=31)
    g, u = _bf(i, k, scale=0.05, seed=32), _bf(i, k, scale=0.05, seed=33)
    w = ops.pack_gate_up(g, u)
    h = torch.empty(m, i, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.gemm_swiglu(x, w, h, bt, status)
    part = torch.empty(1, m, 2 * i, device="cuda")
    ops.gemm_partial(x, w, part, 1, bt)
    h2 = torch.empty_like(h)
    E.swiglu(part, 1, h2, True)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(h, h2)
    gf = (x.float() @ g.float().t()).to(torch.bfloat16).float()
    uf = (x.float() @ u.float().t()).to(torch.bfloat16).float()
    ref = torch.nn.functional.silu(gf).to(torch.bfloat16).float() * uf
    assert (h.float() - ref).abs().max().item() < 0.02 * max(1.0, ref.abs().max().item())


def test_swiglu_interleaved_splits(E):
    from d3d_b200 import ops
    m, i, k = 9, 512, 256
    x = _bf(m, k, seed=34)
    g, u = _bf(i, k, scale=0.05, seed=35), _bf(i, k, scale=0.05, seed=36)
    part = torch.empty(3, m, 2 * i, device="cuda")
    ops.gemm_partial(x, ops.pack_gate_up(g, u), part, 3)
    h = torch.empty(m, i, dtype=torch.bfloat16, device="cuda")
    E.swiglu(part, 3, h, True)
    order = ops.gate_up_order(i).cuda()
    plain = torch.empty_like(part)
    plain[:, :, order] = part
    h2 = torch.empty_like(h)
    E.swiglu(plain, 3, h2, False)
    assert torch.equal(h, h2)


@pytest.mark.parametrize("D", [32, 128])
def test_qkv_rope_kv(E, D):
    from d3d_b200.models.qwen3 import rope_cos_sin, rotate_half
    m, hq, hkv = 6, 4, 2
    n = (hq + 2 * hkv) * D
    part = torch.randn(1, m, n, device="cuda")
    qn, kn = _bf(D, seed=12), _bf(D, seed=13)
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    pos = torch.tensor([0, 5, 17, 300, 1023, 4000], device="cuda")
    slots = torch.tensor([3, 9, 0, 12, 7, 1], device="cuda")
    q = torch.empty(m, hq, D, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(16, hkv, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    E.qkv_rope_kv(part, None, 1, qn, kn, inv.cuda(), pos, slots, q, kc, vc, hq, hkv, D, 1e-6)
    y = part[0].to(torch.bfloat16).float().view(m, hq + 2 * hkv, D)

    def norm(t, w):
        t2 = (t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16).float()
        return (t2 * w.float()).to(torch.bfloat16).float()

    cos, sin = rope_cos_sin(pos.cpu(), D, 1e6, torch.float32)
    cos, sin = cos.cuda()[:, None], sin.cuda()[:, None]
    qr = norm(y[:, :hq], qn)
    kr = norm(y[:, hq:hq + hkv], kn)
    qr = qr * cos + rotate_half(qr) * sin
    kr = kr * cos + rotate_half(kr) * sin
    assert (q.float() - qr).abs().max().item() < 0.05
    assert (kc[slots].float() - kr).abs().max().item() < 0.05
    assert torch.equal(vc[slots], y[:, hq + hkv:].to(torch.bfloat16))


def _attn_case(B, Q, Hq, Hkv, D, prefix, page, rows_fn, chunk, seed=0):
    torch.manual_seed(seed)
    L = prefix + Q
    npages_seq = math.ceil(L / page)
    total_pages = B * npages_seq + 3
    perm = torch.randperm(total_pages)[: B * npages_seq].view(B, npages_seq).int().cuda()
    kc = (torch.randn(total_pages * page, Hkv, D, device="cuda")).to(torch.bfloat16)
    vc = (torch.randn(total_pages * page, Hkv, D, device="cuda")).to(torch.bfloat16)
    q = (torch.randn(B * Q, Hq, D, device="cuda")).to(torch.bfloat16)
    rows = torch.stack([rows_fn(b) for b in range(B)]).int().cuda()  # [B, Q, 3]
    kv_end = torch.full((B,), L, dtype=torch.int32, device="cuda")
    return q, kc, vc, perm, rows, kv_end, L


def _attn_ref(q, kc, vc, bt, rows, L, B, Q, Hq, Hkv, D, page):
    from d3d_b200.engine.layout import rows_to_dense
    outs = []
    g = Hq // Hkv
    for b in range(B):
        slots = torch.arange(L, device="cuda")
        phys = bt[b][slots // page].long() * page + slots % page
        k = kc[phys].float().transpose(0, 1).repeat_interleave(g, 0)   # [Hq, L, D]
        v = vc[phys].float().transpose(0, 1).repeat_interleave(g, 0)
        qq = q[b * Q:(b + 1) * Q].float().transpose(0, 1)             # [Hq, Q, D]
        mask = rows_to_dense(rows[b].long(), L)                         # [Q, L]
        s = qq @ k.transpose(1, 2) / math.sqrt(D)
        s = s.masked_fill(~mask[None], float("-inf"))
        p = torch.softmax(s, -1)
        outs.append((p @ v).transpose(0, 1))
    return torch.cat(outs)


@pytest.mark.parametrize("B,Q,Hq,Hkv,D,prefix,page,chunk", [
    (1, 16, 32, 8, 128, 700, 16, 256), (2, 16, 32, 8, 128, 300, 16, 4096),
    (1, 1, 32, 8, 128, 1000, 16, 256), (3, 9, 4, 2, 32, 50, 16, 64), (1, 16, 32, 8, 128, 1000, 16, 64)])
def test_attention_causal(E, B, Q, Hq, Hkv, D, prefix, page, chunk):
    from d3d_b200.engine.layout import causal_rows
    q, kc, vc, bt, rows, kv_end, L = _attn_case(
        B, Q, Hq, Hkv, D, prefix, page, lambda b: causal_rows(prefix, Q), chunk)
    nch = math.ceil(L / chunk)
    out = torch.empty_like(q)
    po = torch.empty(nch, B * Q, Hq, D, device="cuda")
    pml = torch.empty(nch, B * Q, Hq, 2, device="cuda")
    E.attention(q, kc, vc, bt, rows.view(-1, 3), kv_end, B, Q, Hq, Hkv, page, 1 / math.sqrt(D),
                chunk, nch, po, pml, out)
    ref = _attn_ref(q, kc, vc, bt, rows, L, B, Q, Hq, Hkv, D, page)
    assert (out.float() - ref).abs().max().item() < 2e-2


def test_attention_packed_layout(E):
    """Pending block + anchor branches (structured masks) vs the dense oracle."""
    from d3d_b200.engine.layout import branch_specs, packed_layout
    K, A, prefix, D = 16, 3, 200, 128
    blk = torch.randint(0, 1000, (K,))
    top = torch.randint(0, 1000, (K, A + 1))
    specs = branch_specs(blk.tolist(), top.tolist(), A)
    lay = packed_layout(blk, specs, prefix, K, 999, "causal")
    Q = lay.q_len
    q, kc, vc, bt, rows, kv_end, L = _attn_case(1, Q, 16, 8, D, prefix, 16,
                                                lambda b: lay.rows, 256)
    nch = math.ceil(L / 4096)
    out = torch.empty_like(q)
    E.attention(q, kc, vc, bt, rows.view(-1, 3), kv_end, 1, Q, 16, 8, 16, 1 / math.sqrt(D),
                4096, 1, None, None, out)
    ref = _attn_ref(q, kc, vc, bt, rows, L, 1, Q, 16, 8, D, 16)
    assert (out.float() - ref).abs().max().item() < 2e-2


def test_attention_batch_invariance(E):
    """A verify row equals the same row decoded alone (fixed key chunks)."""
    from d3d_b200.engine.layout import causal_rows
    prefix, Q, D = 900, 16, 128
    q, kc, vc, bt, rows, kv_end, L = _attn_case(1, Q, 32, 8, D, prefix, 16,
                                                lambda b: causal_rows(prefix, Q), 256)
    nch = math.ceil(L / 64)
    out = torch.empty_like(q)
    po = torch.empty(nch, Q, 32, D, device="cuda")
    pml = torch.empty(nch, Q, 32, 2, device="cuda")
    E.attention(q, kc, vc, bt, rows.view(-1, 3), kv_end, 1, Q, 32, 8, 16, 1 / math.sqrt(D),
                64, nch, po, pml, out)
    for t in (0, 7, 15):
        end = torch.tensor([prefix + t + 1], dtype=torch.int32, device="cuda")
        o1 = torch.empty(1, 32, D, dtype=torch.bfloat16, device="cuda")
        nc1 = math.ceil((prefix + t + 1) / 64)
        po1 = torch.empty(nch, 1, 32, D, device="cuda")
        pm1 = torch.empty(nch, 1, 32, 2, device="cuda")
        E.attention(q[t:t + 1].contiguous(), kc, vc, bt, rows[0, t:t + 1].contiguous(), end, 1, 1, 32, 8,
                    16, 1 / math.sqrt(D), 64, nc1, po1, pm1, o1)
        assert torch.equal(o1[0], out[t])


def test_greedy_accept_and_topk_merge(E):
    blocks = torch.tensor([[5, 1, 2, 3], [7, 9, 9, 9]], device="cuda")
    post = torch.tensor([[1, 2, 4, 8], [3, 3, 3, 3]], device="cuda")
    commit = torch.empty(2, dtype=torch.int64, device="cuda")
    corr = torch.empty(2, dtype=torch.int64, device="cuda")
    hid = _bf(8, 64, seed=3)
    hout = torch.empty(2, 64, dtype=torch.bfloat16, device="cuda")
    E.greedy_accept(blocks, post, commit, corr, hid, hout)
    assert commit.tolist() == [3, 1] and corr.tolist() == [4, 3]
    assert torch.equal(hout[0], hid[2]) and torch.equal(hout[1], hid[4])


@pytest.mark.parametrize("m,splits", [(1, 9), (16, 9), (40, 3), (16, 1)])
def test_gemm_in_kernel_split_reduce(E, m, splits):
    """The o/down GEMM's in-kernel split-K reduction into the residual equals
    the stand-alone reduce kernel bit for bit (residual and per-tile row sums
    of squares), and tracks the fp32 reference."""
    from d3d_b200 import ops
    n, k = 4096, 4096
    g = torch.Generator(device="cuda").manual_seed(m + splits)
    w = ops.pack_weight((torch.randn(n, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16))
    xin = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    res = torch.randn(m, n, device="cuda", generator=g).to(torch.bfloat16)
    bt = ops.bt_for(m)
    part = torch.zeros(splits * m * n, device="cuda")
    x1, x2 = res.clone(), res.clone()
    ss1 = torch.zeros(32 * m, device="cuda")
    ss2 = torch.zeros(32 * m, device="cuda")
    ticket = torch.zeros(32 * ((m + bt - 1) // bt), dtype=torch.int32, device="cuda")
    for _ in range(2):      # tickets reset themselves between launches
        x1.copy_(res)
        E.gemm_partial_fin(xin, w.data, part, splits, bt, None, w.n, x1, ss1, ticket)
    E.gemm_partial(xin, w.data, part, splits, bt, None, w.n)
    E.residual_split_reduce(part, splits, x2, ss2)
    torch.cuda.synchronize()
    assert torch.equal(x1, x2) and torch.equal(ss1, ss2)
    assert int(ticket.abs().sum()) == 0
    ref = res.float() + xin.float() @ w.unpack().float().t()
    assert (x1.float() - ref).abs().max().item() < 0.1
    ss_ref = (x1.float() ** 2).view(m, 32, 128).sum(-1).t().reshape(-1)
    assert torch.allclose(ss1, ss_ref, rtol=1e-4, atol=1e-3)
