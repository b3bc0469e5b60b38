"""Training kernels on the GPU vs PyTorch fp32 references: the fused LM-head
KL+CE loss (tcgen05 chunk logits + kl_ce_stats/kl_ce_grad), fused AdamW and
a bf16 trainer step."""
import pytest
import torch

from d3d_b200.train.losses import ce_per_token, forward_kl_per_token, lmhead_distill_loss

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N,V,Hs,Ht,chunk", [(37, 5000, 256, 512, 2048), (200, 151936 // 4, 2048, 4096, 16384)])
def test_fused_lmhead_loss_kernel(N, V, Hs, Ht, chunk):
    torch.manual_seed(0)
    dev = "cuda"
    hs = (torch.randn(N, Hs, device=dev)).to(torch.bfloat16).requires_grad_(True)
    ws = (torch.randn(V, Hs, device=dev) * 0.02).to(torch.bfloat16).requires_grad_(True)
    ht = torch.randn(N, Ht, device=dev).to(torch.bfloat16)
    wt = (torch.randn(V, Ht, device=dev) * 0.02).to(torch.bfloat16)
    tgt = torch.randint(0, V, (N,), device=dev)
    wk = torch.rand(N, device=dev)
    wc = torch.rand(N, device=dev)
    loss, kl, ce = lmhead_distill_loss(hs, ws, ht, wt, tgt, wk, wc, chunk=chunk)
    loss.backward()
    hs32 = hs.detach().float().requires_grad_(True)
    ws32 = ws.detach().float().requires_grad_(True)
    zs = hs32 @ ws32.t()
    zt = ht.float() @ wt.float().t()
    ref = (wk * forward_kl_per_token(zs, zt)).sum() + (wc * ce_per_token(zs, tgt)).sum()
    ref.backward()
    assert abs(loss.item() - ref.item()) < 2e-3 * max(1.0, abs(ref.item()))
    gh_err = (hs.grad.float() - hs32.grad).abs().max().item() / hs32.grad.abs().max().item()
    gw_err = (ws.grad.float() - ws32.grad).abs().max().item() / ws32.grad.abs().max().item()
    assert gh_err < 2e-2 and gw_err < 2e-2, (gh_err, gw_err)


def test_adamw_kernel_matches_torch():
    from d3d_b200 import ops
    torch.manual_seed(1)
    n = 100003
    p = torch.randn(n, device="cuda")
    ref = p.clone().requires_grad_(True)
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    opt = torch.optim.AdamW([ref], lr=1e-3, weight_decay=0.01, eps=1e-8)
    for step in range(1, 4):
        g = torch.randn(n, device="cuda")
        ops.ext().adamw(p, g * 2.0, m, v, out, 1e-3, 0.9, 0.999, 1e-8, 0.01, step, 0.5)
        ref.grad = g.clone()
        opt.step()
    assert torch.allclose(p, ref.detach(), atol=1e-6, rtol=1e-5)
    assert torch.equal(out, p.to(torch.bfloat16))
    sq = torch.zeros(1, device="cuda")
    ops.ext().sumsq(p, sq)
    assert abs(sq.item() - (p.double() ** 2).sum().item()) < 1e-3 * sq.item()


def test_trainer_step_bf16_gpu(tmp_path):
    from d3d_b200.train.args import parser
    from d3d_b200.train.trainer import train
    a = parser().parse_args(["--draft-model", "tiny-drafter", "--target-model", "tiny-target",
                             "--output-dir", str(tmp_path), "--seq-len", "256", "--batch-size", "2",
                             "--parallel-anchors-per-example", "8", "--max-steps", "3", "--block-size", "8",
                             "--vocab-chunk", "512", "--device", "cuda", "--objective", "kl_ce",
                             "--warmup-steps", "0", "--lr", "1e-4"])
    r = train(a)
    losses = [x["loss"] for x in r["log"]]
    assert all(torch.isfinite(torch.tensor(l)) for l in losses)


def test_fast_teacher_matches_module():
    """The teacher forward on the inference kernels (batched, causal, every
    position) tracks the PyTorch module's final-norm hidden states."""
    import torch
    from d3d_b200.config import tiny_target, qwen3_8b
    from d3d_b200.models.qwen3 import build_model
    from d3d_b200.train.model_utils import FastTeacher
    dev = torch.device("cuda")
    for cfg in (tiny_target(), qwen3_8b().replace(num_hidden_layers=2, vocab_size=4096)):
        m = build_model(cfg, seed=4, dtype=torch.bfloat16, device=dev).eval()
        ft = FastTeacher(m, max_batch=3, max_len=300, device=dev)
        ids = torch.randint(0, cfg.vocab_size - 2, (3, 300), device=dev)
        with torch.no_grad():
            ref = m(ids).float()
        out = ft(ids).float()
        rel = (out - ref).norm() / ref.norm()
        assert out.shape == ref.shape and rel < 3e-2, rel
        assert torch.equal(ft(ids[:, :200]), ft(ids[:, :200]))   # padded shapes reuse buffers


def test_tc_linear_forward_backward_matches_fp32():
    """The tcgen05 linear of the training model: output and both gradients
    against an fp32 PyTorch reference of the same bf16 inputs."""
    import torch
    from d3d_b200.models.qwen3 import Linear
    torch.manual_seed(0)
    for (m, k, n) in ((256, 2048, 4096), (72, 128, 384), (1024, 6144, 2048)):
        lin = Linear(k, n, bias=False).cuda().to(torch.bfloat16)
        x = (torch.randn(2, m // 2, k, device="cuda") * 0.5).to(torch.bfloat16).requires_grad_(True)
        gy = torch.randn(2, m // 2, n, device="cuda").to(torch.bfloat16)
        y = lin(x)
        y.backward(gy)
        xf = x.detach().float().reshape(m, k)
        wf = lin.weight.detach().float()
        gf = gy.float().reshape(m, n)
        for got, ref in ((y.float().reshape(m, n), xf @ wf.t()), (x.grad.float().reshape(m, k), gf @ wf),
                         (lin.weight.grad.float(), gf.t() @ xf)):
            rel = (got - ref).norm() / ref.norm()
            assert rel < 1e-2, (m, k, n, rel.item())
