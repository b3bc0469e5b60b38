"""Training stack on CPU: packed block layout, fused LM-head loss vs the
full-logit oracle (values and gradients), sharded AdamW vs torch AdamW
(1 and 2 gloo ranks), checkpoint/resume round trip."""
import os
import random
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from d3d_b200.engine.layout import rows_to_dense
from d3d_b200.train.blocks import Example, build_packed_block_batch
from d3d_b200.train.losses import ce_per_token, forward_kl_per_token, lmhead_distill_loss
from d3d_b200.train.optim import ShardedAdamW


def _reference_mask(batch):
    """Dense mask restated from the reference's construction
    (context before the anchor + own block; invalid blocks see themselves)."""
    B, Q = batch.draft_ids.shape
    Lc, K = batch.clean_ids.shape[1], batch.block_size
    kv = torch.arange(Lc + Q)
    q = torch.arange(Q)
    anchors = batch.anchor_positions.repeat_interleave(K, 1)          # [B, Q]
    ctx = (kv[None, None, :] < Lc) & (kv[None, None, :] < anchors[:, :, None])
    draft = (kv[None, None, :] >= Lc) & (((kv - Lc) // K)[None, None, :] == (q // K)[None, :, None])
    valid = batch.block_keep.repeat_interleave(K, 1)[:, :, None]
    self_m = (kv[None, None, :] - Lc) == q[None, :, None]
    return ((ctx | draft) & valid) | (self_m & ~valid)


def test_packed_blocks_match_reference_mask():
    rng = random.Random(0)
    exs = [Example([rng.randrange(50) for _ in range(7)], [rng.randrange(50) for _ in range(20)]),
           Example([1, 2, 3], [4, 5, 6, 7]), Example([9] * 12, [8] * 3)]
    b = build_packed_block_batch(exs, block_size=4, mask_token_id=99, max_anchors=5, rng=rng)
    dense = rows_to_dense(b.rows, b.clean_ids.shape[1] + b.draft_ids.shape[1])
    assert torch.equal(dense, _reference_mask(b))
    # targets: block row o predicts response[s+o]; teacher position anchor+o-1
    act = b.active
    assert torch.equal(b.teacher_pos[act], (b.positions[act] - 1))
    seqs = [e.prompt_ids + e.response_ids for e in exs]
    for bi in range(3):
        for q in act[bi].nonzero(as_tuple=True)[0].tolist():
            assert b.target_ids[bi, q] == seqs[bi][b.positions[bi, q]]


@pytest.mark.parametrize("chunk", [37, 1000])
def test_fused_lmhead_loss_matches_oracle(chunk):
    torch.manual_seed(0)
    N, V, Hs, Ht = 23, 517, 32, 48
    hs = torch.randn(N, Hs, requires_grad=True)
    ws = (torch.randn(V, Hs) * 0.3).requires_grad_(True)
    ht, wt = torch.randn(N, Ht), torch.randn(V, Ht) * 0.3
    tgt = torch.randint(0, V, (N,))
    wk, wc = torch.rand(N), torch.rand(N)
    loss, kl, ce = lmhead_distill_loss(hs, ws, ht, wt, tgt, wk, wc, chunk=chunk)
    loss.backward()
    g1 = (hs.grad.clone(), ws.grad.clone())
    hs.grad = None
    ws.grad = None
    zs, zt = hs @ ws.t(), ht @ wt.t()
    rk, rc = forward_kl_per_token(zs, zt), ce_per_token(zs, tgt)
    ref = (wk * rk).sum() + (wc * rc).sum()
    ref.backward()
    assert torch.allclose(loss, ref, rtol=1e-5, atol=1e-5)
    assert torch.allclose(kl, rk.detach(), rtol=1e-4, atol=1e-5)
    assert torch.allclose(ce, rc.detach(), rtol=1e-5, atol=1e-5)
    assert torch.allclose(g1[0], hs.grad, rtol=1e-4, atol=1e-5)
    assert torch.allclose(g1[1], ws.grad, rtol=1e-4, atol=1e-5)


def test_sharded_adamw_matches_torch_single_rank():
    torch.manual_seed(1)
    a = torch.nn.Linear(7, 5)
    b = torch.nn.Linear(7, 5)
    b.load_state_dict(a.state_dict())
    opt_a = ShardedAdamW(a.parameters(), lr=1e-2, weight_decay=0.1)
    opt_b = torch.optim.AdamW(b.parameters(), lr=1e-2, weight_decay=0.1, eps=1e-8)
    for _ in range(4):
        x = torch.randn(3, 7)
        for m in (a, b):
            m(x).pow(2).sum().backward()
        opt_a.step()
        opt_b.step()
        opt_a.zero_grad()
        opt_b.zero_grad()
    for pa, pb in zip(a.parameters(), b.parameters()):
        assert torch.allclose(pa, pb, atol=1e-6)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _dp_worker(rank, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    torch.manual_seed(3)
    m = torch.nn.Linear(6, 4)
    opt = ShardedAdamW(m.parameters(), lr=5e-3)
    g = torch.Generator().manual_seed(10)
    xs = [torch.randn(4, 6, generator=g) for _ in range(3)]
    for x in xs:
        part = x[rank * 2:(rank + 1) * 2]
        (m(part).pow(2).sum() * 2).backward()     # mean over ranks happens in step()
        opt.step(grad_clip=0.5)
        opt.zero_grad()
    if rank == 0:
        torch.save({k: v.clone() for k, v in m.state_dict().items()}, out)
    dist.destroy_process_group()


def test_sharded_adamw_two_ranks_equals_full_batch():
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "w.pt")
        mp.spawn(_dp_worker, args=(_port(), out), nprocs=2)
        dp = torch.load(out)
    torch.manual_seed(3)
    m = torch.nn.Linear(6, 4)
    opt = ShardedAdamW(m.parameters(), lr=5e-3)
    g = torch.Generator().manual_seed(10)
    for x in [torch.randn(4, 6, generator=g) for _ in range(3)]:
        m(x).pow(2).sum().backward()
        opt.step(grad_clip=0.5)
        opt.zero_grad()
    for k, v in m.state_dict().items():
        assert torch.allclose(v, dp[k], atol=1e-6), k


def test_trainer_checkpoint_roundtrip(tmp_path):
    from d3d_b200.checkpoint import load_model
    from d3d_b200.train.args import parser
    from d3d_b200.train.trainer import train
    a = parser().parse_args(["--draft-model", "tiny-drafter", "--target-model", "tiny-target",
                             "--output-dir", str(tmp_path), "--seq-len", "80", "--batch-size", "2",
                             "--parallel-anchors-per-example", "3", "--max-steps", "2", "--block-size", "8",
                             "--vocab-chunk", "256", "--save-final", "--device", "cpu", "--dtype", "fp32"])
    r = train(a)
    assert all(torch.isfinite(torch.tensor(x["loss"])) for x in r["log"])
    m = load_model(tmp_path / "step_0000002")
    assert m.cfg.d3d_draft and m.cfg.cond_hidden_size == 128
    a.resume = str(tmp_path / "step_0000002")
    a.max_steps = 3
    a.save_final = False
    r2 = train(a)
    assert [x["step"] for x in r2["log"]] == [3]


def _empty_rank_worker(rank, port, out_dir):
    import datetime
    import json
    import os
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["RANK"], os.environ["WORLD_SIZE"], os.environ["LOCAL_RANK"] = str(rank), "2", str(rank)
    from d3d_b200.train.args import parser
    from d3d_b200.train.trainer import train
    # rank 1 reads only one-token responses: no anchor, nothing to supervise
    data = os.path.join(out_dir, "data.jsonl")
    args = parser().parse_args([
        "--draft-model", "tiny-drafter", "--target-model", "tiny-target", "--output-dir", out_dir,
        "--data-path", data, "--max-steps", "2", "--batch-size", "1", "--device", "cpu", "--dtype", "fp32",
        "--parallel-anchors-per-example", "2", "--vocab-chunk", "256", "--save-every", "2"])
    out = train(args)
    with open(os.path.join(out_dir, f"log{rank}.json"), "w") as f:
        json.dump(out["log"], f)
    if dist.is_initialized():
        dist.destroy_process_group()


def test_rank_with_empty_batches_keeps_collectives_matched(tmp_path):
    import json
    import random
    import socket
    import torch.multiprocessing as mp
    rng = random.Random(0)
    rows = []
    for i in range(4):
        resp = [rng.randrange(2, 1000) for _ in range(12)] if i % 2 == 0 else [5]
        rows.append(json.dumps({"prompt_ids": [rng.randrange(2, 1000) for _ in range(8)], "response_ids": resp}))
    (tmp_path / "data.jsonl").write_text("\n".join(rows) + "\n")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_empty_rank_worker, args=(port, str(tmp_path)), nprocs=2, join=True)
    l0 = json.loads((tmp_path / "log0.json").read_text())
    l1 = json.loads((tmp_path / "log1.json").read_text())
    assert len(l0) == len(l1) == 2
    assert all(r.get("empty_rank") for r in l1) and not any(r.get("empty_rank") for r in l0)
    assert all(a["grad_norm"] == b["grad_norm"] for a, b in zip(l0, l1))
    assert (tmp_path / "trainer_state.json").exists() or any(tmp_path.glob("**/trainer_state.json"))


def test_gradient_checkpointing_keeps_clean_prefix_cache():
    """Per-layer recomputation with a clean-prefix KV cache gives the same
    outputs and gradients as keeping the activations."""
    from d3d_b200.cli.common import model_config
    from d3d_b200.models.qwen3 import DenseKVCache, build_model
    torch.manual_seed(0)
    clean = torch.randint(0, 1000, (2, 20))
    draft = torch.randint(0, 1000, (2, 8))
    pos = torch.arange(20, 28)[None].expand(2, 8)
    mask = torch.ones(2, 8, 28, dtype=torch.bool)
    outs = []
    for ckpt in (False, True):
        m = build_model(model_config("tiny-drafter"), seed=3, dtype=torch.float32, device="cpu")
        m.eval()
        cache = DenseKVCache(m.cfg.num_hidden_layers)
        with torch.no_grad():
            m(clean, cache=cache, store_kv=True)
        m.train()
        m.gradient_checkpointing = ckpt
        h = m(draft, pos, mask=mask, cache=cache, store_kv=False)
        h.square().mean().backward()
        outs.append((h.detach(), [p.grad.clone() for p in m.parameters() if p.grad is not None]))
    assert torch.equal(outs[0][0], outs[1][0])
    assert len(outs[0][1]) == len(outs[1][1]) > 0
    for a, b in zip(outs[0][1], outs[1][1]):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("extra", [[], ["--fsdp"]])
def test_resume_continues_exactly(tmp_path, extra):
    """Two steps, a checkpoint, then the third step from it: the same weights
    as three uninterrupted steps (weights, optimizer shards and moments, data
    cursor all restored)."""
    from d3d_b200.checkpoint import load_model
    from d3d_b200.train.args import parser
    from d3d_b200.train.trainer import train

    def run(out, steps, more):
        train(parser().parse_args([
            "--draft-model", "tiny-drafter", "--target-model", "tiny-target", "--output-dir", str(out),
            "--seq-len", "80", "--batch-size", "2", "--parallel-anchors-per-example", "3",
            "--max-steps", str(steps), "--block-size", "8", "--vocab-chunk", "256", "--device", "cpu",
            "--dtype", "fp32", "--min-lr-ratio", "1.0", "--log-every", "0"] + extra + more))

    run(tmp_path / "a", 3, ["--save-final"])
    run(tmp_path / "b", 2, ["--save-every", "2"])
    run(tmp_path / "b", 3, ["--save-final", "--resume", str(tmp_path / "b" / "step_0000002")])
    ma = dict(load_model(tmp_path / "a" / "step_0000003").named_parameters())
    mb = dict(load_model(tmp_path / "b" / "step_0000003").named_parameters())
    assert all(torch.equal(ma[n], mb[n]) for n in ma)
