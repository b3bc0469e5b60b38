"""Sharded decoder layers (FSDP / ZeRO-3 style) on CPU: the layer shards,
per-layer gather, recomputing backward and per-layer gradient reduce-scatter
must train exactly like the replicated model -- in one process and over two
``gloo`` ranks, with a rank that has nothing to supervise, and through a
checkpoint."""
import json
import os
import random
import socket

import torch
import torch.multiprocessing as mp

from d3d_b200.parallel.zero3 import ShardedLayer, Zero3Layers
from d3d_b200.train.optim import ShardedAdamW


def _tiny():
    from d3d_b200.cli.common import model_config
    from d3d_b200.models.qwen3 import build_model
    return build_model(model_config("tiny-drafter"), seed=3, dtype=torch.float32, device="cpu")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_single_rank_matches_replicated_step():
    torch.manual_seed(0)
    ref, sh = _tiny(), _tiny()
    z = Zero3Layers(sh.model.layers, lr=1e-3)
    assert all(isinstance(m, ShardedLayer) for m in sh.model.layers)
    assert not any(n.startswith("model.layers.") for n, _ in sh.named_parameters())
    ids = torch.randint(0, 1000, (2, 24))
    # forward equality, with gradients through every layer
    h_ref, h_sh = ref(ids), sh(ids)
    assert torch.equal(h_ref, h_sh)
    (h_ref.square().mean()).backward()
    (h_sh.square().mean()).backward()
    # the layer shard gradients are the replicated gradients, flattened per layer
    for i, lay in enumerate(ref.model.layers):
        s = z.specs[i]
        flat = torch.cat([p.grad.reshape(-1) for p in lay.parameters()])
        torch.testing.assert_close(z.grad[s.offset:s.offset + s.numel], flat, rtol=0, atol=0)
    # one optimizer step each: same weights afterwards
    o_ref = ShardedAdamW([p for p in ref.parameters()], lr=1e-3)
    o_sh = ShardedAdamW([p for p in sh.parameters()], lr=1e-3)
    n_ref = o_ref.step(1.0)
    n_sh = o_sh.step(1.0, extra_sumsq=z.sumsq())
    z.step(o_sh.last_scale)
    assert abs(n_ref - n_sh) < 1e-6 * max(1.0, n_ref)
    full = z.full_state("model.layers.")
    for n, p in ref.named_parameters():
        if n.startswith("model.layers."):
            torch.testing.assert_close(full[n], p.detach(), rtol=1e-6, atol=1e-7)
    # and the next forward reads the updated shards
    torch.testing.assert_close(sh(ids), ref(ids), rtol=1e-5, atol=1e-6)


def _train_worker(rank, port, out_dir, extra, tag):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["RANK"], os.environ["WORLD_SIZE"], os.environ["LOCAL_RANK"] = str(rank), "2", str(rank)
    import torch.distributed as dist
    from d3d_b200.train.args import parser
    from d3d_b200.train.trainer import train
    run = os.path.join(out_dir, tag)
    args = parser().parse_args([
        "--draft-model", "tiny-drafter", "--target-model", "tiny-target", "--output-dir", run,
        "--max-steps", "3", "--batch-size", "1", "--device", "cpu", "--dtype", "fp32",
        "--parallel-anchors-per-example", "2", "--vocab-chunk", "256", "--save-final"] + extra)
    out = train(args)
    with open(os.path.join(run, f"log{rank}.json"), "w") as f:
        json.dump(out["log"], f)
    if dist.is_initialized():
        dist.destroy_process_group()


def _run(tmp, extra, tag):
    mp.spawn(_train_worker, args=(_port(), str(tmp), extra, tag), nprocs=2, join=True)
    return [json.loads((tmp / tag / f"log{r}.json").read_text()) for r in range(2)]


def _data(tmp, empty_rank: bool):
    rng = random.Random(0)
    rows = []
    for i in range(6):
        short = empty_rank and i % 2 == 1
        resp = [5] if short else [rng.randrange(2, 1000) for _ in range(12)]
        rows.append(json.dumps({"prompt_ids": [rng.randrange(2, 1000) for _ in range(8)], "response_ids": resp}))
    p = tmp / "data.jsonl"
    p.write_text("\n".join(rows) + "\n")
    return str(p)


def _compare(tmp, a, b):
    from d3d_b200.checkpoint import load_model
    for la, lb in zip(a, b):
        for x, y in zip(la, lb):
            assert abs(x["loss"] - y["loss"]) <= 1e-5 * max(1.0, abs(x["loss"]))
            assert abs(x["grad_norm"] - y["grad_norm"]) <= 1e-5 * max(1.0, x["grad_norm"])
    ma = load_model(tmp / "rep" / "step_0000003")
    mb = load_model(tmp / "fsdp" / "step_0000003")
    sa, sb = dict(ma.named_parameters()), dict(mb.named_parameters())
    assert sa.keys() == sb.keys()
    for n in sa:
        torch.testing.assert_close(sb[n], sa[n], rtol=1e-5, atol=1e-6, msg=n)


def test_two_ranks_match_replicated_training(tmp_path):
    data = _data(tmp_path, empty_rank=False)
    a = _run(tmp_path, ["--data-path", data], "rep")
    b = _run(tmp_path, ["--data-path", data, "--fsdp"], "fsdp")
    _compare(tmp_path, a, b)


def test_two_ranks_with_an_empty_rank_and_ar_loss(tmp_path):
    """Rank 1 has nothing to supervise: it takes part in every layer's
    gradient exchange with zeros (two passes: block loss and AR loss)."""
    data = _data(tmp_path, empty_rank=True)
    extra = ["--data-path", data, "--ar-weight", "0.5"]
    a = _run(tmp_path, extra, "rep")
    b = _run(tmp_path, extra + ["--fsdp"], "fsdp")
    assert all(r.get("empty_rank") for r in b[1])
    _compare(tmp_path, a, b)


def test_frozen_embeddings_still_train_sharded_layers():
    """The first layer's input needs no gradient when the embeddings are
    frozen; the sharded layers must get their gradients all the same."""
    ref, sh = _tiny(), _tiny()
    for m in (ref, sh):
        m.model.embed_tokens.weight.requires_grad_(False)
    z = Zero3Layers(sh.model.layers, lr=1e-3)
    ids = torch.randint(0, 1000, (2, 16))
    ref(ids).square().mean().backward()
    sh(ids).square().mean().backward()
    for i, lay in enumerate(ref.model.layers):
        s = z.specs[i]
        flat = torch.cat([p.grad.reshape(-1) for p in lay.parameters()])
        assert flat.abs().sum() > 0
        torch.testing.assert_close(z.grad[s.offset:s.offset + s.numel], flat, rtol=0, atol=0)
