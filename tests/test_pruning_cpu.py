"""Pruning on CPU: single-layer deletion scoring equals an explicit forward
without the layer; the physical prune remaps tensors and records provenance
(and refuses to overwrite); a recovery step runs; checkpoint choice ranks by
accept length."""
import json
import random

import pytest
import torch

from d3d_b200.checkpoint import load_model, save_model
from d3d_b200.config import tiny_drafter
from d3d_b200.models.qwen3 import build_model
from d3d_b200.pruning.modeling import _inputs, evaluate_single_layer_removals, examples_from_sequences, \
    hard_accept_length
from d3d_b200.pruning.prune import prune_checkpoint
from d3d_b200.pruning.recovery import make_student, recovery_step
from d3d_b200.pruning.select_checkpoint import choose
from d3d_b200.pruning.select_layer import select_layers
from d3d_b200.train.blocks import synthetic_examples
from d3d_b200.train.optim import ShardedAdamW


def _model(layers=4):
    return build_model(tiny_drafter(cond=False).replace(num_hidden_layers=layers), seed=3).eval()


def _examples(k=8):
    rng = random.Random(0)
    seqs = [[rng.randrange(1000) for _ in range(50)] for _ in range(3)]
    return examples_from_sequences(seqs, k, 2, rng)


def test_removal_scores_match_explicit_skip():
    m = _model()
    ex = _examples()
    full, cand = evaluate_single_layer_removals(m, ex, 8)
    for j in range(4):
        rs = []
        for e in ex:
            ids, pos, mask = _inputs(m, e, 8, "causal")
            h = m(ids, pos, mask=mask, layer_skip=[j])
            lg = m.logits(h[:, -8:])[0, 1:]
            rs.append(hard_accept_length(lg.argmax(-1), torch.tensor(e.continuation)))
        assert cand[j][0] == pytest.approx(sum(r[0] for r in rs) / len(rs))
    assert 1.0 <= full[0] <= 8.0


def test_prune_checkpoint_remaps_and_records(tmp_path):
    m = _model()
    save_model(m, tmp_path / "parent")
    out = prune_checkpoint(tmp_path / "parent", tmp_path / "child", removed=1)
    c = load_model(out)
    assert c.cfg.num_hidden_layers == 3
    sd_p, sd_c = m.state_dict(), c.state_dict()
    for new, old in enumerate([0, 2, 3]):
        a = sd_p[f"model.layers.{old}.mlp.down_proj.weight"]
        assert torch.equal(sd_c[f"model.layers.{new}.mlp.down_proj.weight"], a)
    prov = json.loads((out / "layer_prune.json").read_text())
    assert prov["retained_original_layers"] == [0, 2, 3] and prov["removed_original_layer"] == 1
    with pytest.raises(FileExistsError):
        prune_checkpoint(tmp_path / "parent", tmp_path / "child", removed=0)
    out2 = prune_checkpoint(out, tmp_path / "grandchild", removed=2)
    assert json.loads((out2 / "layer_prune.json").read_text())["retained_original_layers"] == [0, 2]


def test_progressive_select_and_recovery():
    m = _model()
    res = select_layers(m, _examples(), 8, drop=2)
    assert len(res["retained_original_layers"]) == 2 and m.cfg.num_hidden_layers == 2
    parent = _model()
    for p in parent.parameters():
        p.requires_grad_(False)
    removed = res["history"][0]["removed_compact_layer"]
    child = make_student(parent, removed)
    opt = ShardedAdamW([p for p in child.parameters() if p.requires_grad], lr=1e-4)
    rng = random.Random(1)
    r = recovery_step(child, parent, removed, [i for i in range(4) if i != removed],
                      synthetic_examples(2, 64, 0.25, 1000, rng), opt, block_size=8, anchors=4, rng=rng)
    assert all(torch.isfinite(torch.tensor(v)) for v in r.values())


def test_choose_checkpoint(tmp_path):
    a, b = _model(), _model()
    save_model(a, tmp_path / "step_10")
    save_model(b, tmp_path / "step_20")
    res = choose([str(tmp_path / "step_10"), str(tmp_path / "step_20")], _examples(), 8)
    assert res["best"]["checkpoint"].endswith("step_10")   # tie -> earliest step


def _recovery_worker(rank, port, root):
    import os
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["RANK"], os.environ["WORLD_SIZE"], os.environ["LOCAL_RANK"] = str(rank), "2", str(rank)
    import torch.distributed as dist
    from d3d_b200.pruning.__main__ import main
    main(["train", "--parent", f"{root}/parent", "--child", f"{root}/child", "--output", f"{root}/recovered",
          "--data-path", f"{root}/data.jsonl", "--batch-size", "1", "--steps", "10", "--block-size", "8",
          "--device", "cpu", "--save-every", "1"])
    if dist.is_initialized():
        dist.destroy_process_group()


def test_distributed_recovery_stops_together_and_records_cursor(tmp_path):
    """Two gloo ranks: the 5-row window runs out for rank 1 at step 3, both
    ranks stop there, and the checkpoints carry the next data cursor."""
    import socket
    import torch.multiprocessing as mp
    m = _model()
    save_model(m, tmp_path / "parent")
    prune_checkpoint(tmp_path / "parent", tmp_path / "child", removed=1)
    rng = random.Random(2)
    rows = [json.dumps({"prompt_ids": [rng.randrange(2, 1000) for _ in range(10)],
                        "response_ids": [rng.randrange(2, 1000) for _ in range(20)]}) for _ in range(5)]
    (tmp_path / "data.jsonl").write_text("\n".join(rows) + "\n")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_recovery_worker, args=(port, str(tmp_path)), nprocs=2, join=True)
    state = json.loads((tmp_path / "recovered" / "trainer_state.json").read_text())
    assert state == {"next_data_cursor": 4, "steps": 2}
    assert json.loads((tmp_path / "recovered.step1" / "trainer_state.json").read_text())["next_data_cursor"] == 2
    assert load_model(tmp_path / "recovered").cfg.num_hidden_layers == 3
    assert (tmp_path / "recovered" / "layer_prune.json").exists()


def _select_worker(rank, port, root):
    import os
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from d3d_b200.pruning.__main__ import main
    main(["select", "--checkpoint", f"{root}/parent", "--output", f"{root}/sel2.json", "--samples", "5",
          "--block-size", "8", "--device", "cpu", "--drop", "2"])
    main(["choose", "--checkpoints", f"{root}/parent", f"{root}/parent_b", "--output", f"{root}/best2.json",
          "--samples", "5", "--block-size", "8", "--device", "cpu"])
    if dist.is_initialized():
        dist.destroy_process_group()


def test_data_parallel_selection_equals_single_process(tmp_path):
    """Layer selection and checkpoint choice on two gloo ranks (examples
    sharded rank::2, rows gathered in example order) give exactly the
    single-process result: same removed layers, same means, same ranking."""
    import socket
    import torch.multiprocessing as mp
    from d3d_b200.pruning.__main__ import main
    save_model(_model(), tmp_path / "parent")
    save_model(build_model(tiny_drafter(cond=False).replace(num_hidden_layers=4), seed=9), tmp_path / "parent_b")
    main(["select", "--checkpoint", str(tmp_path / "parent"), "--output", str(tmp_path / "sel1.json"),
          "--samples", "5", "--block-size", "8", "--device", "cpu", "--drop", "2"])
    main(["choose", "--checkpoints", str(tmp_path / "parent"), str(tmp_path / "parent_b"), "--output",
          str(tmp_path / "best1.json"), "--samples", "5", "--block-size", "8", "--device", "cpu"])
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_select_worker, args=(port, str(tmp_path)), nprocs=2, join=True)
    one = json.loads((tmp_path / "sel1.json").read_text())
    two = json.loads((tmp_path / "sel2.json").read_text())
    assert one["metrics"]["history"] == two["metrics"]["history"]
    assert one["metrics"]["history"][0]["samples"] == 10
    b1 = json.loads((tmp_path / "best1.json").read_text())
    b2 = json.loads((tmp_path / "best2.json").read_text())
    assert b1["ranking"] == b2["ranking"]


def _recovery_fsdp_worker(rank, port, root, tag, extra):
    import os
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["RANK"], os.environ["WORLD_SIZE"], os.environ["LOCAL_RANK"] = str(rank), "2", str(rank)
    import torch.distributed as dist
    from d3d_b200.pruning.__main__ import main
    main(["train", "--parent", f"{root}/parent", "--child", f"{root}/child", "--output", f"{root}/{tag}",
          "--data-path", f"{root}/data.jsonl", "--batch-size", "1", "--steps", "3", "--block-size", "8",
          "--device", "cpu", "--lr", "1e-3"] + extra)
    if dist.is_initialized():
        dist.destroy_process_group()


def test_recovery_with_sharded_layers_equals_replicated(tmp_path):
    """Recovery training of the pruned child with its decoder layers sharded
    over two gloo ranks (``--fsdp``) ends with the same weights and log as the
    replicated run."""
    import socket
    import torch.multiprocessing as mp
    m = _model()
    save_model(m, tmp_path / "parent")
    prune_checkpoint(tmp_path / "parent", tmp_path / "child", removed=1)
    rng = random.Random(3)
    rows = [json.dumps({"prompt_ids": [rng.randrange(2, 1000) for _ in range(10)],
                        "response_ids": [rng.randrange(2, 1000) for _ in range(20)]}) for _ in range(8)]
    (tmp_path / "data.jsonl").write_text("\n".join(rows) + "\n")
    for tag, extra in (("rep", []), ("fsdp", ["--fsdp"])):
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
        s.close()
        mp.spawn(_recovery_fsdp_worker, args=(port, str(tmp_path), tag, extra), nprocs=2, join=True)
    la = json.loads((tmp_path / "rep" / "recovery_log.json").read_text())
    lb = json.loads((tmp_path / "fsdp" / "recovery_log.json").read_text())
    assert len(la) == len(lb) == 3
    for x, y in zip(la, lb):
        assert abs(x["loss"] - y["loss"]) <= 1e-5 * max(1.0, abs(x["loss"]))
    ma, mb = load_model(tmp_path / "rep"), load_model(tmp_path / "fsdp")
    sa, sb = dict(ma.named_parameters()), dict(mb.named_parameters())
    assert sa.keys() == sb.keys()
    for n in sa:
        torch.testing.assert_close(sb[n], sa[n], rtol=1e-5, atol=1e-6, msg=n)
