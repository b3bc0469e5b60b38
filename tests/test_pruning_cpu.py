"""Pruning on CPU: single-layer deletion scoring equals an explicit forward
without the layer; the physical prune remaps tensors and records the full
provenance (and refuses to overwrite); the four stages run end to end through
the command line with the reference's flags and files; selection over two
worker processes or two gloo ranks equals one process; recovery ranks fail
together when data runs out; sharded-layer recovery equals replicated."""
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
from d3d_b200.pruning.select_checkpoint import choose
from d3d_b200.pruning.select_layer import select_layers


def _model(layers=4, seed=3):
    return build_model(tiny_drafter(cond=False).replace(num_hidden_layers=layers), seed=seed).eval()


def _examples(k=8):
    rng = random.Random(0)
    seqs = [[rng.randrange(1000) for _ in range(50)] for _ in range(3)]
    return examples_from_sequences(seqs, k, 2, rng)


def _write_examples(path, n, k=8, seed=0):
    rng = random.Random(seed)
    rows = []
    for split in ("layer_selection", "layer_validation"):
        for i in range(n):
            rows.append({"analysis_id": f"{split}-{i}", "split": split,
                         "prefix_ids": [rng.randrange(2, 1000) for _ in range(rng.randint(10, 30))],
                         "target_ids": [rng.randrange(2, 1000) for _ in range(k)]})
    path.write_text("\n".join(json.dumps(r) for r in rows) + "\n")


def _write_rows(path, n, seed=2):
    rng = random.Random(seed)
    rows = [json.dumps({"prompt_ids": [rng.randrange(2, 1000) for _ in range(10)],
                        "response_ids": [rng.randrange(2, 1000) for _ in range(20)]}) for _ in range(n)]
    path.write_text("\n".join(rows) + "\n")


def _port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


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
    out = prune_checkpoint(tmp_path / "parent", tmp_path / "child", removed=1, block_size=8)
    c = load_model(out)
    assert c.cfg.num_hidden_layers == 3
    sd_p, sd_c = m.state_dict(), c.state_dict()
    for new, old in enumerate([0, 2, 3]):
        a = sd_p[f"model.layers.{old}.mlp.down_proj.weight"]
        assert torch.equal(sd_c[f"model.layers.{new}.mlp.down_proj.weight"], a)
    prov = json.loads((out / "layer_prune.json").read_text())
    assert prov["retained_original_layers"] == [0, 2, 3] and prov["removed_original_layer"] == 1
    assert prov["retained_parent_layers"] == [0, 2, 3] and prov["removed_parent_layer"] == 1
    assert prov["teacher_checkpoint"] == str((tmp_path / "parent").resolve()) and prov["original_depth"] == 4
    assert prov["block_size"] == 8 and prov["parameters"] == sum(v.numel() for v in sd_c.values()) - (
        0 if not c.cfg.tie_word_embeddings else 0)
    with pytest.raises(FileExistsError):
        prune_checkpoint(tmp_path / "parent", tmp_path / "child", removed=0)
    out2 = prune_checkpoint(out, tmp_path / "grandchild", removed=2)
    p2 = json.loads((out2 / "layer_prune.json").read_text())
    assert p2["retained_original_layers"] == [0, 2] and p2["removed_original_layer"] == 3
    assert p2["teacher_checkpoint"] == prov["teacher_checkpoint"] and p2["original_depth"] == 4


def test_progressive_select_in_memory():
    m = _model()
    res = select_layers(m, _examples(), 8, drop=2)
    assert len(res["retained_original_layers"]) == 2 and m.cfg.num_hidden_layers == 2


def test_choose_checkpoint_prefers_earliest_on_tie(tmp_path):
    a, b = _model(), _model()
    save_model(a, tmp_path / "step-10")
    save_model(b, tmp_path / "step-20")
    res = choose([str(tmp_path / "step-20"), str(tmp_path / "step-10")], _examples(), 8)
    assert res["best"]["checkpoint"].endswith("step-10")


def test_four_stages_through_the_cli(tmp_path):
    """select -> prune -> train -> choose, then a second select/prune cycle on
    the recovered child: outputs, provenance and data cursor as specified."""
    import pandas as pd
    from d3d_b200.pruning.__main__ import main
    save_model(_model(), tmp_path / "parent")
    _write_examples(tmp_path / "ex.jsonl", 6)
    _write_rows(tmp_path / "data.jsonl", 12)
    sel = main(["select", "--parent", str(tmp_path / "parent"), "--examples", str(tmp_path / "ex.jsonl"),
                "--output-dir", str(tmp_path / "sel"), "--expected-samples", "6", "--block-size", "8",
                "--devices", "cpu", "--dtype", "fp32", "--bootstrap-samples", "300"])
    s = json.loads((tmp_path / "sel" / "selection.json").read_text())
    assert s["parent_depth"] == 4 and s["child_depth"] == 3 and s["selection_samples"] == 6
    assert s["removed_compact_layer"] == sel["summary"][0]["removed_compact_layer"]
    table = pd.read_csv(tmp_path / "sel" / "candidate_summary.csv")
    assert list(table["rank"]) == [1, 2, 3, 4] and table["selected"].sum() == 1
    assert (table["damage_ci95_low"] <= table["damage_ci95_high"]).all()
    assert len(pd.read_parquet(tmp_path / "sel" / "candidate_metrics.parquet")) == 4 * 6
    with pytest.raises(FileExistsError):
        main(["select", "--parent", str(tmp_path / "parent"), "--examples", str(tmp_path / "ex.jsonl"),
              "--output-dir", str(tmp_path / "sel"), "--expected-samples", "6", "--devices", "cpu"])
    with pytest.raises(ValueError, match="Expected"):
        main(["select", "--parent", str(tmp_path / "parent"), "--examples", str(tmp_path / "ex.jsonl"),
              "--output-dir", str(tmp_path / "sel_bad"), "--expected-samples", "7", "--block-size", "8",
              "--devices", "cpu", "--dtype", "fp32"])
    main(["prune", "--selection", str(tmp_path / "sel" / "selection.json"), "--output", str(tmp_path / "child")])
    prov = json.loads((tmp_path / "child" / "layer_prune.json").read_text())
    assert prov["block_size"] == 8 and prov["child_depth"] == 3
    summ = main(["train", "--student", str(tmp_path / "child"), "--dataset", str(tmp_path / "data.jsonl"),
                 "--output-dir", str(tmp_path / "run"), "--max-steps", "2", "--gradient-accumulation-steps", "2",
                 "--save-steps", "1", "--log-steps", "1", "--learning-rate", "1e-3", "--min-lr", "1e-4",
                 "--warmup-ratio", "0.5", "--anchors-per-example", "4", "--device", "cpu"])
    assert summ["completed_steps"] == 2 and summ["next_data_cursor"] == 8        # 2 x 2 x 1 x multiplier 2
    recs = [json.loads(x) for x in (tmp_path / "run" / "training_metrics.jsonl").read_text().splitlines()]
    # one warm-up step ends at the base rate; the cosine then reaches the minimum at the last step
    assert [r["optimizer_step"] for r in recs] == [1, 2]
    assert [r["learning_rate"] for r in recs] == pytest.approx([1e-3, 1e-4])
    assert all(torch.isfinite(torch.tensor(r["loss"])) for r in recs)
    for step in (1, 2):
        d = tmp_path / "run" / f"step-{step}"
        assert (d / "layer_prune.json").exists()
        assert json.loads((d / "recovery_info.json").read_text())["optimizer_step"] == step
    assert load_model(tmp_path / "run" / "step-2").cfg.num_hidden_layers == 3
    main(["choose", "--run-dir", str(tmp_path / "run"), "--examples", str(tmp_path / "ex.jsonl"),
          "--output-dir", str(tmp_path / "best"), "--expected-samples", "6", "--block-size", "8",
          "--devices", "cpu", "--dtype", "fp32"])
    best = json.loads((tmp_path / "best" / "selected_checkpoint.json").read_text())
    assert best["selected_step"] in (1, 2) and best["samples"] == 6
    # the next cycle starts from the chosen checkpoint; the teacher stays the original
    main(["select", "--parent", best["selected_checkpoint"], "--examples", str(tmp_path / "ex.jsonl"),
          "--output-dir", str(tmp_path / "sel2"), "--expected-samples", "6", "--block-size", "8",
          "--devices", "cpu", "--dtype", "fp32", "--bootstrap-samples", "100"])
    s2 = json.loads((tmp_path / "sel2" / "selection.json").read_text())
    assert s2["teacher_checkpoint"] == str((tmp_path / "parent").resolve()) and s2["original_depth"] == 4
    main(["prune", "--selection", str(tmp_path / "sel2" / "selection.json"), "--output", str(tmp_path / "child2")])
    p2 = json.loads((tmp_path / "child2" / "layer_prune.json").read_text())
    assert len(p2["retained_original_layers"]) == 2
    assert set(p2["retained_original_layers"]) < set(prov["retained_original_layers"])


def test_selection_on_two_worker_processes_equals_one(tmp_path):
    from d3d_b200.pruning.__main__ import main
    save_model(_model(), tmp_path / "parent")
    _write_examples(tmp_path / "ex.jsonl", 5)
    outs = []
    for tag, devs in (("one", ["cpu"]), ("two", ["cpu:0", "cpu:1"])):
        main(["select", "--parent", str(tmp_path / "parent"), "--examples", str(tmp_path / "ex.jsonl"),
              "--output-dir", str(tmp_path / tag), "--expected-samples", "5", "--block-size", "8",
              "--dtype", "fp32", "--bootstrap-samples", "50", "--devices", *devs])
        s = json.loads((tmp_path / tag / "selection.json").read_text())
        s.pop("elapsed_seconds")
        outs.append(s)
    assert outs[0] == outs[1]


def _select_worker(rank, port, root):
    import os
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from d3d_b200.pruning.__main__ import main
    main(["select", "--parent", f"{root}/parent", "--examples", f"{root}/ex.jsonl", "--output-dir", f"{root}/sel2",
          "--expected-samples", "5", "--block-size", "8", "--devices", "cpu", "--dtype", "fp32",
          "--bootstrap-samples", "50"])
    main(["choose", "--checkpoints", f"{root}/parent", f"{root}/parent_b", "--examples", f"{root}/ex.jsonl",
          "--output-dir", f"{root}/best2", "--expected-samples", "5", "--block-size", "8", "--devices", "cpu",
          "--dtype", "fp32"])
    if dist.is_initialized():
        dist.destroy_process_group()


def test_data_parallel_selection_equals_single_process(tmp_path):
    """Layer selection and checkpoint choice on two gloo ranks (examples
    sharded rank::2, rows gathered in example order) give exactly the
    single-process result."""
    import torch.multiprocessing as mp
    from d3d_b200.pruning.__main__ import main
    save_model(_model(), tmp_path / "parent")
    save_model(_model(seed=9), tmp_path / "parent_b")
    _write_examples(tmp_path / "ex.jsonl", 5)
    main(["select", "--parent", str(tmp_path / "parent"), "--examples", str(tmp_path / "ex.jsonl"), "--output-dir",
          str(tmp_path / "sel1"), "--expected-samples", "5", "--block-size", "8", "--devices", "cpu", "--dtype",
          "fp32", "--bootstrap-samples", "50"])
    main(["choose", "--checkpoints", str(tmp_path / "parent"), str(tmp_path / "parent_b"), "--examples",
          str(tmp_path / "ex.jsonl"), "--output-dir", str(tmp_path / "best1"), "--expected-samples", "5",
          "--block-size", "8", "--devices", "cpu", "--dtype", "fp32"])
    mp.spawn(_select_worker, args=(_port(), str(tmp_path)), nprocs=2, join=True)
    one = json.loads((tmp_path / "sel1" / "selection.json").read_text())
    two = json.loads((tmp_path / "sel2" / "selection.json").read_text())
    for d in (one, two):
        d.pop("elapsed_seconds")
    assert one == two
    b1 = json.loads((tmp_path / "best1" / "selected_checkpoint.json").read_text())
    b2 = json.loads((tmp_path / "best2" / "selected_checkpoint.json").read_text())
    assert b1 == b2


def _recovery_worker(rank, port, root, tag, extra):
    import os
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from d3d_b200.pruning.__main__ import main
    try:
        main(["train", "--student", f"{root}/child", "--dataset", f"{root}/data.jsonl", "--output-dir",
              f"{root}/{tag}", "--gradient-accumulation-steps", "1", "--device", "cpu",
              "--anchors-per-example", "4", "--learning-rate", "1e-3", "--min-lr", "1e-4"] + extra)
    except RuntimeError as e:
        (__import__("pathlib").Path(root) / f"{tag}.err{rank}").write_text(str(e))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _child(tmp_path):
    save_model(_model(), tmp_path / "parent")
    prune_checkpoint(tmp_path / "parent", tmp_path / "child", removed=1, block_size=8)


def test_distributed_recovery_fails_together_when_data_runs_out(tmp_path):
    """Two gloo ranks and a window with no spare candidates (multiplier 1)
    over rows of which half are too short to hold a block: a rank runs out,
    and both ranks stop with the same error before any collective of the
    failing step."""
    import torch.multiprocessing as mp
    _child(tmp_path)
    rng = random.Random(5)
    rows = [json.dumps({"prompt_ids": [rng.randrange(2, 1000) for _ in range(10)],
                        "response_ids": [rng.randrange(2, 1000) for _ in range(20 if i % 2 else 3)]})
            for i in range(6)]
    (tmp_path / "data.jsonl").write_text("\n".join(rows) + "\n")
    # (the block size comes from the child's layer_prune.json)
    extra = ["--max-steps", "4", "--candidate-multiplier", "1", "--save-steps", "1"]
    mp.spawn(_recovery_worker, args=(_port(), str(tmp_path), "run", extra), nprocs=2, join=True)
    errs = [(tmp_path / f"run.err{r}").read_text() for r in (0, 1)]
    assert all("ran out" in e for e in errs) and errs[0] == errs[1]
    assert not (tmp_path / "run" / "training_summary.json").exists()


def test_recovery_with_sharded_layers_equals_replicated(tmp_path):
    """Recovery of the pruned child with its decoder layers sharded over two
    gloo ranks (``--fsdp``) ends with the same weights and log as the
    replicated run."""
    import torch.multiprocessing as mp
    _child(tmp_path)
    _write_rows(tmp_path / "data.jsonl", 8, seed=3)
    base = ["--max-steps", "3", "--save-steps", "3", "--optimizer", "adamw"]
    for tag, extra in (("rep", base), ("fsdp", base + ["--fsdp"])):
        mp.spawn(_recovery_worker, args=(_port(), str(tmp_path), tag, extra), nprocs=2, join=True)
    la = [json.loads(x) for x in (tmp_path / "rep" / "training_metrics.jsonl").read_text().splitlines()]
    lb = [json.loads(x) for x in (tmp_path / "fsdp" / "training_metrics.jsonl").read_text().splitlines()]
    assert len(la) == len(lb) == 3
    for x, y in zip(la, lb):
        assert abs(x["loss"] - y["loss"]) <= 1e-5 * max(1.0, abs(x["loss"]))
    ma, mb = load_model(tmp_path / "rep" / "step-3"), load_model(tmp_path / "fsdp" / "step-3")
    sa, sb = dict(ma.named_parameters()), dict(mb.named_parameters())
    assert sa.keys() == sb.keys()
    # Adam divides by sqrt(v) + eps: gradients near eps turn reduction-order
    # rounding into update differences of a few 1e-6 at this learning rate
    for n in sa:
        torch.testing.assert_close(sb[n], sa[n], rtol=1e-5, atol=1e-5, msg=n)


def test_eight_bit_moments_track_fp32_adam():
    """The 8-bit moment codes round-trip within their companding error, and
    AdamW with 8-bit moments reaches the fp32 optimum of a quadratic."""
    from d3d_b200.train.optim import (ShardedAdamW, dequantize_positive, dequantize_signed, quantize_positive,
                                      quantize_signed)
    torch.manual_seed(0)
    x = torch.randn(3000) * torch.logspace(-6, 0, 3000)
    y = dequantize_signed(*quantize_signed(x))
    big = x.abs() > 1e-2 * x.abs().max()
    assert ((y - x).abs() / x.abs())[big].max() < 0.2
    v = torch.rand(3000) * torch.logspace(-10, 0, 3000)
    w = dequantize_positive(*quantize_positive(v))
    assert (w[v > 0] > 0).float().mean() > 0.5
    A = torch.randn(64, 64)
    A = A @ A.t() / 64 + 0.1 * torch.eye(64)
    b = torch.randn(64)
    final = {}
    for bits in (32, 8):
        p = torch.nn.Parameter(torch.zeros(64))
        opt = ShardedAdamW([p], lr=0.05, state_bits=bits)
        for _ in range(300):
            loss = 0.5 * p @ A @ p - b @ p
            p.grad = None
            loss.backward()
            opt.step()
        final[bits] = float(loss.detach())
    assert abs(final[8] - final[32]) < 1e-2 * abs(final[32])
    sd = opt.state_dict()
    q = torch.nn.Parameter(torch.zeros(64))
    o2 = ShardedAdamW([q], lr=0.05, state_bits=8)
    o2.load_state_dict(sd)
    assert o2.step_count == 300
    with pytest.raises(ValueError):
        ShardedAdamW([q], state_bits=8, offload=True)


def test_recovery_losses_under_bf16_autocast():
    """The recovery objective runs under bf16 autocast with a bf16 teacher and
    an fp32 student (the GPU configuration) and stays close to fp32."""
    from d3d_b200.pruning.recovery import make_student, recovery_losses
    from d3d_b200.train.blocks import build_packed_block_batch, synthetic_examples
    parent = _model()
    student = make_student(parent, 1)
    exs = synthetic_examples(1, 48, 0.25, 1000, random.Random(4))
    batch = build_packed_block_batch(exs, block_size=8, mask_token_id=int(parent.cfg.mask_token_id), max_anchors=3,
                                     rng=random.Random(0), full_blocks=True)
    plen = torch.tensor([len(exs[0].prompt_ids)])
    ref = recovery_losses(student, parent, [0, 2, 3], batch, plen)
    teacher16 = _model().to(torch.bfloat16)
    with torch.autocast("cpu", dtype=torch.bfloat16):
        got = recovery_losses(student, teacher16, [0, 2, 3], batch, plen)
    loss = sum(got[k] for k in ("autoregressive_loss", "cross_entropy", "kl", "hidden"))
    loss.backward()
    assert all(p.grad is None or torch.isfinite(p.grad).all() for p in student.parameters())
    for k in ("autoregressive_loss", "cross_entropy"):
        g, r = float(got[k].detach()), float(ref[k].detach())
        assert abs(g - r) < 0.05 * abs(r) + 0.05, k
