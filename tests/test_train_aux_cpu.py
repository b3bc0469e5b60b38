"""Auxiliary training objectives and hidden-trajectory distillation (CPU):
closed forms of the hard-negative CE and margin losses, the trajectory
selection and relation loss, and a trainer run with every option on."""
import math

import torch


def test_hard_negative_ce_and_margin_closed_forms():
    from d3d_b200.train.losses import ce_aux_per_token, hard_negative_ce_per_token, target_margin_per_token
    z = torch.tensor([[2.0, 1.0, 0.5, -1.0], [0.0, 3.0, 2.5, 1.0]])
    y = torch.tensor([0, 2])
    hn = hard_negative_ce_per_token(z, y, top_k=2, margin=0.0)
    want0 = math.log(1 + math.exp(1.0 - 2.0) + math.exp(0.5 - 2.0))
    want1 = math.log(1 + math.exp(3.0 - 2.5) + math.exp(1.0 - 2.5))
    assert torch.allclose(hn, torch.tensor([want0, want1]), atol=1e-6)
    # with every competitor included it equals plain CE
    full = hard_negative_ce_per_token(z, y, top_k=3)
    assert torch.allclose(full, torch.nn.functional.cross_entropy(z, y, reduction="none"), atol=1e-6)
    mg = target_margin_per_token(z, y, top_k=1, margin=1.0, smooth=False)
    assert torch.allclose(mg, torch.tensor([max(0.0, 1.0 - 2.0 + 1.0), max(0.0, 3.0 - 2.5 + 1.0)]))
    tot, ce, h2, m2 = ce_aux_per_token(z, y, ce_weight=1.0, hnce_weight=0.5, hnce_top_k=2, margin_weight=2.0,
                                       margin_top_k=1, margin_smooth=False)
    assert torch.allclose(tot, ce + 0.5 * h2 + 2.0 * m2)


def test_trajectory_selection_and_relation_loss():
    from d3d_b200.train import trajectory as T
    pred = torch.tensor([[[1, 2, 3], [1, 9, 3]]])
    tgt = torch.tensor([[[1, 2, 3], [1, 2, 3]]])
    valid = torch.ones_like(pred, dtype=torch.bool)
    acc = T.block_accept_lengths(pred, tgt, valid)
    assert acc.tolist() == [[3, 1]]
    sel = T.selection_mask(torch.tensor([[3, 3]]), acc, torch.tensor([[3, 3]]), torch.tensor([[True, True]]))
    assert sel.tolist() == [[True, True]]          # both full; teacher better
    h = torch.randn(1, 2, 4, 8)
    valid4 = torch.ones(1, 2, 4, dtype=torch.bool)
    loss, cnt = T.relational_loss(h, h * 3.0, valid4, sel)   # same directions -> same relations
    assert cnt == 2 and float(loss) < 1e-6
    loss2, _ = T.relational_loss(h, torch.randn(1, 2, 4, 16), valid4, sel)
    assert float(loss2) > 0
    assert float(T.distributed_block_mean(loss2, 4.0, 2)) == float(loss2) * 0.5


def test_trainer_with_aux_and_trajectory(tmp_path):
    from d3d_b200.train.args import parser as build_parser
    from d3d_b200.train.trainer import train
    args = build_parser().parse_args([
        "--draft-model", "tiny-drafter", "--target-model", "tiny-target", "--output-dir", str(tmp_path),
        "--max-steps", "2", "--batch-size", "2", "--seq-len", "64", "--device", "cpu", "--dtype", "fp32",
        "--hnce-weight", "0.5", "--margin-weight", "0.5", "--trajectory-weight", "1.0", "--ar-weight", "0.5",
        "--parallel-anchors-per-example", "4", "--vocab-chunk", "256"])
    out = train(args)
    assert len(out["log"]) == 2 and all(math.isfinite(r["loss"]) for r in out["log"])


def _rows_file(path, n, seed=0):
    import json
    import random
    rng = random.Random(seed)
    path.write_text("\n".join(json.dumps({"prompt_ids": [rng.randrange(2, 1000) for _ in range(8)],
                                          "response_ids": [rng.randrange(2, 1000) for _ in range(24)]})
                              for _ in range(n)) + "\n")


def _run(tmp_path, tag, extra):
    from d3d_b200.train.args import parser as build_parser
    from d3d_b200.train.trainer import train
    base = ["--draft-model", "tiny-drafter", "--target-model", "tiny-target", "--output-dir", str(tmp_path / tag),
            "--device", "cpu", "--dtype", "fp32", "--block-size", "8", "--parallel-anchors-per-example", "3",
            "--vocab-chunk", "256", "--lr", "1e-4", "--warmup-steps", "0", "--save-every", "0"]
    return train(build_parser().parse_args(base + extra))


def test_schedule_from_epochs_micro_steps_and_accumulation(tmp_path):
    """Without --max-steps the run length follows the data: epochs x rows per
    micro-step batch, capped by --max-micro-steps, over the accumulation."""
    import json
    import pytest
    _rows_file(tmp_path / "d.jsonl", 6)
    d = str(tmp_path / "d.jsonl")
    r = _run(tmp_path, "ep", ["--data-path", d, "--epochs", "2", "--gradient-accumulation-steps", "3"])
    assert r["steps"] == 4 and len(r["log"]) == 4                  # 2 x 6 micro-steps / 3
    r = _run(tmp_path, "cap", ["--data-path", d, "--epochs", "2", "--max-micro-steps", "5"])
    assert r["steps"] == 5
    assert any((tmp_path / "cap" / "tensorboard").glob("events.out.tfevents.*"))
    r = _run(tmp_path, "acc", ["--data-path", d, "--max-steps", "2", "--gradient-accumulation-steps", "2",
                               "--save-final"])
    st = json.loads(next((tmp_path / "acc").glob("step_*/trainer_state.json")).read_text())
    assert st["data_cursor"] == 4 and st["step"] == 2               # 2 steps x 2 micro-steps x 1 row
    with pytest.raises(ValueError, match="synthetic"):
        _run(tmp_path, "syn", ["--seq-len", "64"])


def test_inline_packing_equals_prefetch_threads(tmp_path):
    _rows_file(tmp_path / "d.jsonl", 4, seed=1)
    d = str(tmp_path / "d.jsonl")
    a = _run(tmp_path, "w0", ["--data-path", d, "--max-steps", "2", "--workers", "0"])
    b = _run(tmp_path, "w2", ["--data-path", d, "--max-steps", "2", "--workers", "2", "--prefetch", "3"])
    assert [x["loss"] for x in a["log"]] == [x["loss"] for x in b["log"]]


def test_reverse_kl_objective_and_chunked_loss(tmp_path):
    import torch
    from d3d_b200.train.losses import reverse_kl_per_token
    from d3d_b200.train.trainer import _reverse_kl
    torch.manual_seed(0)
    hs, ht = torch.randn(300, 16, requires_grad=True), torch.randn(300, 16)
    ws, wt = torch.randn(50, 16), torch.randn(50, 16)
    w = torch.rand(300)
    got = _reverse_kl(hs, ws, ht, wt, w, rows=64)
    ref = (w * reverse_kl_per_token(hs @ ws.t(), ht @ wt.t())).sum()
    assert torch.allclose(got, ref, rtol=1e-5)
    got.backward()
    assert torch.isfinite(hs.grad).all()
    r = _run(tmp_path, "rkl", ["--objective", "rkl", "--max-steps", "2", "--seq-len", "64", "--batch-size", "2"])
    assert all(x["loss"] > 0 for x in r["log"])
    import pytest
    with pytest.raises(ValueError, match="needs --target-model"):
        from d3d_b200.train.args import parser as build_parser
        from d3d_b200.train.trainer import train
        train(build_parser().parse_args(["--draft-model", "tiny-drafter", "--output-dir", str(tmp_path / "x"),
                                         "--objective", "forward_kl", "--max-steps", "1", "--device", "cpu"]))


def test_trajectory_probe_shuffle_and_separate_teacher(tmp_path):
    import math
    r = _run(tmp_path, "traj", ["--max-steps", "2", "--seq-len", "64", "--batch-size", "2",
                                "--trajectory-weight", "1.0", "--trajectory-gradient-probe-steps", "1",
                                "--trajectory-shuffle-teacher-blocks", "--trajectory-teacher-model", "tiny-target",
                                "--margin-weight", "0.5", "--margin-smooth", "--fsdp-cpu-offload"])
    first, second = r["log"]
    assert "trajectory_grad_norm" in first and "trajectory_grad_norm" not in second
    assert math.isfinite(first["ce_grad_norm"]) and first["ce_grad_norm"] > 0


def test_shuffle_among_equal_length_keeps_groups():
    import torch
    from d3d_b200.train.trajectory import shuffle_among_equal_length
    rt = torch.arange(6, dtype=torch.float32).view(1, 6, 1, 1).expand(1, 6, 2, 2).contiguous()
    sel = torch.tensor([[True, True, True, False, True, True]])
    ln = torch.tensor([[3, 3, 5, 3, 5, 3]])
    out = shuffle_among_equal_length(rt, sel, ln, torch.Generator().manual_seed(0))
    ids = out[0, :, 0, 0].long().tolist()
    assert ids[3] == 3                                    # not selected: untouched
    assert sorted(ids[i] for i in (0, 1, 5)) == [0, 1, 5] and sorted(ids[i] for i in (2, 4)) == [2, 4]


def test_random_init_and_mask_token_lookup(tmp_path):
    import json
    import types
    import torch
    from d3d_b200.checkpoint import save_model
    from d3d_b200.config import tiny_drafter
    from d3d_b200.models.qwen3 import build_model
    from d3d_b200.train.args import parser as build_parser
    from d3d_b200.train.trainer import _build, _mask_id
    m = build_model(tiny_drafter(), seed=5)
    save_model(m, tmp_path / "d")
    r = _build(str(tmp_path / "d"), "cpu", torch.float32, seed=11, random_init=True)
    assert not torch.equal(r.model.layers[0].mlp.up_proj.weight, m.model.layers[0].mlp.up_proj.weight)
    assert r.cfg.num_hidden_layers == m.cfg.num_hidden_layers
    tok = types.SimpleNamespace(convert_tokens_to_ids=lambda t: 77 if t == "<MASK>" else 0, unk_token_id=0)
    a = build_parser().parse_args(["--draft-model", str(tmp_path / "d"), "--output-dir", str(tmp_path / "o")])
    assert _mask_id(a, tok) is None                       # the checkpoint names its own mask id
    cfg = json.loads((tmp_path / "d" / "config.json").read_text())
    cfg.pop("mask_token_id")
    (tmp_path / "d" / "config.json").write_text(json.dumps(cfg))
    assert _mask_id(a, tok) == 77
    a.mask_token_id = 5
    assert _mask_id(a, tok) == 5


def test_training_flag_checks(tmp_path):
    import pytest
    for bad in (["--block-size", "1"], ["--workers", "-1"], ["--min-lr-ratio", "2"], ["--loss-decay-gamma", "0"],
                ["--trajectory-shuffle-teacher-blocks"], ["--trajectory-gradient-probe-steps", "2"]):
        with pytest.raises(ValueError):
            _run(tmp_path, "bad", ["--max-steps", "1", "--seq-len", "64"] + bad)
    _run(tmp_path, "ok", ["--max-steps", "1", "--seq-len", "64"])
    import json
    assert json.loads((tmp_path / "ok" / "args.json").read_text())["world_size"] == 1
