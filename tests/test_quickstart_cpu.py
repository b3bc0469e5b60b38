"""The ready-made runs: every command line a recipe builds parses with the
parser of the entry point it calls (so a renamed flag breaks here), later
flags are appended, and the import half of the smoke check passes."""
import pytest


def _after(cmd, module):
    return cmd[cmd.index(module) + 1:]


def test_recipes_parse_with_their_entry_points(monkeypatch):
    from d3d_b200.cli import quickstart as q
    from d3d_b200.cli import serve, single
    from d3d_b200.pruning.__main__ import parser as prune_parser
    from d3d_b200.train.args import parser as train_parser
    monkeypatch.setenv("DATASETS", "gsm8k math500")
    monkeypatch.setenv("CONCURRENCY", "1")
    (cmd,) = q.plan("single", ["--max-new-tokens", "64"])
    a = single.parser().parse_args(_after(cmd, "d3d_b200.cli.single"))
    assert a.max_new_tokens == 64 and a.draft_device == "cuda:1" and a.anchor_num == 3
    (cmd,) = q.plan("concurrent", [])
    a = serve.parser().parse_args(_after(cmd, "d3d_b200.cli.serve"))
    assert a.concurrency == "1" and a.anchor_num == 3 and a.datasets == ["math500"]
    cmds = q.plan("benchmark", [])
    assert [single.parser().parse_args(_after(c, "d3d_b200.cli.single")).dataset for c in cmds] == ["gsm8k",
                                                                                                     "math500"]
    (cmd,) = q.plan("train", ["--max-steps", "3"])
    a = train_parser().parse_args(_after(cmd, "d3d_b200.train"))
    assert a.gradient_accumulation_steps == 8 and a.ar_weight == 1.0 and a.max_steps == 3
    assert cmd[cmd.index("--nproc-per-node") + 1] == "4"
    (cmd,) = q.plan("prune", ["prune", "--selection", "s.json", "--output", "o"])
    assert prune_parser().parse_args(_after(cmd, "d3d_b200.pruning")).stage == "prune"
    (cmd,) = q.plan("prune", ["train", "--student", "c", "--dataset", "d", "--output-dir", "o", "--max-steps", "1"])
    assert "torch.distributed.run" in cmd
    with pytest.raises(SystemExit):
        q.plan("prune", ["bogus"])
    with pytest.raises(SystemExit):
        q.plan("nothing", [])


def test_smoke_imports_every_module():
    from d3d_b200.cli import quickstart as q
    q.smoke(require_gpus=0)
