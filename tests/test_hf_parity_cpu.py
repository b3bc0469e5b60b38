"""Parity with the Hugging Face Qwen3 implementation the reference validates
against (``serving/bench.py:88-109``): checkpoints written here load in
``transformers`` unchanged, give the same logits, and greedy decoding through
this framework's AR path equals ``generate``."""
import torch

from d3d_b200.checkpoint import save_model
from d3d_b200.config import tiny_target
from d3d_b200.engine.backends import TorchTarget
from d3d_b200.engine.spec import ar_generate
from d3d_b200.models.qwen3 import build_model


def test_logits_and_greedy_match_transformers(tmp_path):
    import transformers
    m = build_model(tiny_target(), seed=0)
    save_model(m, tmp_path / "t")
    hf = transformers.AutoModelForCausalLM.from_pretrained(str(tmp_path / "t"), dtype=torch.float32).eval()
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(2, 1000, (2, 23), generator=g)
    with torch.no_grad():
        torch.testing.assert_close(m.logits(m(ids)), hf(ids).logits, rtol=1e-5, atol=1e-5)
    prompts = [ids[0].tolist(), ids[1, :11].tolist()]
    ours = ar_generate(TorchTarget(m), prompts, 16, ignore_eos=True)["outputs"]
    for p, o in zip(prompts, ours):
        with torch.no_grad():
            ref = hf.generate(torch.tensor([p]), max_new_tokens=16, do_sample=False, min_new_tokens=16,
                              pad_token_id=0)[0, len(p):].tolist()
        assert o == ref


def test_serve_cli_validates_against_transformers(tmp_path):
    from d3d_b200.cli import serve
    save_model(build_model(tiny_target(), seed=0), tmp_path / "t")
    rows = serve.main(["--target", str(tmp_path / "t"), "--draft", "tiny-drafter", "--device", "cpu",
                       "--pages", "256", "--concurrency", "2", "--max-new-tokens", "12", "--block-size", "8",
                       "--max-samples", "2", "--prompt-min", "8", "--prompt-max", "14", "--ignore-eos",
                       "--validate-hf"])
    hf = rows[0]["hf_greedy"]
    assert hf["identical"] == hf["requests"] == 2 and hf["first_divergence"] == [None, None]


def test_ar_baseline_cli_validation_retests_and_records(tmp_path):
    """The AR baseline CLI: transformers validation passes, every attempt is
    recorded with telemetry, a strict slow fraction forces the retest, and
    the summary and table cover each concurrency."""
    import json
    from d3d_b200.cli import baseline
    save_model(build_model(tiny_target(), seed=0), tmp_path / "t")
    out = baseline.main(["--target", str(tmp_path / "t"), "--device", "cpu", "--datasets", "synthetic",
                         "--concurrency", "1", "2", "--max-new-tokens", "6", "--warmup-new-tokens", "2",
                         "--max-samples", "3", "--prompt-min", "8", "--prompt-max", "14", "--ignore-eos",
                         "--repeats", "2", "--max-retests", "1", "--slow-fraction", "0.999999",
                         "--pages", "64", "--run-id", "r1", "--output-root", str(tmp_path / "res")])
    d = tmp_path / "res" / "synthetic" / "r1"
    bench = json.loads((d / "benchmark.json").read_text())
    assert bench["status"] == "complete" and bench["validation"] == "passed"
    assert all(c["equal"] for c in json.loads((d / "validation.json").read_text()))
    for c in ("1", "2"):
        s = bench["summary"][c]
        assert s["attempts"] in (2, 3) and s["min_tps"] <= s["median_tps"] <= s["max_tps"]
    raw = json.loads((d / "c2_attempt0.json").read_text())
    assert raw["max_active"] <= 2 and len(raw["outputs"]) == 3 and all(len(o) == 6 for o in raw["outputs"])
    assert raw["length_limit_fraction"] == 1.0 and "telemetry_before" in raw
    assert "| 2 |" in (d / "table.md").read_text()
    assert out["synthetic"]["requests"] == 3
    assert baseline.slow_attempts([{"attempt": 0, "tps": 10.0}, {"attempt": 1, "tps": 5.0}], 0.85) == [1]
    assert baseline.slow_attempts([{"attempt": i, "tps": t} for i, t in enumerate((10.0, 9.0, 2.0))], 0.85) == [2]


def test_ar_baseline_fixed_batch_mode(tmp_path):
    import json
    from d3d_b200.cli import baseline
    out = baseline.main(["--target", "tiny-target", "--device", "cpu", "--datasets", "synthetic", "--max-samples", "2",
                         "--prompt-min", "8", "--prompt-max", "12", "--batch-sizes", "1", "3", "--max-new-tokens", "5",
                         "--repeats", "1", "--pages", "64", "--run-id", "fb", "--output-root", str(tmp_path)])
    cells = out["synthetic"]["cells"]
    assert [(c["batch_size"], c["tokens"]) for c in cells] == [(1, 5), (3, 15)]
    assert json.loads((tmp_path / "synthetic" / "fb" / "benchmark.json").read_text())["status"] == "complete"
