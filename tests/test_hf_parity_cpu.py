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
