"""Synchronous multi-step denoising decode (oracle path): greedy output is
token-identical to target-only AR decoding for every schedule/remasking mode,
with and without KV caches; sampling runs end to end."""
import random

import pytest
import torch

from d3d_b200.config import tiny_drafter, tiny_target
from d3d_b200.engine.backends import TorchTarget
from d3d_b200.engine.spec import ar_generate
from d3d_b200.engine.sync import (num_transfer_tokens, select_transfer, sync_generate,
                                  sync_generate_nocache)
from d3d_b200.models.qwen3 import build_model


@pytest.fixture(scope="module")
def pair():
    return build_model(tiny_target(), seed=0), build_model(tiny_drafter(cond=True), seed=1)


def _prompts(n=3, seed=2):
    rng = random.Random(seed)
    return [[rng.randrange(2, 1000) for _ in range(rng.randint(10, 40))] for _ in range(n)]


def test_transfer_schedule():
    assert num_transfer_tokens(15, 4) == [4, 4, 4, 3]
    assert sum(num_transfer_tokens(7, 3)) == 7
    block = torch.tensor([[5, 9, 9, 9]])
    x0 = torch.tensor([[5, 1, 2, 3]])
    p = torch.tensor([[0.0, 0.2, 0.9, 0.5]])
    select_transfer(block, block == 9, x0, p, 2, "low_confidence", 0.9)
    assert block.tolist() == [[5, 9, 2, 3]]
    block = torch.tensor([[5, 9, 9, 9]])
    select_transfer(block, block == 9, x0, p, 3, "dynamic", 0.8)
    assert block.tolist() == [[5, 9, 2, 9]]


@pytest.mark.parametrize("steps,remask,mode", [(1, "low_confidence", "block_causal"),
                                               (2, "low_confidence", "causal"),
                                               (3, "dynamic", "block_causal")])
def test_sync_matches_ar(pair, steps, remask, mode):
    t, d = pair
    d.cfg.mask_token_id = 1023
    prompts = _prompts()
    ar = ar_generate(TorchTarget(t), prompts, 24, ignore_eos=True)["outputs"]
    for p, ref in zip(prompts, ar):
        st = sync_generate(t, d, p, 24, block_size=8, denoising_steps=steps, remasking=remask, mode=mode)
        assert st.output_tokens == ref
        assert sum(st.acceptance_lengths) >= 24
        nc = sync_generate_nocache(t, d, p, 24, block_size=8, denoising_steps=steps, remasking=remask,
                                   mode=mode)
        assert nc.output_tokens == ref


def test_sync_sampling_runs(pair):
    t, d = pair
    st = sync_generate(t, d, _prompts(1)[0], 20, block_size=8, temperature=0.7, top_k=20, seed=3)
    assert len(st.output_tokens) == 20


def test_sync_cli_tiny_pair(tmp_path):
    """The synchronous denoising CLI end to end on the tiny pair, cached and
    uncached, with the AR baseline and its JSON summary."""
    import json
    from d3d_b200.cli import sync
    for extra in ([], ["--no-kvcache"]):
        out = tmp_path / f"sync{len(extra)}.json"
        rows = sync.main(["--verifier", "tiny-target", "--drafter", "tiny-drafter", "--device", "cpu",
                          "--max-new-tokens", "10", "--block-size", "4", "--denoising-steps", "2",
                          "--max-samples", "2", "--prompt-min", "6", "--prompt-max", "12", "--baseline",
                          "--output-json", str(out)] + extra)
        assert len(rows) == 2 and all(r["tokens"] for r in rows)
        d = json.loads(out.read_text())
        assert len(d["rows"]) == 2 and "config" in d
