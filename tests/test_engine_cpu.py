"""CPU oracle tests of the async speculative decoder: greedy output must be
token-identical to target-only AR decoding (tiny pair, fp32)."""
import random

import pytest
import torch

from d3d_b200.config import tiny_drafter, tiny_target
from d3d_b200.engine.backends import TorchDraft, TorchTarget
from d3d_b200.engine.controlled import ControlledAcceptance, expected_commit, rate_for_mean_accept
from d3d_b200.engine.spec import DecodeConfig, SpecDecoder, ar_generate
from d3d_b200.models.qwen3 import build_model


def _prompts(n=4, seed=0, lo=16, hi=64, vocab=1000):
    rng = random.Random(seed)
    return [[rng.randrange(2, vocab) for _ in range(rng.randint(lo, hi))] for _ in range(n)]


@pytest.fixture(scope="module")
def pair():
    torch.manual_seed(0)
    t = build_model(tiny_target(), seed=0)
    d = build_model(tiny_drafter(), seed=1)
    return t, d


@pytest.mark.parametrize("mode,anchors,conc", [("causal", 1, 1), ("block_causal", 3, 2),
                                               ("causal", 0, 4)])
def test_spec_matches_ar(pair, mode, anchors, conc):
    t, d = pair
    prompts = _prompts()
    ar = ar_generate(TorchTarget(t), prompts, max_new_tokens=32, ignore_eos=True)
    cfg = DecodeConfig(block_size=8, anchor_num=anchors, attention_mask_mode=mode,
                       max_new_tokens=32, ignore_eos=True)
    res = SpecDecoder(TorchTarget(t), TorchDraft(d), cfg).generate(prompts, concurrency=conc)
    for o, ref in zip(res["outputs"], ar["outputs"]):
        assert o.tokens == ref
        assert sum(o.accepts) >= len(o.tokens) - 1


def test_controlled_acceptance_matches_ar_and_rate(pair):
    t, d = pair
    prompts = _prompts(n=3, seed=3)
    ar = ar_generate(TorchTarget(t), prompts, max_new_tokens=48, ignore_eos=True)
    rate = rate_for_mean_accept(4.0, 8)
    assert abs(expected_commit(rate, 8) - 4.0) < 1e-6

    def ctl(i):
        return ControlledAcceptance(oracle=prompts[i] + ar["outputs"][i], rate=rate,
                                    vocab_size=1024, seed=7, stream=i, exclude=(1023,))

    cfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=48, ignore_eos=True)
    res = SpecDecoder(TorchTarget(t), TorchDraft(d), cfg).generate(prompts, controlled=ctl)
    for o, ref in zip(res["outputs"], ar["outputs"]):
        assert o.tokens == ref
    # every corrupted position is offered as the first alternative → anchors hit
    hits = sum(o.hits for o in res["outputs"])
    assert hits > 0
    assert res["mean_accept_length"] > 2.0


def test_sampling_runs(pair):
    t, d = pair
    prompts = _prompts(n=2, seed=5)
    cfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=24, ignore_eos=True,
                       temperature=0.8, top_k=8)
    res = SpecDecoder(TorchTarget(t, temperature=0.8, top_k=0, seed=1), TorchDraft(d, seed=2),
                      cfg).generate(prompts)
    for o in res["outputs"]:
        assert len(o.tokens) == 24
        assert all(0 <= x < 1024 for x in o.tokens)


def test_gate_up_interleave_order():
    """The interleaved gate|up row order is a permutation that puts gate row
    64t+16w+j and its up row in lanes j and j+16 of warp w of tile t."""
    from d3d_b200 import ops
    i = 384
    order = ops.gate_up_order(i)
    assert sorted(order.tolist()) == list(range(2 * i))
    for t in range(2 * i // 128):
        for w in range(4):
            for j in range(16):
                r = 128 * t + 32 * w + j
                assert order[r] == 64 * t + 16 * w + j
                assert order[r + 16] == i + 64 * t + 16 * w + j
    g = torch.randn(i, 64).to(torch.bfloat16)
    u = torch.randn(i, 64).to(torch.bfloat16)
    pw = ops.pack_gate_up(g, u)
    full = torch.cat([g, u], 0)
    assert torch.equal(pw.unpack(), full[order])
