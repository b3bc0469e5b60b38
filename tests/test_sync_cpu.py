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
    for run in (sync_generate, sync_generate_nocache):
        st = run(t, d, _prompts(1)[0], 20, block_size=8, temperature=0.7, top_k=20, target_top_k=50,
                 target_top_p=0.9, seed=3, collect_stage_timings=True)
        assert len(st.output_tokens) == 20
        assert len(st.stage_records) == len(st.acceptance_lengths) == len(st.draft_blocks)
        assert [r["accept_length"] for r in st.stage_records] == st.acceptance_lengths
        assert sum(len(e) for e in st.emitted_blocks) >= 20
        assert st.stage_records[-1]["generated_len_after"] >= 20


def test_sync_stop_tokens(pair):
    """Decoding ends at the first stop token, which is kept."""
    t, d = pair
    d.cfg.mask_token_id = 1023
    p = _prompts(1)[0]
    full = sync_generate(t, d, p, 24, block_size=8).output_tokens
    stop = full[9]
    first = full.index(stop)
    for run in (sync_generate, sync_generate_nocache):
        st = run(t, d, p, 24, block_size=8, stop_ids=[stop])
        assert st.output_tokens == full[:first + 1] and st.stopped[-1]


def test_dense_pq_acceptance_is_lossless():
    """The first committed token after a drafted position follows the
    target distribution whatever the proposal (``pq_accept_dense``)."""
    from d3d_b200.engine.sync import pq_accept_dense
    torch.manual_seed(0)
    V, n = 6, 20000
    p = torch.softmax(torch.randn(2, V) * 1.5, -1)
    q = torch.softmax(torch.randn(1, V) * 1.5, -1)
    g = torch.Generator().manual_seed(1)
    counts = torch.zeros(V)
    for _ in range(n):
        draft = torch.multinomial(q[0], 1, generator=g).view(1, 1)
        acc, corr = pq_accept_dense(draft, p[None], q[None], g)
        counts[int(draft[0, 0]) if acc == 1 else int(corr[0])] += 1
    assert (counts / n - p[0]).abs().max() < 0.015


def test_eager_attention_matches_sdpa(pair):
    t, _ = pair
    x = torch.randint(2, 900, (2, 19))
    try:
        a = t(x)
        assert t.set_attn_implementation("eager") == "eager"
        b = t(x)
    finally:
        assert t.set_attn_implementation("flash_attention_2") == "sdpa"
    assert (a - b).abs().max() < 1e-4
    with pytest.raises(ValueError):
        t.set_attn_implementation("xformers")


def test_sync_cli_tiny_pair(tmp_path):
    """The synchronous denoising CLI end to end on the tiny pair, cached and
    uncached, with the AR baseline and its JSON summary."""
    import json
    from d3d_b200.cli import sync
    for extra in ([], ["--no-kvcache", "--collect-stage-timings", "--target-attn-implementation", "eager"]):
        out = tmp_path / f"sync{len(extra)}.json"
        rows = sync.main(["--verifier", "tiny-target", "--drafter", "tiny-drafter", "--device", "cpu",
                          "--max-new-tokens", "10", "--block-size", "4", "--denoising-steps", "2",
                          "--max-samples", "2", "--prompt-min", "6", "--prompt-max", "12", "--baseline",
                          "--dtype", "fp32", "--output-json", str(out)] + extra)
        assert len(rows) == 2 and all(r["tokens"] for r in rows)
        assert all(r["matches_ar"] for r in rows)
        d = json.loads(out.read_text())
        assert len(d["rows"]) == 2 and "config" in d and d["summary"]["matches_ar"] is True
        assert d["summary"]["use_kvcache"] is (not extra)
        assert bool(d["rows"][0]["stage_timings"]) is bool(extra)
    # one example by index, sampled with target truncation, a compact summary and a drafter tag
    summ = tmp_path / "compact.json"
    rows = sync.main(["--verifier", "tiny-target", "--drafter", "tiny-drafter", "--device", "cpu",
                      "--draft-device", "cpu", "--verifier-device", "cpu", "--max-new-tokens", "8",
                      "--block-size", "4", "--prompt-min", "6", "--prompt-max", "12", "--sample-index", "3",
                      "--temperature", "0.8", "--proposal-top-p", "0.9", "--target-top-k", "40",
                      "--target-top-p", "0.95", "--eos-token-id", "7", "--draft-tokens", "3",
                      "--drafter-tag", "tiny", "--use-kvcache", "--verbose", "--summary-json", str(summ)])
    assert len(rows) == 1
    c = json.loads(summ.read_text())
    assert c["drafter_tag"] == "tiny" and c["num_prompts"] == 1
    with pytest.raises(SystemExit):
        sync.main(["--verifier", "tiny-target", "--drafter", "tiny-drafter", "--device", "cpu",
                   "--draft-tokens", "0"])
